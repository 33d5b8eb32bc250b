"""Type-3 NUFFT plan (B200 / CUDA): f[k] = sum_j c[j] exp(i*isign s_k . x_j).

Drop-in for mlx_nufft.gpu_t3.GpuT3Plan (exported as Type3Plan; reference
mlx_nufft/gpu_t3.py:287-1364).  The plan sizes the spread grid nf and the
inner FFT grid n_up from the source / target extents exactly as the
reference (centres C, D; half-widths X, S; FINUFFT set_nhg_type3), then runs
prephase+spread (nf grid) -> pad/deconvolve ((-1)^q / phihat) -> cuFFT ->
interp x post on the GPU (libnufft_b200).

Differences from the reference (documented, not silent):
  * dimension is taken from the coordinate tuples (1, 2 or 3); the
    reference embeds 1D/2D problems in 3D with zero coordinates, which
    gives the same transform with w-fold redundant work per missing axis;
  * there is no slab mode: the whole-grid pipeline fits B200 HBM for every
    grid the reference's slab mode targets up to ~2e10 cells, so
    `slab_mode` is always False and `execute_batch` works for every size
    (the reference raises NotImplementedError outside slab mode);
  * the FFT is cuFFT; fft_backend='mlx' (the default name) means cuFFT,
    'vkfft' is rejected (VkFFT is not part of this build);
  * low_mem is accepted and ignored (no host/GPU unified memory to trim).
"""

import numpy as np
import torch

from ._device import as_c64, as_f64, finish, numel
from ._plan import NativePlan
from .sizing import kernel_params

PI = np.pi


class Type3Plan:
    def __init__(self, x, s, eps=1e-5, isign=+1, upsampfac=1.25,
                 prec="crit64", sigma_inner=None, sort_points=True,
                 low_mem=None, source_extent=None, fft_backend="mlx",
                 kerevalmeth=1):
        assert prec in ("fp32", "coords64", "phases64", "crit64")
        assert fft_backend in ("mlx", "cufft", "vkfft")
        if fft_backend == "vkfft":
            raise RuntimeError("fft_backend='vkfft' is not available: this "
                               "build uses cuFFT for every fine-grid FFT")
        self.fft_backend = "cufft"
        self.prec = prec
        self.isign = +1 if isign >= 0 else -1   # finufft: non-negative -> +
        self.eps = eps
        self.sigma = upsampfac
        self.w, self.beta = kernel_params(eps, upsampfac)
        xs = tuple(x) if not isinstance(x, np.ndarray) or x.ndim != 1 else (x,)
        ss = tuple(s) if not isinstance(s, np.ndarray) or s.ndim != 1 else (s,)
        if len(xs) != len(ss) or not 1 <= len(xs) <= 3:
            raise ValueError("sources and targets need the same number (1-3) "
                             "of coordinate arrays")
        self.dim = len(xs)
        self.low_mem = bool(low_mem) if low_mem is not None else False
        self.slab_mode = False
        self._sort_points = sort_points
        if source_extent is not None:
            source_extent = [(float(lo), float(hi))
                             for lo, hi in list(source_extent)[:self.dim]]
        self._plan = NativePlan(3, self.dim, None, 1, eps, self.isign,
                                upsampfac=upsampfac, sigma_inner=sigma_inner,
                                prec=prec, sort_points=sort_points,
                                source_extent=source_extent,
                                kerevalmeth=kerevalmeth)
        dev = self._plan.device
        xt = [as_f64(v, dev) for v in xs]
        st = [as_f64(v, dev) for v in ss]
        P, M = xt[0].numel(), st[0].numel()
        if P < 1 or M < 1:
            raise ValueError("at least one source and one target are required")
        if any(v.numel() != P for v in xt) or any(v.numel() != M for v in st):
            raise ValueError("coordinate arrays must have equal length")
        self._plan.setpts(P, xt, M, st)
        self.P, self.M = P, M
        inf = self._plan.info()
        self.w2, self.beta2 = inf.w2, inf.beta2
        self.sigma_in = inf.sigma_inner
        self.nf = [int(inf.nf[d]) for d in range(self.dim)]
        self.n_up = [int(inf.n_up[d]) for d in range(self.dim)]
        self.C = [float(inf.C[d]) for d in range(self.dim)]
        self.D = [float(inf.D[d]) for d in range(self.dim)]
        self.gam = [float(inf.gam[d]) for d in range(self.dim)]

    # ------------------------------------------------------------------
    def set_sources(self, x, backend="host"):
        """Re-point the sources against the frozen grids / targets
        (gpu_t3.py:444-506).  Raises ValueError when a source leaves the
        sized extent plus the kernel guard band."""
        if backend not in ("host", "gpu"):
            raise ValueError(f"unknown backend {backend!r}")
        xs = tuple(x) if not isinstance(x, np.ndarray) or x.ndim != 1 else (x,)
        if len(xs) != self.dim:
            raise ValueError(f"expected {self.dim} source coordinate arrays")
        xt = [as_f64(v, self._plan.device) for v in xs]
        P = xt[0].numel()
        if P < 1 or any(v.numel() != P for v in xt):
            raise ValueError("coordinate arrays must be non-empty, equal length")
        self._plan.set_sources(P, xt)
        self.P = P

    def cells(self, which=0):
        """Device geometry (i1, fr, perm) of sources (0) or targets (1)."""
        n = self.P if which == 0 else self.M
        return self._plan.debug_points(which, self.dim, n)

    def _run(self, cs, nvec):
        out = torch.empty((nvec, self.M), dtype=torch.complex64,
                          device=cs.device)
        self._plan.execute(cs, out, nvec)
        return out

    def execute(self, c, return_np=True, out=None):
        assert numel(c) == self.P, \
            f"c.size ({numel(c)}) must equal number of sources ({self.P})"
        cs = as_c64(c, self._plan.device).reshape(-1)
        return finish(self._run(cs, 1)[0], return_np, out)

    def execute_batch(self, cs, return_np=True, out=None):
        """(nch, P) strength channels -> (nch, M) through one batched pass."""
        t = as_c64(cs, self._plan.device)
        if t.dim() != 2:
            raise ValueError("cs must be 2-D (nch, P)")
        assert t.shape[1] == self.P
        return finish(self._run(t.reshape(-1), int(t.shape[0])), return_np, out)

    def execute_profiled(self, c):
        """execute() with per-stage device times in seconds
        (gpu_t3.py:1351-1364)."""
        self._plan.set_profile(True)
        try:
            res = self.execute(c, return_np=False)
            t = self._plan.stage_times()
        finally:
            self._plan.set_profile(False)
        times = {"prephase+spread+pad": t["spread_or_pad"] / 1e3,
                 "fft": t["fft"] / 1e3, "gather": t["interp_or_crop"] / 1e3}
        return res.cpu().numpy(), times


# the reference exports GpuT3Plan as Type3Plan (mlx_nufft/__init__.py:23)
GpuT3Plan = Type3Plan
