"""Type-1 / type-2 NUFFT plans in dimensions 1, 2, 3 (B200 / CUDA).

Drop-in for mlx_nufft.nd (Type1PlanND, Type2PlanND; reference
mlx_nufft/nd.py:386-1119) with the same constructor arguments, defaults,
attributes, methods and error types:

  type 1:  f[k] = sum_j c[j] exp(i*isign * k . x_j)
  type 2:  c[j] = sum_k f[k] exp(i*isign * k . x_j)

modeord=0 mode boxes k_d in [-(N_d//2), (N_d-1)//2] (even or odd N_d); x in
[-pi, pi)^d, any value accepted and folded mod 2pi in fp64 ('crit64').

All geometry work (fold, cell/fraction split, bin sort, subproblem tables)
and every execute stage runs in libnufft_b200 on the GPU; this module only
validates arguments, moves data to the device and shapes results.
Results are numpy arrays (return_np=True, the default) or torch CUDA tensors
(return_np=False, where the reference returns an mx.array).
"""

import numpy as np
import torch

from ._device import as_c64, as_f64, finish, numel
from ._plan import NativePlan
from .sizing import kernel_ft, kernel_params, next235even

PI = np.pi


def _coords_tuple(x):
    if isinstance(x, (np.ndarray, torch.Tensor)) and x.ndim == 1:
        return (x,)
    return tuple(x)


class _PointsND:
    """Shared point/mode setup for ND types 1 and 2 (nd.py:94-150)."""

    _TYPE = 0

    def __init__(self, x, n_modes, eps, isign, upsampfac, prec, sort_points,
                 spread_method, kerevalmeth=1):
        if prec not in ("fp32", "crit64"):
            raise ValueError("prec must be 'fp32' or 'crit64'")
        x = _coords_tuple(x)
        self.dim = len(x)
        if self.dim not in (1, 2, 3):
            raise ValueError("dims 1, 2, 3 supported")
        if np.isscalar(n_modes):
            n_modes = (int(n_modes),) * self.dim
        self.N = tuple(int(n) for n in n_modes)
        if len(self.N) != self.dim:
            raise ValueError(f"n_modes length {len(self.N)} must match "
                             f"dim {self.dim}")
        if any(n < 1 for n in self.N):
            raise ValueError("mode dims must be >= 1")
        if upsampfac in (None, 0, 0.0):       # finufft auto sentinel
            upsampfac = 2.0
        if not 1.0 < upsampfac <= 4.0:
            raise ValueError(f"upsampfac must be in (1, 4], got {upsampfac}")
        if spread_method not in ("auto", "od", "gm"):
            raise AssertionError(f"unknown spread_method {spread_method!r}")
        self.prec = prec
        self.isign = +1 if isign >= 0 else -1
        self.eps = eps
        self.sigma = upsampfac
        self.w, self.beta = kernel_params(eps, upsampfac)
        self.n_up = [next235even(max(2 * self.w, int(np.ceil(upsampfac * n))))
                     for n in self.N]
        self._sort_points = bool(sort_points)
        self._method = spread_method
        self._plan = NativePlan(self._TYPE, self.dim, self.N, 1, eps,
                                self.isign, upsampfac=upsampfac, prec=prec,
                                method=spread_method, sort_points=sort_points,
                                kerevalmeth=kerevalmeth)
        self._perm_cache = None
        self._set_points(x)

    # -- geometry ----------------------------------------------------------
    def _set_points(self, x):
        dev = self._plan.device
        xs = [as_f64(v, dev) for v in x]
        P = xs[0].numel()
        if P < 1:
            raise ValueError("at least one nonuniform point is required")
        if not all(v.numel() == P for v in xs):
            raise ValueError("coordinate arrays must have equal length")
        self._plan.setpts(P, xs)
        self.P = P
        self._perm_cache = None
        inf = self._plan.info()
        self._od = bool(inf.tiled)
        self.sorted = bool(inf.tiled) or self._sort_points

    @property
    def decs(self):
        """fp64 mode corrections 1/phihat(2 pi k / n_up) per dimension
        (nd.py:140-145; no FFT scale folded in -- cuFFT is unnormalised)."""
        out = []
        for d in range(self.dim):
            k = np.arange(-(self.N[d] // 2), self.N[d] - self.N[d] // 2,
                          dtype=np.float64)
            out.append(1.0 / kernel_ft(2.0 * PI * k / self.n_up[d], self.beta,
                                       self.w))
        return out

    @property
    def perm(self):
        """Plan point order (sorted position -> caller index), numpy."""
        if self._perm_cache is None:
            _, _, perm = self._plan.debug_points(0, self.dim, self.P)
            self._perm_cache = perm
        return self._perm_cache

    def cells(self):
        """(i1, fr, perm) of the plan's points in plan order: the device
        crit64 geometry (nd.py:152-165), i1 normalised so that i1 + w//2 is
        in [0, n_up)."""
        return self._plan.debug_points(0, self.dim, self.P)

    def set_sources(self, x, backend="host"):
        """Re-point the plan to new coordinates, reusing the mode
        corrections, FFT plans and grids (nd.py:627-681).  Both backends run
        the same fp64 device setpts here; `backend` is validated for
        compatibility.  P may change.  Returns self."""
        x = _coords_tuple(x)
        if len(x) != self.dim:
            raise ValueError(f"expected {self.dim} coordinate arrays, "
                             f"got {len(x)}")
        if backend not in ("host", "gpu"):
            raise ValueError(f"unknown backend {backend!r}")
        sizes = [numel(v) for v in x]
        if sizes[0] < 1 or any(s != sizes[0] for s in sizes):
            raise ValueError("coordinate arrays must be non-empty, equal length")
        self._set_points(x)
        return self

    def stage_times(self):
        return self._plan.stage_times()


class Type1PlanND(_PointsND):
    """f[k] = sum_j c[j] exp(i*isign * k . x_j), modeord=0 box, dims 1-3
    (reference nd.py:386-855)."""

    _TYPE = 1

    def __init__(self, x, n_modes, eps=1e-6, isign=+1, upsampfac=2.0,
                 prec="crit64", sort_points=True, spread_method="auto",
                 kerevalmeth=1):
        super().__init__(x, n_modes, eps, isign, upsampfac, prec, sort_points,
                         spread_method, kerevalmeth)
        if spread_method == "od" and not self._od:
            raise ValueError("OD spreading not applicable to this geometry")

    def _run(self, cs, nvec):
        out = torch.empty((nvec,) + self.N, dtype=torch.complex64,
                          device=cs.device)
        self._plan.execute(cs, out, nvec)
        return out

    def execute(self, c, return_np=True, out=None):
        if numel(c) != self.P:
            raise ValueError(f"c.size ({numel(c)}) must equal the number of "
                             f"nonuniform points ({self.P})")
        cs = as_c64(c, self._plan.device).reshape(-1)
        return finish(self._run(cs, 1)[0], return_np, out)

    def execute_batch(self, cs, return_np=True, out=None):
        """B strength vectors over the same points through one shared spread
        (weights computed once per point) and one batched FFT; cs (B, P),
        returns (B, *N) (nd.py:744-794)."""
        shape = tuple(cs.shape) if hasattr(cs, "shape") else np.shape(cs)
        if len(shape) != 2 or shape[1] != self.P:
            raise ValueError(f"cs must have shape (B, {self.P})")
        B = int(shape[0])
        t = as_c64(cs, self._plan.device)
        if B == 0:
            return finish(torch.empty((0,) + self.N, dtype=torch.complex64,
                                      device=t.device), return_np, out)
        return finish(self._run(t, B), return_np, out)

    def execute_disjoint(self, c, groups, return_np=True, out=None):
        """G disjoint subsets of the plan's points (groups[j] in [0, G)),
        each transformed independently; returns (G, *N) (nd.py:796-855)."""
        g = np.asarray(groups.cpu() if isinstance(groups, torch.Tensor)
                       else groups)
        if g.shape != (self.P,):
            raise ValueError(f"groups must have shape ({self.P},)")
        if numel(c) != self.P:
            raise ValueError(f"c.size ({numel(c)}) must equal the number of "
                             f"nonuniform points ({self.P})")
        G = int(g.max()) + 1 if g.size else 0
        dev = self._plan.device
        res = torch.zeros((G,) + self.N, dtype=torch.complex64,
                          device=torch.device("cuda", dev))
        if G > 0:
            gt = torch.from_numpy(np.ascontiguousarray(g.astype(np.int32))).to(
                res.device)
            cs = as_c64(c, dev).reshape(-1)
            self._plan.execute_disjoint(cs, gt, G, res)
        return finish(res, return_np, out)


class Type2PlanND(_PointsND):
    """c[j] = sum_k f[k] exp(i*isign * k . x_j), modeord=0 box, dims 1-3
    (reference nd.py:858-1119)."""

    _TYPE = 2

    def __init__(self, x, n_modes, eps=1e-6, isign=-1, upsampfac=2.0,
                 prec="crit64", sort_points=False, spread_method="auto",
                 kerevalmeth=1):
        super().__init__(x, n_modes, eps, isign, upsampfac, prec, sort_points,
                         spread_method, kerevalmeth)
        if spread_method == "od" and not self._od:
            raise ValueError("OD interp not applicable to this geometry")

    def _run(self, fs, nvec):
        out = torch.empty((nvec, self.P), dtype=torch.complex64,
                          device=fs.device)
        self._plan.execute(fs, out, nvec)
        return out

    def execute(self, fk, return_np=True, out=None):
        K = int(np.prod(self.N))
        if numel(fk) != K:
            raise ValueError(f"f.size ({numel(fk)}) must equal the mode-box "
                             f"size {tuple(self.N)}")
        fs = as_c64(fk, self._plan.device).reshape(-1)
        return finish(self._run(fs, 1)[0], return_np, out)

    def execute_batch(self, fks, return_np=True, out=None):
        """B mode arrays (B, *N) -> (B, P) through one shared interp pass."""
        K = int(np.prod(self.N))
        t = as_c64(fks, self._plan.device)
        if t.numel() % K != 0:
            raise ValueError(f"fks must have shape (B, *{tuple(self.N)})")
        B = t.numel() // K
        return finish(self._run(t.reshape(-1), B), return_np, out)
