"""Owner of one native plan handle (libnufft_b200 `nufft_plan_t`).

The plan classes of nd.py / t3.py compose this: it creates the plan on the
current CUDA device, forwards setpts / execute to the C ABI on torch's
current stream, and destroys the plan (and every device buffer it owns)
when garbage-collected.
"""

import ctypes

import numpy as np
import torch

from . import _lib
from ._lib import lib, check
from ._device import require_cuda, stream_ptr

_STAGE_NAMES = ("spread_or_pad", "fft", "interp_or_crop", "total")


class NativePlan:
    def __init__(self, nufft_type, dim, n_modes, n_trans, eps, isign,
                 upsampfac=None, sigma_inner=None, prec="crit64",
                 method="auto", sort_points=True, max_batch=0, profile=False,
                 source_extent=None, kerevalmeth=1):
        self.device = require_cuda()
        opts = _lib.default_opts()
        if kerevalmeth not in (0, 1):
            raise ValueError("kerevalmeth must be 0 (exp/sqrt) or 1 (polynomial)")
        opts.kerevalmeth = int(kerevalmeth)
        opts.upsampfac = float(upsampfac) if upsampfac else 0.0
        opts.sigma_inner = float(sigma_inner) if sigma_inner else 0.0
        if prec not in _lib.PREC:
            raise ValueError(f"unknown prec {prec!r}")
        opts.prec = _lib.PREC[prec]
        if method not in _lib.METHOD:
            raise ValueError(f"unknown spread_method {method!r}")
        opts.method = _lib.METHOD[method]
        opts.sort_points = 1 if sort_points else 0
        opts.max_batch = int(max_batch)
        opts.profile = 1 if profile else 0
        if source_extent is not None:
            opts.has_source_extent = 1
            for d, (lo, hi) in enumerate(source_extent):
                opts.source_extent[2 * d] = float(lo)
                opts.source_extent[2 * d + 1] = float(hi)
        nm = (ctypes.c_int64 * 3)(*([int(n) for n in (n_modes or ())] +
                                     [1] * (3 - len(n_modes or ()))))
        h = ctypes.c_void_p()
        self._h = None
        check(lib.nufft_plan_create(int(nufft_type), int(dim), nm, int(n_trans),
                                    float(eps), int(isign), ctypes.byref(opts),
                                    int(self.device), ctypes.byref(h)))
        self._h = h

    # ------------------------------------------------------------------
    @property
    def handle(self):
        return self._h

    def info(self):
        inf = _lib.NufftPlanInfo()
        check(lib.nufft_plan_get_info(self._h, ctypes.byref(inf)))
        return inf

    def setpts(self, M, xs, N=0, ss=(None, None, None)):
        """xs / ss: fp64 device tensors (or None)."""
        def ptr(t):
            return None if t is None else t.data_ptr()
        xs = list(xs) + [None] * (3 - len(xs))
        ss = list(ss) + [None] * (3 - len(ss))
        with torch.cuda.device(self.device):
            check(lib.nufft_setpts(self._h, int(M), ptr(xs[0]), ptr(xs[1]),
                                   ptr(xs[2]), int(N), ptr(ss[0]), ptr(ss[1]),
                                   ptr(ss[2]), stream_ptr()))

    def set_sources(self, M, xs):
        xs = list(xs) + [None] * (3 - len(xs))
        with torch.cuda.device(self.device):
            check(lib.nufft_set_sources(
                self._h, int(M),
                *[None if t is None else t.data_ptr() for t in xs],
                stream_ptr()))

    def execute(self, inp, out, nvec):
        with torch.cuda.device(self.device):
            check(lib.nufft_execute(self._h, inp.data_ptr(), out.data_ptr(),
                                    int(nvec), stream_ptr()))

    def execute_adjoint(self, inp, out, nvec):
        """nufft_execute_adjoint: the sibling transform with the opposite
        sign on the plan's own points (types 1/2) or on a sibling plan the
        library builds once (type 3)."""
        with torch.cuda.device(self.device):
            check(lib.nufft_execute_adjoint(self._h, inp.data_ptr(), out.data_ptr(),
                                            int(nvec), stream_ptr()))

    def check(self):
        """nufft_plan_check: synchronise and raise a device-side failure
        recorded by earlier executes."""
        with torch.cuda.device(self.device):
            check(lib.nufft_plan_check(self._h, stream_ptr()))

    def execute_stage(self, stage, inp, out, nvec):
        with torch.cuda.device(self.device):
            check(lib.nufft_execute_stage(
                self._h, int(stage), None if inp is None else inp.data_ptr(),
                None if out is None else out.data_ptr(), int(nvec),
                stream_ptr()))

    def grid(self):
        p = ctypes.c_void_p()
        n = ctypes.c_int64()
        check(lib.nufft_get_grid(self._h, ctypes.byref(p), ctypes.byref(n)))
        return p.value, n.value

    def execute_disjoint(self, c, groups, ngroups, out):
        with torch.cuda.device(self.device):
            check(lib.nufft_execute_disjoint(self._h, c.data_ptr(),
                                             groups.data_ptr(), int(ngroups),
                                             out.data_ptr(), stream_ptr()))

    def set_profile(self, on):
        check(lib.nufft_plan_set_profile(self._h, 1 if on else 0))

    def stage_times(self):
        ms = (ctypes.c_float * 4)()
        check(lib.nufft_get_stage_times(self._h, ms, 4))
        return dict(zip(_STAGE_NAMES, [float(v) for v in ms]))

    def debug_points(self, which, dim, count):
        """Sorted geometry (i1 [dim, count] int32, fr [dim, count] float32,
        perm [count] uint32-as-int64) as numpy arrays."""
        dev = torch.device("cuda", self.device)
        i1 = torch.empty(dim * count, dtype=torch.int32, device=dev)
        fr = torch.empty(dim * count, dtype=torch.float32, device=dev)
        perm = torch.empty(count, dtype=torch.int32, device=dev)
        with torch.cuda.device(self.device):
            check(lib.nufft_debug_points(self._h, int(which), i1.data_ptr(),
                                         fr.data_ptr(), perm.data_ptr(),
                                         stream_ptr()))
        return (i1.cpu().numpy().reshape(dim, count),
                fr.cpu().numpy().reshape(dim, count),
                perm.cpu().numpy().view(np.uint32).astype(np.int64))

    def close(self):
        h, self._h = self._h, None
        if h is not None and lib is not None:
            lib.nufft_plan_destroy(h)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
