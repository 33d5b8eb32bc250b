"""finufft-compatible API (nufft{1,2,3}d{1,2,3}, Plan) on the B200 core.

Drop-in mirror of mlx_nufft.api (reference mlx_nufft/api.py:1-388), which
itself mirrors the `finufft` Python package:

    import mlx_nufft_b200 as finufft
    fk = finufft.nufft2d1(x, y, c, (N1, N2), eps=1e-6)
    plan = finufft.Plan(1, (N1, N2), n_trans=8, eps=1e-6)
    plan.setpts(x, y)
    fk = plan.execute(c)

Semantics kept from the reference: modeord=0 boxes (even or odd N); isign
>= 0 means +i; leading n_trans axis on multi-vector data; out= filled in
place; eps below 1e-6 clamps with a warning (fp32 pipeline floor);
complex128 in -> complex128 out (fp32-grade transform); modeord=1 raises
NotImplementedError; unknown options warn, finufft tuning options are
ignored.  Multi-vector calls run as one batched execute (shared point
weights, batched cuFFT) instead of the reference's per-vector loop.
"""

import warnings

import numpy as np
import torch

from .nd import Type1PlanND, Type2PlanND
from .t3 import Type3Plan

_EPS_FLOOR = 1e-6
_IGNORED_OPTS = {
    "nthreads", "debug", "spread_debug", "showwarn", "fftw", "spread_sort",
    "spread_kerevalmeth", "spread_kerpad", "chkbnds", "maxbatchsize",
    "spread_thread", "spread_nthr_atomic", "spread_max_sp_size",
}


def _check_opts(kwargs):
    """api.py:47-61"""
    opts = dict(kwargs)
    if opts.pop("modeord", 0) not in (0,):
        raise NotImplementedError("modeord=1 (FFT ordering) not implemented")
    upsampfac = opts.pop("upsampfac", None)
    if upsampfac in (0, 0.0):                 # finufft auto sentinel
        upsampfac = None
    prec = opts.pop("prec", "crit64")
    fft_backend = opts.pop("fft_backend", "mlx")   # accepted for compatibility
    for k in list(opts):
        if k in _IGNORED_OPTS:
            opts.pop(k)
    if opts:
        warnings.warn(f"mlx_nufft_b200: ignoring unknown options {sorted(opts)}")
    return upsampfac, prec, fft_backend


def _norm_eps(eps):
    eps = float(eps)
    if eps < _EPS_FLOOR:
        warnings.warn(
            f"mlx_nufft_b200: eps={eps:g} is below the fp32 pipeline floor; "
            f"clamping to {_EPS_FLOOR:g}")
        eps = _EPS_FLOOR
    return eps


def _norm_isign(isign, default):
    if isign is None:
        return default
    return +1 if isign >= 0 else -1


def _dtype_of(a):
    if isinstance(a, torch.Tensor):
        return {torch.complex128: np.complex128, torch.float64: np.float64,
                torch.complex64: np.complex64}.get(a.dtype, np.float32)
    return np.asarray(a).dtype


def _out_dtype(*arrays):
    for a in arrays:
        if _dtype_of(a) in (np.complex128, np.float64):
            return np.complex128
    return np.complex64


def _shape(a):
    return tuple(a.shape) if hasattr(a, "shape") else np.shape(a)


def _vec_shape(data, inner_ndim, inner_shape=None):
    """(n_trans, data with a leading vector axis); api.py:87-102."""
    shp = _shape(data)
    if len(shp) == inner_ndim:
        n, inner = 1, shp
        data = data.reshape((1,) + tuple(shp)) if hasattr(data, "reshape") \
            else np.asarray(data)[None, ...]
    elif len(shp) == inner_ndim + 1:
        n, inner = shp[0], shp[1:]
    else:
        raise ValueError(f"data must have {inner_ndim} or {inner_ndim + 1} "
                         f"dims, got shape {shp}")
    if inner_shape is not None and tuple(inner) != tuple(inner_shape):
        raise ValueError(f"data inner shape {tuple(inner)} must be "
                         f"{tuple(inner_shape)}")
    return int(n), data


def _fill_out(out, res, dtype):
    res = np.asarray(res).astype(dtype, copy=False)
    if out is not None:
        if out.shape != res.shape and out.shape != (1,) + res.shape \
                and (1,) + out.shape != res.shape:
            raise ValueError(f"out.shape {out.shape} does not match result "
                             f"shape {res.shape}")
        np.copyto(out, res.reshape(out.shape))
        return out
    return res


def _modes_tuple(n_modes, dim, out, out_offset=0):
    if n_modes is None:
        if out is None:
            raise ValueError("either n_modes or out must be supplied")
        shape = out.shape[out_offset:]
        if len(shape) != dim:
            raise ValueError(f"out shape {out.shape} does not match dim {dim}")
        return tuple(int(n) for n in shape)
    if np.isscalar(n_modes):
        return (int(n_modes),) * dim
    return tuple(int(n) for n in n_modes)


def _ndim(a):
    return len(_shape(a))


# ---------------------------------------------------------------------------
# type 1: nonuniform -> uniform

def _nufft_t1(dim, coords, c, n_modes, out, eps, isign, kwargs):
    upsampfac, prec, _ = _check_opts(kwargs)
    eps = _norm_eps(eps)
    isign = _norm_isign(isign, +1)
    dtype = _out_dtype(c)
    M = int(np.prod(_shape(coords[0])))
    n_tr, cv = _vec_shape(c, 1, inner_shape=(M,))
    if out is not None and n_modes is None:
        n_modes = _modes_tuple(None, dim, out, out_offset=(1 if n_tr > 1 else 0))
    N = _modes_tuple(n_modes, dim, out)
    kw = {} if upsampfac is None else {"upsampfac": upsampfac}
    plan = Type1PlanND(coords, N, eps=eps, isign=isign, prec=prec, **kw)
    res = plan.execute_batch(cv)
    if n_tr == 1 and _ndim(c) == 1:
        res = res[0]
    return _fill_out(out, res, dtype)


def nufft1d1(x, c, n_modes=None, out=None, eps=1e-6, isign=1, **kwargs):
    """1D type-1: f[k] = sum_j c[j] exp(+/-i k x(j))."""
    return _nufft_t1(1, (x,), c, n_modes, out, eps, isign, kwargs)


def nufft2d1(x, y, c, n_modes=None, out=None, eps=1e-6, isign=1, **kwargs):
    """2D type-1: f[k1,k2] = sum_j c[j] exp(+/-i (k1 x(j) + k2 y(j)))."""
    return _nufft_t1(2, (x, y), c, n_modes, out, eps, isign, kwargs)


def nufft3d1(x, y, z, c, n_modes=None, out=None, eps=1e-6, isign=1, **kwargs):
    """3D type-1: f[k1,k2,k3] = sum_j c[j] exp(+/-i k . x_j)."""
    return _nufft_t1(3, (x, y, z), c, n_modes, out, eps, isign, kwargs)


# ---------------------------------------------------------------------------
# type 2: uniform -> nonuniform

def _nufft_t2(dim, coords, f, out, eps, isign, kwargs):
    upsampfac, prec, _ = _check_opts(kwargs)
    eps = _norm_eps(eps)
    isign = _norm_isign(isign, -1)
    dtype = _out_dtype(f)
    n_tr, fv = _vec_shape(f, dim)
    N = tuple(_shape(fv)[1:])
    kw = {} if upsampfac is None else {"upsampfac": upsampfac}
    plan = Type2PlanND(coords, N, eps=eps, isign=isign, prec=prec, **kw)
    res = plan.execute_batch(fv)
    if n_tr == 1 and _ndim(f) == dim:
        res = res[0]
    return _fill_out(out, res, dtype)


def nufft1d2(x, f, out=None, eps=1e-6, isign=-1, **kwargs):
    """1D type-2: c[j] = sum_k f[k] exp(+/-i k x(j))."""
    return _nufft_t2(1, (x,), f, out, eps, isign, kwargs)


def nufft2d2(x, y, f, out=None, eps=1e-6, isign=-1, **kwargs):
    """2D type-2: c[j] = sum_{k1,k2} f[k1,k2] exp(+/-i (k1 x(j) + k2 y(j)))."""
    return _nufft_t2(2, (x, y), f, out, eps, isign, kwargs)


def nufft3d2(x, y, z, f, out=None, eps=1e-6, isign=-1, **kwargs):
    """3D type-2: c[j] = sum_k f[k] exp(+/-i k . x_j)."""
    return _nufft_t2(3, (x, y, z), f, out, eps, isign, kwargs)


# ---------------------------------------------------------------------------
# type 3: nonuniform -> nonuniform

def _nufft_t3(dim, src, c, trg, out, eps, isign, kwargs):
    upsampfac, prec, _ = _check_opts(kwargs)
    if upsampfac is not None and upsampfac != 1.25:
        warnings.warn("mlx_nufft_b200: type-3 runs the validated sigma=1.25 "
                      "pipeline; upsampfac ignored")
    eps = _norm_eps(eps)
    isign = _norm_isign(isign, +1)
    dtype = _out_dtype(c)
    M = int(np.prod(_shape(src[0])))
    n_tr, cv = _vec_shape(c, 1, inner_shape=(M,))
    plan = Type3Plan(src, trg, eps=eps, isign=isign, prec=prec)
    res = plan.execute_batch(cv)
    if n_tr == 1 and _ndim(c) == 1:
        res = res[0]
    return _fill_out(out, res, dtype)


def nufft1d3(x, c, s, out=None, eps=1e-6, isign=1, **kwargs):
    """1D type-3: f[k] = sum_j c[j] exp(+/-i s[k] x[j])."""
    return _nufft_t3(1, (x,), c, (s,), out, eps, isign, kwargs)


def nufft2d3(x, y, c, s, t, out=None, eps=1e-6, isign=1, **kwargs):
    """2D type-3: f[k] = sum_j c[j] exp(+/-i (s[k] x[j] + t[k] y[j]))."""
    return _nufft_t3(2, (x, y), c, (s, t), out, eps, isign, kwargs)


def nufft3d3(x, y, z, c, s, t, u, out=None, eps=1e-6, isign=1, **kwargs):
    """3D type-3: f[k] = sum_j c[j] exp(+/-i (s,t,u)_k . (x,y,z)_j)."""
    return _nufft_t3(3, (x, y, z), c, (s, t, u), out, eps, isign, kwargs)


# ---------------------------------------------------------------------------
# Plan interface

class Plan:
    """finufft.Plan-compatible plan/setpts/execute interface (api.py:258-388).

    Plan(nufft_type, n_modes_or_dim, n_trans=1, eps=1e-6, isign=None,
         dtype='complex128', **kwargs)

    For types 1/2, n_modes_or_dim is the mode tuple (dim inferred from its
    length); for type 3 it is the dimension.  setpts() builds the device
    plan; execute() runs all n_trans vectors in one batched pass.
    """

    def __init__(self, nufft_type, n_modes_or_dim, n_trans=1, eps=1e-6,
                 isign=None, dtype="complex128", **kwargs):
        if nufft_type not in (1, 2, 3):
            raise ValueError("nufft_type must be 1, 2 or 3")
        self.type = int(nufft_type)
        self.n_trans = int(n_trans)
        self.eps = _norm_eps(eps)
        self.isign = _norm_isign(isign, -1 if self.type == 2 else +1)
        self.dtype = np.dtype(dtype)
        if self.dtype not in (np.complex64, np.complex128):
            raise ValueError("dtype must be complex64 or complex128")
        self._upsampfac, self._prec, _ = _check_opts(kwargs)
        if self.type == 3:
            self.dim = int(n_modes_or_dim)
            self.n_modes = None
        else:
            if np.isscalar(n_modes_or_dim):
                n_modes_or_dim = (n_modes_or_dim,)
            self.n_modes = tuple(int(n) for n in n_modes_or_dim)
            self.dim = len(self.n_modes)
        if self.dim not in (1, 2, 3):
            raise ValueError("dim must be 1, 2 or 3")
        self._plan = None
        self._adjoint = None
        self._n_targets = None

    def setpts(self, x=None, y=None, z=None, s=None, t=None, u=None):
        coords = [v for v in (x, y, z) if v is not None]
        if len(coords) != self.dim:
            raise ValueError(f"expected {self.dim} coordinate arrays, "
                             f"got {len(coords)}")
        kw = {} if self._upsampfac is None else {"upsampfac": self._upsampfac}
        self._adjoint = None
        if self.type == 1:
            self._plan = Type1PlanND(tuple(coords), self.n_modes, eps=self.eps,
                                     isign=self.isign, prec=self._prec, **kw)
        elif self.type == 2:
            self._plan = Type2PlanND(tuple(coords), self.n_modes, eps=self.eps,
                                     isign=self.isign, prec=self._prec, **kw)
        else:
            if self._upsampfac is not None and self._upsampfac != 1.25:
                warnings.warn("mlx_nufft_b200: type-3 runs the validated "
                              "sigma=1.25 pipeline; upsampfac ignored")
            trg = [v for v in (s, t, u) if v is not None]
            if len(trg) != self.dim:
                raise ValueError(f"expected {self.dim} target arrays, "
                                 f"got {len(trg)}")
            self._plan = Type3Plan(tuple(coords), tuple(trg), eps=self.eps,
                                   isign=self.isign, prec=self._prec)
            self._n_targets = int(np.prod(_shape(trg[0])))
        self._coords = list(coords)
        self._targets = None if self.type != 3 else \
            [v for v in (s, t, u) if v is not None]

    def _run(self, plan, data, inner, ishape, out):
        n_tr, dv = _vec_shape(data, inner, inner_shape=ishape)
        if n_tr != self.n_trans:
            raise ValueError(f"data has {n_tr} vectors, plan has "
                             f"n_trans={self.n_trans}")
        res = plan.execute_batch(dv)
        if self.n_trans == 1 and _ndim(data) == inner:
            res = res[0]
        return _fill_out(out, res, self.dtype)

    def execute(self, data, out=None):
        if self._plan is None:
            raise RuntimeError("setpts() must be called before execute()")
        if self.type == 2:
            inner, ishape = self.dim, self.n_modes
        else:
            inner, ishape = 1, (self._plan.P,)
        return self._run(self._plan, data, inner, ishape, out)

    def execute_adjoint(self, data, out=None):
        """Adjoint of the planned transform (finufft 2.5 API): the sibling
        transform with isign negated (api.py:347-388)."""
        if self._plan is None:
            raise RuntimeError("setpts() must be called before "
                               "execute_adjoint()")
        if self._adjoint is None:
            kw = {} if self._upsampfac is None \
                else {"upsampfac": self._upsampfac}
            if self.type == 1:
                self._adjoint = Type2PlanND(tuple(self._coords), self.n_modes,
                                            eps=self.eps, isign=-self.isign,
                                            prec=self._prec, **kw)
            elif self.type == 2:
                self._adjoint = Type1PlanND(tuple(self._coords), self.n_modes,
                                            eps=self.eps, isign=-self.isign,
                                            prec=self._prec, **kw)
            else:
                self._adjoint = Type3Plan(tuple(self._targets),
                                          tuple(self._coords), eps=self.eps,
                                          isign=-self.isign, prec=self._prec)
        if self.type == 1:
            inner, ishape = self.dim, self.n_modes
        elif self.type == 2:
            inner, ishape = 1, (self._plan.P,)
        else:
            inner, ishape = 1, (self._n_targets,)
        return self._run(self._adjoint, data, inner, ishape, out)
