"""finufft-style interface: nufft{1,2,3}d{1,2,3} and Plan.

Same public names, signatures, defaults, exception types and warnings as
mlx_nufft.api (reference mlx_nufft/api.py:1-388, itself a mirror of the
`finufft` Python package), so a caller switches with one import line:

    import mlx_nufft_b200 as finufft
    fk = finufft.nufft2d1(x, y, c, (N1, N2), eps=1e-6)
    plan = finufft.Plan(1, (N1, N2), n_trans=8, eps=1e-6)
    plan.setpts(x, y)
    fk = plan.execute(c)

How a call is served: the keyword options become one `_Request` (eps,
isign, upsampfac, prec); the data argument becomes one `_Batch` (its
vectors stacked on a leading axis, the vector shape checked against the
plan); one native plan is built from a per-type factory table and runs all
vectors in one batched device pass; the batch then shapes, casts and
delivers the result (into `out` when given).  `Plan.execute_adjoint` runs
the library's adjoint entry point (nufft_execute_adjoint) on the plan's own
points instead of building a second plan.

Observable behaviour kept from the reference: modeord=0 mode boxes (even or
odd N); isign >= 0 means +i, default +1 for types 1/3 and -1 for type 2;
multi-vector data carries a leading n_trans axis; eps below 1e-6 is raised
to 1e-6 with a warning (fp32 pipeline); complex128 (or float64) input gives
complex128 output of an fp32-grade transform; modeord=1 raises
NotImplementedError; finufft tuning options are accepted and ignored,
unknown options warn; type 3 warns when upsampfac is not 1.25.  1-D / 2-D
type 3 run the native 1-D / 2-D pipeline (the reference runs them as 3-D
with zero third coordinates: the same sums).
"""

import warnings

import numpy as np
import torch

from .nd import Type1PlanND, Type2PlanND
from .t3 import Type3Plan

EPS_MIN = 1e-6

# finufft options that tune its CPU library and mean nothing here; accepted
# without a warning (the set mlx_nufft/api.py:40-44 accepts)
FINUFFT_NOOP_OPTIONS = frozenset(
    "nthreads debug spread_debug showwarn fftw spread_sort spread_kerevalmeth "
    "spread_kerpad chkbnds maxbatchsize spread_thread spread_nthr_atomic "
    "spread_max_sp_size".split())

_DEFAULT_ISIGN = {1: +1, 2: -1, 3: +1}


class _Request:
    """The normalised keyword options of one call or plan."""

    __slots__ = ("type", "eps", "isign", "upsampfac", "prec")

    def __init__(self, nufft_type, eps, isign, kwargs):
        opts = dict(kwargs)
        if opts.pop("modeord", 0) != 0:
            raise NotImplementedError("modeord=1 (FFT-ordered modes) is not "
                                      "supported; use modeord=0")
        up = opts.pop("upsampfac", None)
        self.upsampfac = None if up in (None, 0, 0.0) else float(up)
        self.prec = opts.pop("prec", "crit64")
        opts.pop("fft_backend", None)      # every fine-grid FFT is cuFFT / own
        unknown = sorted(k for k in opts if k not in FINUFFT_NOOP_OPTIONS)
        if unknown:
            warnings.warn(f"mlx_nufft_b200: unknown options {unknown} ignored")
        self.type = int(nufft_type)
        self.eps = float(eps)
        if self.eps < EPS_MIN:
            warnings.warn(f"mlx_nufft_b200: eps={self.eps:g} is below what the "
                          f"fp32 pipeline delivers; clamping to {EPS_MIN:g}")
            self.eps = EPS_MIN
        self.isign = (_DEFAULT_ISIGN[self.type] if isign is None
                      else (+1 if isign >= 0 else -1))

    def plan(self, coords, n_modes=None, targets=None, isign=None):
        """A native plan of this request's type over `coords`."""
        sign = self.isign if isign is None else isign
        if self.type == 3:
            if self.upsampfac is not None and self.upsampfac != 1.25:
                warnings.warn("mlx_nufft_b200: type 3 runs at upsampfac 1.25; the "
                              f"requested {self.upsampfac:g} is ignored")
            return Type3Plan(tuple(coords), tuple(targets), eps=self.eps,
                             isign=sign, prec=self.prec)
        cls = Type1PlanND if self.type == 1 else Type2PlanND
        extra = {} if self.upsampfac is None else {"upsampfac": self.upsampfac}
        return cls(tuple(coords), n_modes, eps=self.eps, isign=sign,
                   prec=self.prec, **extra)


def _shape(a):
    return tuple(a.shape) if hasattr(a, "shape") else np.shape(a)


def _size(a):
    return int(np.prod(_shape(a)))


def _wide(a):
    """True if the array is double precision (complex128 or float64)."""
    if isinstance(a, torch.Tensor):
        return a.dtype in (torch.complex128, torch.float64)
    return np.asarray(a).dtype in (np.complex128, np.float64)


class _Batch:
    """A data argument as n vectors of `vec_ndim` dims on a leading axis,
    and the rule that shapes a batched result back."""

    def __init__(self, data, vec_ndim, vec_shape=None, what="data"):
        shp = _shape(data)
        if len(shp) == vec_ndim:
            self.n, self.single, vec = 1, True, shp
        elif len(shp) == vec_ndim + 1:
            self.n, self.single, vec = int(shp[0]), False, shp[1:]
        else:
            raise ValueError(f"{what} must have {vec_ndim} or {vec_ndim + 1} "
                             f"dimensions, got shape {shp}")
        if vec_shape is not None and tuple(vec) != tuple(vec_shape):
            raise ValueError(f"{what} vectors have shape {tuple(vec)}, the plan "
                             f"needs {tuple(vec_shape)}")
        self.vec_shape = tuple(int(v) for v in vec)
        if not isinstance(data, (np.ndarray, torch.Tensor)):
            data = np.asarray(data)
        self.stacked = data.reshape((self.n,) + self.vec_shape)

    def deliver(self, res, out, dtype):
        """Result of all vectors (leading axis) -> the caller's shape and
        dtype, copied into `out` when given."""
        res = res.cpu().numpy() if isinstance(res, torch.Tensor) else np.asarray(res)
        if self.single:
            res = res[0]
        res = res.astype(dtype, copy=False)
        if out is None:
            return res
        oshape = tuple(out.shape)
        if oshape not in (res.shape, (1,) + res.shape) and (1,) + oshape != res.shape:
            raise ValueError(f"out has shape {oshape}; the result has shape "
                             f"{res.shape}")
        np.copyto(out, res.reshape(oshape))
        return out


def _mode_box(n_modes, dim, out, batch):
    """The type-1 mode box from n_modes, or from out's trailing dims."""
    if n_modes is None:
        if out is None:
            raise ValueError("give n_modes or an out array to size the modes")
        box = tuple(out.shape)[0 if batch.single else 1:]
        if len(box) != dim:
            raise ValueError(f"out has shape {tuple(out.shape)}, which does not "
                             f"hold {dim}-D modes")
        return tuple(int(n) for n in box)
    if np.isscalar(n_modes):
        return (int(n_modes),) * dim
    return tuple(int(n) for n in n_modes)


def _transform(nufft_type, coords, data, out, eps, isign, kwargs,
               n_modes=None, targets=None):
    """One functional call: request -> batch -> plan -> batched execute."""
    req = _Request(nufft_type, eps, isign, kwargs)
    dim = len(coords)
    dtype = np.complex128 if _wide(data) else np.complex64
    if nufft_type == 2:
        batch = _Batch(data, dim, what="f")
        plan = req.plan(coords, n_modes=batch.vec_shape)
    else:
        batch = _Batch(data, 1, (_size(coords[0]),), what="c")
        if nufft_type == 1:
            plan = req.plan(coords, n_modes=_mode_box(n_modes, dim, out, batch))
        else:
            plan = req.plan(coords, targets=targets)
    res = plan.execute_batch(batch.stacked, return_np=False)
    return batch.deliver(res, out, dtype)


# ---------------------------------------------------------------------------
# functional API (finufft signatures)

def nufft1d1(x, c, n_modes=None, out=None, eps=1e-6, isign=1, **kwargs):
    """1D type-1: f[k] = sum_j c[j] exp(+/-i k x(j))."""
    return _transform(1, (x,), c, out, eps, isign, kwargs, n_modes=n_modes)


def nufft2d1(x, y, c, n_modes=None, out=None, eps=1e-6, isign=1, **kwargs):
    """2D type-1: f[k1,k2] = sum_j c[j] exp(+/-i (k1 x(j) + k2 y(j)))."""
    return _transform(1, (x, y), c, out, eps, isign, kwargs, n_modes=n_modes)


def nufft3d1(x, y, z, c, n_modes=None, out=None, eps=1e-6, isign=1, **kwargs):
    """3D type-1: f[k1,k2,k3] = sum_j c[j] exp(+/-i k . x_j)."""
    return _transform(1, (x, y, z), c, out, eps, isign, kwargs, n_modes=n_modes)


def nufft1d2(x, f, out=None, eps=1e-6, isign=-1, **kwargs):
    """1D type-2: c[j] = sum_k f[k] exp(+/-i k x(j))."""
    return _transform(2, (x,), f, out, eps, isign, kwargs)


def nufft2d2(x, y, f, out=None, eps=1e-6, isign=-1, **kwargs):
    """2D type-2: c[j] = sum_{k1,k2} f[k1,k2] exp(+/-i (k1 x(j) + k2 y(j)))."""
    return _transform(2, (x, y), f, out, eps, isign, kwargs)


def nufft3d2(x, y, z, f, out=None, eps=1e-6, isign=-1, **kwargs):
    """3D type-2: c[j] = sum_k f[k] exp(+/-i k . x_j)."""
    return _transform(2, (x, y, z), f, out, eps, isign, kwargs)


def nufft1d3(x, c, s, out=None, eps=1e-6, isign=1, **kwargs):
    """1D type-3: f[k] = sum_j c[j] exp(+/-i s[k] x[j])."""
    return _transform(3, (x,), c, out, eps, isign, kwargs, targets=(s,))


def nufft2d3(x, y, c, s, t, out=None, eps=1e-6, isign=1, **kwargs):
    """2D type-3: f[k] = sum_j c[j] exp(+/-i (s[k] x[j] + t[k] y[j]))."""
    return _transform(3, (x, y), c, out, eps, isign, kwargs, targets=(s, t))


def nufft3d3(x, y, z, c, s, t, u, out=None, eps=1e-6, isign=1, **kwargs):
    """3D type-3: f[k] = sum_j c[j] exp(+/-i (s,t,u)_k . (x,y,z)_j)."""
    return _transform(3, (x, y, z), c, out, eps, isign, kwargs,
                      targets=(s, t, u))


# ---------------------------------------------------------------------------
# Plan interface

class Plan:
    """finufft.Plan-style plan / setpts / execute (reference
    mlx_nufft/api.py:258-388).

    Plan(nufft_type, n_modes_or_dim, n_trans=1, eps=1e-6, isign=None,
         dtype='complex128', **kwargs)

    Types 1/2: n_modes_or_dim is the mode box (its length is the
    dimension); type 3: the dimension.  setpts() builds the native plan
    (device setpts: fold, sort, subproblem tables); execute() runs the
    n_trans vectors in one batched pass; execute_adjoint() applies the
    adjoint (the sibling transform with the opposite sign) through the
    library on the same points.
    """

    def __init__(self, nufft_type, n_modes_or_dim, n_trans=1, eps=1e-6,
                 isign=None, dtype="complex128", **kwargs):
        if nufft_type not in (1, 2, 3):
            raise ValueError(f"nufft_type must be 1, 2 or 3, got {nufft_type!r}")
        self._req = _Request(nufft_type, eps, isign, kwargs)
        self.type = self._req.type
        self.eps = self._req.eps
        self.isign = self._req.isign
        self.n_trans = int(n_trans)
        self.dtype = np.dtype(dtype)
        if self.dtype not in (np.complex64, np.complex128):
            raise ValueError(f"dtype must be complex64 or complex128, got {dtype!r}")
        if self.type == 3:
            self.dim, self.n_modes = int(n_modes_or_dim), None
        else:
            box = ((n_modes_or_dim,) if np.isscalar(n_modes_or_dim)
                   else n_modes_or_dim)
            self.n_modes = tuple(int(n) for n in box)
            self.dim = len(self.n_modes)
        if self.dim not in (1, 2, 3):
            raise ValueError(f"dimension must be 1, 2 or 3, got {self.dim}")
        self._plan = None
        self._n_targets = None

    def setpts(self, x=None, y=None, z=None, s=None, t=None, u=None):
        coords = tuple(v for v in (x, y, z) if v is not None)
        if len(coords) != self.dim:
            raise ValueError(f"a {self.dim}-D plan needs {self.dim} coordinate "
                             f"arrays, got {len(coords)}")
        if self.type == 3:
            targets = tuple(v for v in (s, t, u) if v is not None)
            if len(targets) != self.dim:
                raise ValueError(f"a {self.dim}-D type-3 plan needs {self.dim} "
                                 f"target arrays, got {len(targets)}")
            self._plan = self._req.plan(coords, targets=targets)
            self._n_targets = _size(targets[0])
        else:
            self._plan = self._req.plan(coords, n_modes=self.n_modes)

    # vector shapes: (dims, shape) of a forward input and of a forward output
    def _vec(self, forward_input):
        points = (1, (self._plan.P,))
        if self.type == 1:
            modes = (self.dim, self.n_modes)
            return points if forward_input else modes
        if self.type == 2:
            modes = (self.dim, self.n_modes)
            return modes if forward_input else points
        return points if forward_input else (1, (self._n_targets,))

    def _batch(self, data, forward_input, what):
        if self._plan is None:
            raise RuntimeError(f"setpts() must be called before {what}()")
        ndim, shape = self._vec(forward_input)
        batch = _Batch(data, ndim, shape)
        if batch.n != self.n_trans:
            raise ValueError(f"data holds {batch.n} vectors; the plan was made "
                             f"for n_trans={self.n_trans}")
        return batch

    def execute(self, data, out=None):
        batch = self._batch(data, True, "execute")
        res = self._plan.execute_batch(batch.stacked, return_np=False)
        return batch.deliver(res, out, self.dtype)

    def execute_adjoint(self, data, out=None):
        """Adjoint of the planned transform (finufft 2.5 API): type 1 maps
        modes -> points, type 2 points -> modes, type 3 targets -> sources;
        the sibling transform with isign negated, run by the library
        (nufft_execute_adjoint) on this plan's points."""
        batch = self._batch(data, False, "execute_adjoint")
        native = self._plan._plan
        dev = torch.device("cuda", native.device)
        inp = _as_c64_device(batch.stacked, dev)
        nd, shape = self._vec(True)
        res = torch.empty((batch.n,) + tuple(shape), dtype=torch.complex64, device=dev)
        native.execute_adjoint(inp, res, batch.n)
        return batch.deliver(res, out, self.dtype)


def _as_c64_device(data, dev):
    from ._device import as_c64
    return as_c64(data, dev.index).reshape(-1)
