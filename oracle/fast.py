"""TEST INFRASTRUCTURE ONLY: ctypes front end of the OpenMP direct sum
(oracle/direct.c), same contract as oracle.port.direct_sum."""

import ctypes

import numpy as np

from .build import build

_lib = None


def _load():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        p = ctypes.c_void_p
        _lib.oracle_direct_sum.argtypes = [
            ctypes.c_int, ctypes.c_int64, p, p, p, p, p, ctypes.c_int64, p, p,
            p, ctypes.c_int, p, p]
        _lib.oracle_direct_sum.restype = None
    return _lib


def direct_sum(x, c, s, isign=+1, idx=None):
    """f[k] = sum_j c_j exp(i isign s_k . x_j), fp64, OpenMP over k."""
    lib = _load()
    x = [np.ascontiguousarray(np.asarray(v, dtype=np.float64).ravel()) for v in x]
    s = [np.asarray(v, dtype=np.float64).ravel() for v in s]
    if idx is not None:
        s = [v[idx] for v in s]
    s = [np.ascontiguousarray(v) for v in s]
    c = np.asarray(c, dtype=np.complex128).ravel()
    cre = np.ascontiguousarray(c.real)
    cim = np.ascontiguousarray(c.imag)
    dim = len(x)
    M, N = x[0].size, s[0].size
    ore = np.empty(N)
    oim = np.empty(N)
    xp = [v.ctypes.data for v in x] + [None] * (3 - dim)
    sp = [v.ctypes.data for v in s] + [None] * (3 - dim)
    lib.oracle_direct_sum(dim, M, xp[0], xp[1], xp[2], cre.ctypes.data,
                          cim.ctypes.data, N, sp[0], sp[1], sp[2],
                          1 if isign >= 0 else -1, ore.ctypes.data,
                          oim.ctypes.data)
    return ore + 1j * oim


def direct_t1(x, c, N, isign=+1, idx=None):
    from .port import mode_lattice
    return direct_sum(x, c, mode_lattice(N, idx), isign)


def direct_t2(x, f, isign=-1, idx=None):
    from .port import mode_lattice
    f = np.asarray(f)
    xs = [np.asarray(v, dtype=np.float64).ravel() for v in x]
    if idx is not None:
        xs = [v[idx] for v in xs]
    return direct_sum(mode_lattice(f.shape), f.ravel(), xs, isign)
