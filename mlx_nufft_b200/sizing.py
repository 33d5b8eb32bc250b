"""Kernel-width, grid-size and kernel-transform helpers (host fp64).

Thin wrappers over the C++ restatements in libnufft_b200.so
(csrc/sizing.cpp), which follow the reference's mlx_nufft/sizing.py
(FINUFFT's setup_spreader / set_nhg_type3).  They need no GPU.
"""

import ctypes

import numpy as np

from ._lib import lib, check

PI = np.pi


def next235even(n: int) -> int:
    """Smallest even integer >= n whose prime factors are all in {2, 3, 5}.

    mlx_nufft/sizing.py:13-25."""
    return int(lib.nufft_next235even(int(n)))


def kernel_params(eps: float, upsampfac: float):
    """ES kernel width w and shape beta for tolerance eps at upsampling
    factor upsampfac (mlx_nufft/sizing.py:28-50)."""
    w = ctypes.c_int()
    beta = ctypes.c_double()
    check(lib.nufft_kernel_params(float(eps), float(upsampfac),
                                  ctypes.byref(w), ctypes.byref(beta)))
    return w.value, beta.value


def kernel_ft(xi, beta, w, nquad=128):
    """phihat(xi) = int_{-w/2}^{w/2} psi(d) e^{i xi d} dd by 128-node
    Gauss-Legendre in fp64 (mlx_nufft/sizing.py:74-85)."""
    if nquad != 128:
        raise ValueError("only the 128-node rule is implemented")
    xi = np.ascontiguousarray(np.atleast_1d(np.asarray(xi, dtype=np.float64)))
    out = np.empty_like(xi)
    check(lib.nufft_kernel_ft(
        xi.size, xi.ctypes.data_as(ctypes.POINTER(ctypes.c_double)),
        float(beta), int(w), out.ctypes.data_as(ctypes.POINTER(ctypes.c_double))))
    return out


def es_kernel(d, beta, w):
    """ES kernel value psi(d) = exp(beta (sqrt(1 - (2d/w)^2) - 1)) at distance
    d (fine-grid units), zero outside |d| <= w/2 (mlx_nufft/sizing.py:53-65)."""
    z2 = (2.0 * np.asarray(d, dtype=np.float64) / w) ** 2
    inside = z2 <= 1.0
    out = np.zeros_like(z2)
    out[inside] = np.exp(beta * (np.sqrt(1.0 - z2[inside]) - 1.0))
    return out


def set_nhg_type3(S, X, upsampfac, w):
    """Type-3 grid size nf, spacing h and scale gam for one dimension
    (mlx_nufft/sizing.py:88-111)."""
    nf = ctypes.c_int64()
    h = ctypes.c_double()
    gam = ctypes.c_double()
    check(lib.nufft_set_nhg_type3(float(S), float(X), float(upsampfac), int(w),
                                  ctypes.byref(nf), ctypes.byref(h),
                                  ctypes.byref(gam)))
    return int(nf.value), h.value, gam.value
