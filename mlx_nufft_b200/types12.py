"""Legacy 3D type-1 / type-2 plans (mlx_nufft.types12 compatibility).

The reference keeps Type1Plan / Type2Plan (mlx_nufft/types12.py:24-290) as
its first, 3D-only, even-mode, sigma=1.25 implementation and still exports
them (mlx_nufft/__init__.py:24).  Here they are the ND plans with the legacy
defaults (eps=1e-5, upsampfac=1.25, type-2 isign=+1) and the legacy argument
checks (AssertionError for non-3D or odd mode boxes).  Type2Plan results are
always returned in caller point order.
"""

import numpy as np

from .nd import Type1PlanND, Type2PlanND


def _check_legacy(x, n_modes, prec):
    assert prec in ("fp32", "crit64")
    N = tuple(int(n) for n in n_modes)
    assert len(N) == 3 and all(n % 2 == 0 for n in N), \
        "mode dims must be 3D and even"
    assert len(tuple(x)) == 3


class Type1Plan(Type1PlanND):
    """f[k] = sum_j c[j] exp(i*isign * k . x_j) on an even 3D mode box."""

    def __init__(self, x, n_modes, eps=1e-5, isign=+1, upsampfac=1.25,
                 prec="crit64", sort_points=True):
        _check_legacy(x, n_modes, prec)
        super().__init__(tuple(x), n_modes, eps=eps, isign=isign,
                         upsampfac=upsampfac, prec=prec,
                         sort_points=sort_points)


class Type2Plan(Type2PlanND):
    """c[j] = sum_k f[k] exp(i*isign * k . x_j), f on an even 3D mode box."""

    def __init__(self, x, n_modes, eps=1e-5, isign=+1, upsampfac=1.25,
                 prec="crit64", sort_points=False):
        _check_legacy(x, n_modes, prec)
        super().__init__(tuple(x), n_modes, eps=eps, isign=isign,
                         upsampfac=upsampfac, prec=prec,
                         sort_points=sort_points)
