"""mlx_nufft_b200: non-uniform FFTs on NVIDIA B200 (sm_100a), types 1/2/3 in
dimensions 1/2/3, as a drop-in for mlx-nufft's finufft-mirroring interface:

    import mlx_nufft_b200 as finufft
    fk = finufft.nufft2d1(x, y, c, (N1, N2), eps=1e-6)
    plan = finufft.Plan(1, (N1, N2), eps=1e-6)
    plan.setpts(x, y)
    fk = plan.execute(c)

plus the native plan classes (Type1PlanND, Type2PlanND, Type3Plan, the legacy
Type1Plan / Type2Plan) and expi.  Every transform runs in the native library
libnufft_b200.so (hand-written CUDA + cuFFT, reached through its C ABI,
include/nufft_b200.h); importing this package fails if that library has not
been built (`python mlx_nufft_b200/build.py`).  Inputs may be numpy arrays or
torch tensors; results are numpy by default or torch CUDA tensors with
return_np=False.
"""

from .t3 import Type3Plan, GpuT3Plan
from .types12 import Type1Plan, Type2Plan
from .nd import Type1PlanND, Type2PlanND
from .dfmath import expi, EXPI_MAX_PHASE
from .sizing import kernel_params, next235even
from .api import (Plan,
                  nufft1d1, nufft1d2, nufft1d3,
                  nufft2d1, nufft2d2, nufft2d3,
                  nufft3d1, nufft3d2, nufft3d3)


def vkfft_available():
    """Always False: the VkFFT-Metal backend of the reference is replaced by
    cuFFT in this build (reference: mlx_nufft/__init__.py:27-31)."""
    return False


__version__ = "0.1.3+b200"
__all__ = ["Type3Plan", "Type1Plan", "Type2Plan",
           "Type1PlanND", "Type2PlanND", "Plan",
           "nufft1d1", "nufft1d2", "nufft1d3",
           "nufft2d1", "nufft2d2", "nufft2d3",
           "nufft3d1", "nufft3d2", "nufft3d3",
           "kernel_params", "next235even", "vkfft_available",
           "expi", "EXPI_MAX_PHASE"]
