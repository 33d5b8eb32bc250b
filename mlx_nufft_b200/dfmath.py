"""expi: e^{i*isign*phi} on the GPU for large-magnitude fp64 phases.

Drop-in for mlx_nufft.dfmath (expi, EXPI_MAX_PHASE; reference
mlx_nufft/dfmath.py:1-134).  The reference needs double-single (df64)
arithmetic because Apple GPUs have no fp64; B200 has native fp64, so the
kernel (libnufft_b200 `nufft_expi`, csrc/deconv.cu) sums the phase
components in fp64, reduces mod 2pi with an fma-exact two-constant
Cody-Waite step and evaluates the O(1) residual with fp32 sincos plus a
first-order correction for the residual's low part.  The result is more
accurate than the reference's at every magnitude (no 24-bit quotient limit),
while keeping its interface and validation rules.
"""

import ctypes

import numpy as np
import torch

from ._device import require_cuda, stream_ptr, finish
from ._lib import lib, check

PI = np.pi

# |phi| up to which the reference's f32 quotient rint(phi / 2pi) is exact
# (mlx_nufft/dfmath.py:24); kept for interface compatibility -- the fp64
# reduction here stays accurate beyond it.
EXPI_MAX_PHASE = float(2 ** 24 * 2.0 * PI)


def _as_f64_array(v, device):
    if isinstance(v, torch.Tensor):
        return v.detach().to(device=device, dtype=torch.float64).contiguous()
    # np.array (not ascontiguousarray, which promotes 0-d input to 1-d)
    a = np.array(v, dtype=np.float64, copy=True, order="C")
    return torch.from_numpy(a).to(device)


def expi(phases, isign=1, return_np=False):
    """e^{i*isign*phi} as complex64, same shape as the input.

    phases: an fp64 array (the phase), or a list/tuple of same-shape fp64
    arrays that are summed (in fp64, on the GPU) to form the phase.  A flat
    list of scalars is rejected rather than silently summed.  isign is
    normalised by sign (>= 0 -> +1).  NaN/inf phases give NaN elements.
    Returns a torch CUDA tensor, or numpy when return_np=True."""
    dev = require_cuda()
    if isinstance(phases, (list, tuple)):
        comps = [_as_f64_array(v, dev) for v in phases]
    else:
        comps = [_as_f64_array(phases, dev)]
    if len(comps) < 1:
        raise ValueError("expi: at least one phase component is required")
    shape = tuple(comps[0].shape)
    if any(tuple(c.shape) != shape for c in comps):
        raise ValueError("expi: all phase components must share one shape")
    if len(comps) > 1 and shape == ():
        raise ValueError(
            "expi: got a multi-element sequence of scalars, which would be "
            "summed into a single phase. Pass np.asarray(...) for a vector of "
            "per-element phases, or 1-D arrays as summable phase components.")
    isign = +1 if isign >= 0 else -1
    n = int(np.prod(shape)) if shape else 1
    out = torch.empty(shape, dtype=torch.complex64,
                      device=torch.device("cuda", dev))
    ptrs = (ctypes.c_void_p * len(comps))(*[c.data_ptr() for c in comps])
    with torch.cuda.device(dev):
        check(lib.nufft_expi(len(comps), ptrs, n, isign, out.data_ptr(),
                             stream_ptr()))
    return finish(out, return_np)
