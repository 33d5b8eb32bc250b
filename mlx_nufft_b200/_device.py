"""Device plumbing shared by the plan classes: CUDA context checks, the
current torch stream, and conversion of numpy / torch inputs to contiguous
device tensors of the dtypes the C ABI expects (fp64 coordinates, complex64
data)."""

import numpy as np
import torch


def require_cuda():
    """Current CUDA device ordinal; raises if no GPU is present (this library
    has no CPU execution path)."""
    if not torch.cuda.is_available():
        raise RuntimeError("mlx_nufft_b200 requires a CUDA GPU (sm_100a); "
                           "no CPU execution path exists")
    return torch.cuda.current_device()


def stream_ptr(device=None):
    return torch.cuda.current_stream(device).cuda_stream


def as_f64(x, device):
    """1-D contiguous fp64 device tensor from a numpy / torch / sequence."""
    if isinstance(x, torch.Tensor):
        t = x.detach().reshape(-1)
        if t.is_complex():
            raise ValueError("coordinates must be real")
        return t.to(device=device, dtype=torch.float64).contiguous()
    a = np.asarray(x, dtype=np.float64).ravel()
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def as_c64(c, device):
    """Contiguous complex64 device tensor (shape preserved)."""
    if isinstance(c, torch.Tensor):
        t = c.detach()
        if not t.is_complex():
            t = t.to(torch.complex64)
        return t.to(device=device, dtype=torch.complex64).contiguous()
    a = np.asarray(c)
    if a.dtype != np.complex64:
        a = a.astype(np.complex64)
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def numel(x):
    if isinstance(x, torch.Tensor):
        return int(x.numel())
    return int(np.asarray(x).size)


def finish(t, return_np):
    """Return a device tensor or its numpy copy."""
    if return_np:
        return t.cpu().numpy()
    return t
