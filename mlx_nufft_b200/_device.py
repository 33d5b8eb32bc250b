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


def finish(t, return_np, out=None):
    """Return a device tensor or its numpy copy; with `out` (a host numpy
    array or a torch tensor of the result's size, e.g. pinned host memory),
    copy the result into it and return `out`."""
    if out is not None:
        if isinstance(out, torch.Tensor):
            if out.numel() != t.numel():
                raise ValueError(f"out has {out.numel()} elements, result {t.numel()}")
            out.view(-1).copy_(t.reshape(-1).to(out.dtype))
            if out.device.type == "cpu":
                torch.cuda.current_stream(t.device).synchronize()
        else:
            a = np.asarray(out)
            if a.size != t.numel():
                raise ValueError(f"out has {a.size} elements, result {t.numel()}")
            host = torch.from_numpy(a.reshape(-1)) if a.dtype == np.complex64 \
                else None
            if host is not None and a.flags.c_contiguous:
                host.copy_(t.reshape(-1))
            else:
                np.copyto(a, t.cpu().numpy().reshape(a.shape))
        return out
    if return_np:
        return t.cpu().numpy()
    return t
