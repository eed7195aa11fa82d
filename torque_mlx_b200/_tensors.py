"""Host-side tensor plumbing shared by the public API.

Public functions accept numpy arrays or torch tensors.  Inputs are moved to
the current CUDA device (numpy/CPU tensors are copied host -> device), the
work runs in the CUDA library, and results come back in the caller's kind:
numpy in -> numpy out, torch in -> CUDA torch tensor out."""

from __future__ import annotations

import numpy as np
import torch

from . import _lib


def device() -> torch.device:
    _lib.load()
    return torch.device("cuda", torch.cuda.current_device())


def _on_current_device(t: torch.Tensor) -> bool:
    return t.is_cuda and t.device.index == torch.cuda.current_device()


def is_numpy(x) -> bool:
    return not isinstance(x, torch.Tensor)


_FLOATS = (torch.float16, torch.bfloat16, torch.float32)


def to_cuda(x, dtype: torch.dtype | None = None, *, keep_half: bool = False) -> torch.Tensor:
    """Contiguous CUDA tensor.  ``keep_half`` keeps fp16/bf16 inputs as they are
    (the kernels widen them exactly); otherwise the result is ``dtype``."""
    if isinstance(x, torch.Tensor):
        # fast path: already a usable tensor on the current device
        if (x.is_contiguous() and (dtype is None or x.dtype == dtype or (keep_half and x.dtype in _FLOATS))
                and _lib.load() is not None and _on_current_device(x)):
            return x
        t = x
    else:
        a = np.asarray(x)
        if a.dtype == np.uint32:
            a = a.view(np.int32)
        t = torch.from_numpy(np.ascontiguousarray(a))
    if keep_half and t.dtype in (torch.float16, torch.bfloat16, torch.float32):
        pass
    elif dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t.to(device(), non_blocking=False).contiguous()


def words_to_cuda(x) -> torch.Tensor:
    """uint32 words (numpy uint32 / torch uint32 or int32) -> CUDA int32 storage."""
    dev = device()
    if isinstance(x, torch.Tensor):
        t = x.view(torch.int32) if x.dtype == torch.uint32 else x
        if t.dtype != torch.int32:
            t = t.to(torch.int64).to(torch.int32)
        return t.to(dev).contiguous()
    a = np.ascontiguousarray(np.asarray(x, dtype=np.uint32)).view(np.int32)
    return torch.from_numpy(a).to(dev).contiguous()


def words_out(t: torch.Tensor, numpy_out: bool):
    """int32 word storage -> numpy uint32 or torch uint32 view."""
    if numpy_out:
        return t.cpu().numpy().view(np.uint32)
    return t.view(torch.uint32)


def out(t: torch.Tensor, numpy_out: bool):
    return t.cpu().numpy() if numpy_out else t
