"""ctypes binding of ``libtorque_b200.so`` (declared in include/torque_b200.h).

The library is the only compute path: if it cannot be loaded, or no CUDA
device is present, every operation raises ``RuntimeError``.  There is no CPU
fallback.  Status codes map to exceptions the way the reference raises them:
argument/shape errors -> ``ValueError``, device failures -> ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_int, c_int32, c_int64, c_size_t, c_uint8, c_uint32, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("TORQUE_B200_LIB", Path(__file__).resolve().parent / "libtorque_b200.so"))

TQ_OK = 0
TQ_E_BITS = -1
TQ_E_HEAD_DIM = -2
TQ_E_SHAPE = -3
TQ_E_CUDA = -4
TQ_E_TIMEOUT = -5
TQ_E_WORKSPACE = -6
TQ_E_ARG = -7
TQ_E_SCRATCH_LIMIT = -8

TQ_F32, TQ_F16, TQ_BF16 = 0, 1, 2
DECODE_AUTO, DECODE_EXACT, DECODE_TENSOR = 0, 1, 2

_VALUE_ERRORS = {TQ_E_BITS, TQ_E_HEAD_DIM, TQ_E_SHAPE, TQ_E_ARG, TQ_E_SCRATCH_LIMIT}

# name -> (restype, argtypes); must match include/torque_b200.h
SIGNATURES: dict[str, tuple] = {
    "tq_abi_version": (c_int, []),
    "tq_status_string": (ctypes.c_char_p, [c_int]),
    "tq_last_cuda_error": (c_int, []),
    "tq_rotate": (c_int, [c_void_p, c_int, c_void_p, c_int64, c_int, c_void_p, c_void_p, c_void_p]),
    "tq_quantize": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_int, c_void_p]),
    "tq_pack": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p]),
    "tq_unpack": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p]),
    "tq_dequantize_packed": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p]),
    "tq_append_kv": (c_int, [c_void_p, c_void_p, c_int, c_int64, c_int, c_int, c_int, c_void_p, c_void_p,
                             c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
                             c_int, c_int64, c_void_p]),
    "tq_quantize_pack_boundaries": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p,
                                            c_void_p, c_void_p, c_void_p]),
    "tq_lengths_add": (c_int, [c_void_p, c_int, c_int, c_void_p]),
    "tq_decode_workspace_size": (c_int, [c_int64, c_int, c_int, c_int, c_int64, c_int, POINTER(c_size_t)]),
    "tq_decode": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_int,
                          c_int64, c_int64, c_int64, c_int, c_int, c_int, c_void_p, c_void_p, c_float,
                          c_void_p, c_void_p, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "tq_decode_causal": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_int,
                                 c_int64, c_int64, c_int64, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_float,
                                 c_void_p, c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "tq_decode_append": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                 c_void_p, c_void_p, c_int64, c_void_p, c_int, c_int64, c_int64, c_int, c_int,
                                 c_int, c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_int, c_int, c_void_p,
                                 c_size_t, c_void_p]),
    "tq_decode_static": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_int,
                                 c_int64, c_int64, c_int64, c_int, c_int, c_int, c_void_p, c_void_p, c_float,
                                 c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "tq_exchange_buffer_bytes": (c_int, [c_int, c_int, c_int64, POINTER(c_size_t)]),
    "tq_exchange_alloc": (c_int, [c_size_t, POINTER(c_void_p), c_void_p]),
    "tq_exchange_open": (c_int, [c_void_p, POINTER(c_void_p)]),
    "tq_exchange_close": (c_int, [c_void_p]),
    "tq_exchange_free": (c_int, [c_void_p]),
    "tq_decode_exchange": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int, c_void_p,
                                   c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_int, c_int64, c_int64,
                                   c_int64, c_int, c_int, c_int, c_void_p, c_void_p, c_float, c_void_p, c_void_p,
                                   c_int, c_int, c_void_p, c_size_t, c_void_p, c_int, c_int, c_void_p, c_int64,
                                   c_void_p, c_void_p]),
    "tq_rmsnorm": (c_int, [c_void_p, c_void_p, c_float, c_int64, c_int, c_void_p, c_void_p]),
    "tq_rope_qk": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p,
                           c_void_p]),
    "tq_silu_mul": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_void_p]),
    "tq_gemv": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_float, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "tq_lse_merge": (c_int, [c_void_p, c_void_p, c_int, c_int64, c_int, c_void_p, c_void_p, c_int, c_void_p,
                             c_void_p, c_void_p]),
}

_lib: ctypes.CDLL | None = None
_cuda_ok = False  # a CUDA device was found once; the per-call check is skipped after that


def load(require_cuda: bool = True) -> ctypes.CDLL:
    """Load the library (once).  ``require_cuda`` additionally demands a CUDA
    device, which every compute entry point needs."""
    global _lib, _cuda_ok
    if _lib is not None and (_cuda_ok or not require_cuda):
        return _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built; run `python -m torque_mlx_b200.build` "
                "(the CUDA library is required, there is no CPU path)")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    if require_cuda:
        if not torch.cuda.is_available():
            raise RuntimeError("torque_mlx_b200 needs a CUDA device (B200); none is available")
        _cuda_ok = True
    return _lib


def check(status: int, what: str) -> None:
    if status == TQ_OK:
        return
    lib = load(require_cuda=False)
    msg = lib.tq_status_string(status).decode()
    if status == TQ_E_CUDA:
        msg += f" (cudaError {lib.tq_last_cuda_error()})"
    exc = ValueError if status in _VALUE_ERRORS else RuntimeError
    raise exc(f"{what}: {msg}")


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(device: torch.device | None = None) -> int:
    """Handle of the current CUDA stream of ``device`` (default: current device)."""
    if device is None and _raw_stream is not None:
        return _raw_stream(torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return TQ_F32
    if dt == torch.float16:
        return TQ_F16
    if dt == torch.bfloat16:
        return TQ_BF16
    raise ValueError(f"unsupported input dtype {dt} (expected float32, float16 or bfloat16)")
