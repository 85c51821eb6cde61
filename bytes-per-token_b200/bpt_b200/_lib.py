"""The ctypes binding of libbpt_b200.so (include/bpt_b200.h).

The library is loaded lazily, so importing the package never needs a GPU or the built library. A call that
reaches a kernel without the library raises: there is no CPU fallback anywhere in this package.
"""

from __future__ import annotations

import ctypes
import functools
from pathlib import Path

import torch

LIB_PATH = Path(__file__).with_name("libbpt_b200.so")

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_ALIGNMENT, ERR_WORKSPACE, ERR_CUDA = range(6)
DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
KV_FP8, KV_INT8 = 1, 2
FLAG_PDL = 1
FLAG_KV_READY = 2

_DTYPES = {torch.float32: DTYPE_F32, torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16}

P, I64, I32, F32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float

# name -> argument types (the header's order)
SIGNATURES: dict[str, list] = {
    "bpt_abi_version": [],
    "bpt_last_error": [],
    "bpt_device_error": [],
    "bpt_w4a16_linear": [P, I64, P, P, P, P, I64, I64, I64, I64, I64, I32, P],
    "bpt_w4a16_gate_up_silu": [P, I64, P, P, P, P, I64, I64, I64, I64, I64, I32, P],
    "bpt_w4a16_kernel": [I64, I64, I64, I64, I32],
    "bpt_rms_norm_residual": [P, P, P, P, P, I64, I64, F32, I32, P],
    "bpt_qk_norm_rope_kv_write": [P, I64, I64, I64, I64, I64, P, P, P, P, F32, P, P, P, P, P, F32, F32, I64, I64, I32,
                                  P],
    "bpt_rms_norm_int8": [P, I32, I64, P, I32, P, P, P, P, I64, I64, F32, I32, P],
    "bpt_w4a16_quantize": [P, I32, I64, I64, I64, P, P, P, P],
    "bpt_paged_decode_partials": [P, I32, I64, I64, P, P, I32, F32, F32, P, P, P, I64, P, I64, I64, I64, I64, I64, I64,
                                  I64, I64, F32, P, P, I32, P],
    "bpt_paged_attend_workspace_bytes": [I64, I64, I64, I64],
    "bpt_paged_attend": [P, I32, I64, I64, P, P, I32, F32, F32, P, P, P, I64, P, I64, I64, I64, I64, I64, I64, I64, I64,
                         F32, P, I32, P, I64, I32, P],
    "bpt_paged_attend_noalloc": [P, I32, I64, I64, P, P, I32, F32, F32, P, P, P, I64, P, I64, I64, I64, I64, I64, I64,
                                 I64, I64, F32, P, I32, I32, P],
    "bpt_merge_partials": [P, P, I64, I64, I64, I64, P, I32, P],
    "bpt_kivi_decode_partials": [P, I32, I64, I64, I32, I32, P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, I64,
                                 I64, I64, F32, P, P, P],
    "bpt_paged_kv_write": [P, P, I32, I64, I64, I64, I64, I64, I64, I64, P, P, P, P, I32, F32, F32, P, P, I64, I64, P],
    "bpt_kivi_quantize": [P, P, I32, I64, I64, I64, I64, I32, I64, P, P, P, P, P, P, I64, I64, I64, P],
}
RESTYPES = {"bpt_last_error": ctypes.c_char_p, "bpt_paged_attend_workspace_bytes": ctypes.c_int64}


class KernelLibraryMissing(RuntimeError):
    """libbpt_b200.so is not built (run bytes-per-token_b200/build.py)."""


@functools.cache
def lib() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise KernelLibraryMissing(f"{LIB_PATH} is not built: run `python bytes-per-token_b200/build.py`")
    handle = ctypes.CDLL(str(LIB_PATH))
    for name, args in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.argtypes = args
        fn.restype = RESTYPES.get(name, ctypes.c_int)
    return handle


def check(status: int, what: str) -> None:
    """Turn a status code into the exception the reference would raise for the same mistake."""
    if status == OK:
        return
    message = lib().bpt_last_error().decode(errors="replace")
    if status == ERR_CUDA:
        raise RuntimeError(f"{what}: {message}")
    raise ValueError(f"{what}: {message}")


def dtype_code(t: torch.dtype) -> int:
    try:
        return _DTYPES[t]
    except KeyError:
        raise ValueError(f"unsupported dtype {t}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    """Every tensor on one CUDA device (that device is returned); anything else is a ValueError."""
    device = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError(f"expected CUDA tensors, got one on {t.device}: these kernels have no CPU path")
        if device is None:
            device = t.device
        elif t.device != device:
            raise ValueError(f"tensors on different devices: {device} and {t.device}")
    if device is None:
        raise ValueError("no tensor given")
    return device


def device_error() -> int:
    """Synchronize and return (and clear) the first device-side error code the kernels recorded."""
    return int(lib().bpt_device_error())
