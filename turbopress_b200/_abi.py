"""ctypes binding of the native C ABI (``include/turbopress_b200.h``).

The shared library ``_lib/libturbopress_b200.so`` is built in-tree by
``turbopress_b200.build``.  There is no fallback: if the library is missing
or a CUDA device is absent, every entry point raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libturbopress_b200.so"
_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

TP_OK, TP_ERR_ARG, TP_ERR_UNSUPPORTED, TP_ERR_ALIGN, TP_ERR_CUDA, TP_ERR_WORKSPACE = 0, 1, 2, 3, 4, 6
TP_ERR_DEVICE = 7
TP_F16, TP_F32, TP_BF16 = 0, 1, 2

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int

# name -> (restype, argtypes); must mirror include/turbopress_b200.h
SIGNATURES: dict[str, tuple] = {
    "tp_abi_version": (_I, []),
    "tp_last_error": (ctypes.c_char_p, []),
    "tp_pack_le": (_I, [_P, _P, _I64, _I64, _I, _P]),
    "tp_unpack_le": (_I, [_P, _P, _I64, _I64, _I, _P]),
    "tp_window_decode_levels": (_I, [_P, _P, _P, _I64, _I64, _I, _P]),
    "tp_decode_rows": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _I, _P]),
    "tp_rot_scale": (_I, [_P, _P, _P, _I64, _P]),
    "tp_v1_to_v2": (_I, [_P, _P, _I64, _I64, _I, _P]),
    "tp_rotate": (_I, [_P, _I, _P, _P, _I, _I64, _I64, _I64, _P]),
    "tp_fold_rows": (_I, [_P, _P, _P, _I64, _I64, _I64, _P]),
    "tp_stream_bytes": (_I64, [_I64, _I64, _I]),
    "tp_relayout_v2": (_I, [_P, _P, _P, _I64, _I64, _I, _P]),
    "tp_relayout_v1": (_I, [_P, _P, _P, _I64, _I64, _I, _P]),
    "tp_decode_stream": (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _I, _P]),
    "tp_gemv_workspace_bytes": (_I64, [_I64, _I64, _I64, _I]),
    "tp_tcq_gemv": (_I, [_P, _I, _P, _P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _I, _I, _P, _I64, _P]),
    "tp_tcq_gemv_noalloc": (_I, [_P, _I, _P, _P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _I, _I, _P]),
    "tp_gemv_status": (_I, [_P, _P]),
    "tp_gemv_noalloc_status": (_I, [_P]),
    "tp_gemm_tc_workspace_bytes": (_I64, [_I64, _I64, _I64]),
    "tp_tcq_gemm_tc": (_I, [_P, _I, _P, _P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _I, _I, _P, _I64, _P]),
    "tp_lm_head_workspace_bytes": (_I64, [_I64]),
    "tp_lm_head_argmax": (_I, [_P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _I64, _P]),
    "tp_engine_image_bytes": (_I64, [_I]),
    "tp_engine_build": (_I, [_P, _I, _I, _I, _I, _P, _P, _I64]),
    "tp_engine_counter_bytes": (_I64, [_I]),
    "tp_engine_run": (_I, [_P, _P, _P, _P]),
    "tp_engine_build_tp": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _I64]),
    "tp_ipc_alloc": (_I, [_I64, _P]),
    "tp_ipc_free": (_I, [_P]),
    "tp_ipc_get_handle": (_I, [_P, _P]),
    "tp_ipc_open": (_I, [_P, _P]),
    "tp_ipc_close": (_I, [_P]),
    "tp_gemv_v2": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I, _I, _P]),
    "tp_step_image_bytes": (_I64, [_I]),
    "tp_step_act_bytes": (_I64, [_P]),
    "tp_step_build": (_I, [_P, _P, _P, _I64, _P]),
    "tp_step_bind": (_I, [_P, _P, _I64]),
    "tp_step_run": (_I, [_P, _P, _P, _P, _I64, _P]),
    "tp_step_status": (_I, [_P, _P]),
    "tp_step_set_wait": (_I, [_P, _I64, _I]),
}


def library_path() -> Path:
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    """Load (once) and return the native library; raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not _LIB_PATH.exists():
                raise RuntimeError(
                    f"turbopress_b200 native library not built ({_LIB_PATH}); "
                    "run `python -m turbopress_b200.build`")
            handle = ctypes.CDLL(str(_LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    """Map a tp_status to the reference's exception conventions."""
    if status == TP_OK:
        return
    msg = lib().tp_last_error().decode(errors="replace")
    if status in (TP_ERR_ARG, TP_ERR_ALIGN, TP_ERR_WORKSPACE):
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg}")


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float16:
        return TP_F16
    if dt == torch.float32:
        return TP_F32
    if dt == torch.bfloat16:
        return TP_BF16
    raise ValueError(f"unsupported activation dtype {dt}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("turbopress_b200 kernels need CUDA tensors (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must be on the same CUDA device")
    if dev is None:
        raise ValueError("no tensor given")
    return dev
