"""Loads libwginfer_b200.so (the C-ABI in include/wginfer_b200.h) via ctypes.

There is no fallback: if the library is missing or cannot be loaded, every op
raises. Build it with ``python -m wginfer_b200.build``.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libwginfer_b200.so")

# wginferDataType_t
DT_I64, DT_F16, DT_F32, DT_BF16 = 6, 12, 13, 15
NUMERICS_FAST, NUMERICS_REFERENCE = 0, 1
STATUS = {0: "ok", 1: "invalid argument", 2: "unsupported dtype", 3: "CUDA error", 4: "out of range",
          5: "out of memory", 6: "timeout", 7: "unsupported"}

_P, _S, _I, _F = C.c_void_p, C.c_size_t, C.c_int, C.c_float

# name -> (restype, argtypes); mirrors include/wginfer_b200.h
SIGNATURES = {
    "wgb_status_string": (C.c_char_p, [_I]),
    "wgb_last_error": (C.c_char_p, []),
    "wgb_version": (_I, []),
    "wgb_set_numerics": (_I, [_I]),
    "wgb_get_numerics": (_I, []),
    "wgb_device_error": (_I, [_P, _P, _P]),
    "wgb_add": (_I, [_P, _P, _P, _I, _S, _P]),
    "wgb_argmax": (_I, [_P, _P, _P, _I, _S, _P]),
    "wgb_argmax_rows": (_I, [_P, _P, _P, _I, _S, _S, _P]),
    "wgb_sample_rows": (_I, [_P, _P, _I, _S, _S, _I, _F, _F, C.c_ulonglong, C.c_ulonglong, _P]),
    "wgb_embedding": (_I, [_P, _P, _P, _I, _S, _S, _S, _P]),
    "wgb_linear": (_I, [_P, _P, _P, _P, _I, _S, _S, _S, _P]),
    "wgb_rms_norm": (_I, [_P, _P, _P, _I, _S, _S, _F, _P]),
    "wgb_rope": (_I, [_P, _P, _P, _I, _S, _S, _S, _F, _P]),
    "wgb_self_attention": (_I, [_P, _P, _P, _P, _I, _S, _S, _S, _S, _S, _S, _F, _P]),
    "wgb_self_attention_workspace_size": (_S, [_S, _S, _S, _S, _S, _S]),
    "wgb_self_attention_ex": (_I, [_P, _P, _P, _P, _I, _S, _S, _S, _S, _S, _S, _F, _P, _S, _P]),
    "wgb_self_attention_noalloc": (_I, [_P, _P, _P, _P, _I, _S, _S, _S, _S, _S, _S, _F, _P]),
    "wgb_self_attention_noalloc_max_scratch": (_S, []),
    "wgb_swiglu": (_I, [_P, _P, _P, _I, _S, _P]),
    "wgb_qwen2_create": (_I, [_P, _I, _I, _P]),
    "wgb_qwen2_destroy": (_I, [_P]),
    "wgb_qwen2_set_weight": (_I, [_P, C.c_char_p, _I, _P, _S, _I]),
    "wgb_qwen2_reset_cache": (_I, [_P]),
    "wgb_qwen2_infer": (_I, [_P, _P, _S, _I, _F, _F, _P]),
    "wgb_qwen2_decode_step": (_I, [_P, _I]),
    "wgb_qwen2_prefill": (_I, [_P, _I, _P, _S]),
    "wgb_qwen2_token_buffer": (_P, [_P]),
    "wgb_qwen2_stream": (_P, [_P]),
    "wgb_qwen2_cache_len": (_S, [_P, _I]),
    "wgb_qwen2_logits": (_P, [_P, _I]),
    "wgb_qwen2_read_tokens": (_I, [_P, _P, _I]),
    "wgb_qwen2_trace_step": (_I, [_P, _I, _I, _P, _P, _S, _P]),
    "wgb_qwen2_read_logits": (_I, [_P, _I, _P]),
}

_lock = threading.Lock()
_lib = None


class WgbError(RuntimeError):
    def __init__(self, status: int, where: str, msg: str):
        self.status = status
        super().__init__(f"{where}: {STATUS.get(status, status)}: {msg}")


class WgbInvalidArgument(WgbError, ValueError):
    pass


def lib() -> C.CDLL:
    """The loaded library; raises if it was not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(f"{LIB_PATH} not built: run python -m wginfer_b200.build")
                l = C.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(l, name)
                    fn.restype, fn.argtypes = res, args
                _lib = l
    return _lib


def check(status: int, where: str) -> None:
    if status != 0:
        msg = lib().wgb_last_error().decode(errors="replace")
        cls = WgbInvalidArgument if status in (1, 2, 4) else WgbError
        raise cls(status, where, msg)


def set_numerics(mode: int) -> None:
    check(lib().wgb_set_numerics(mode), "wgb_set_numerics")


def get_numerics() -> int:
    return lib().wgb_get_numerics()


class numerics:
    """Context manager selecting WGB_NUMERICS_* on the calling thread."""

    def __init__(self, mode):
        self.mode = {"fast": NUMERICS_FAST, "reference": NUMERICS_REFERENCE}.get(mode, mode)

    def __enter__(self):
        self.prev = get_numerics()
        set_numerics(self.mode)
        return self

    def __exit__(self, *exc):
        set_numerics(self.prev)
