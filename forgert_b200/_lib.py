"""Loads libforgert_b200.so (the CUDA kernels + C ABI of include/forgert_attn.h).

There is no fallback: if the library is missing or fails to load, importing
the operators raises, so a GPU run can never silently use another path.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libforgert_b200.so"

FR_OK = 0
FR_ERR_INVALID_ARG = 1
FR_ERR_UNSUPPORTED = 2
FR_ERR_MISALIGNED = 3
FR_ERR_CUDA = 4
FR_ERR_TIMEOUT = 5
FR_ERR_WORKSPACE = 6
FR_ERR_SCRATCH_LIMIT = 7

# Every symbol include/forgert_attn.h declares, with its ctypes signature.
_vp = ctypes.c_void_p
_i = ctypes.c_int
_fp = ctypes.POINTER(ctypes.c_float)
SIGNATURES = {
    "fr_decode_attn": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "fr_decode_attn_noalloc": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "fr_decode_attn_batched": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i,
                                    ctypes.c_longlong, _i, _vp]),
    "fr_decode_attn_paged": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i,
                                  _i, _vp]),
    "fr_decode_attn_partial": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _i, _i, _i, _vp]),
    "fr_lse_merge": (_i, [_vp, _vp, _i, _vp, _i, _i, _vp]),
    "fr_lse_merge_strided": (_i, [_vp, _vp, _i, _vp, _i, _i, ctypes.c_longlong,
                                  ctypes.c_longlong, _vp]),
    "fr_rope_tables": (_i, [_vp, _vp, _i, _i, ctypes.c_float, ctypes.c_float]),
    "fr_rope_tables_device": (_i, [_vp, _vp, _i, _i, ctypes.c_float, ctypes.c_float, _vp]),
    "fr_rope_append": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp]),
    "fr_qkv_bias_rope_append": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i,
                                     _i, _i, _i, _vp]),
    "fr_prefill_attn": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "fr_reserve_workspace": (_i, [ctypes.c_size_t]),
    "fr_exchange_bytes": (ctypes.c_size_t, [_i, _i, _i]),
    "fr_exchange_alloc": (_i, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), _vp]),
    "fr_exchange_open": (_i, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "fr_exchange_close": (_i, [_vp]),
    "fr_exchange_free": (_i, [_vp]),
    "fr_exchange_reset": (_i, [_vp, ctypes.c_size_t, _vp]),
    "fr_decode_attn_exchange": (_i, [_vp, _vp, _vp, _i, _vp, _i, _i, _i,
                                     ctypes.POINTER(ctypes.c_void_p), _i, _i, _vp]),
    "fr_exchange_wait_limit_ms": (_i, []),
    "fr_decode_workspace_size": (ctypes.c_size_t, [_i, _i, _i, _i, _i]),
    "fr_prefill_workspace_size": (ctypes.c_size_t, [_i, _i, _i]),
    "fr_get_device_error": (_i, [_i, ctypes.POINTER(_i)]),
    "fr_allocated_bytes": (ctypes.c_size_t, []),
    "fr_last_cuda_error": (_i, []),
    "fr_status_string": (ctypes.c_char_p, [_i]),
    "fr_version": (_i, []),
    "fr_launch_count": (ctypes.c_ulonglong, []),
    "fr_set_launch_overlap": (_i, [_i]),
    "fr_copy_async": (_i, [_vp, _vp, ctypes.c_size_t, _vp]),
}


class ForgeRTError(RuntimeError):
    """A non-zero status from the C ABI (the reference's launchers surface
    failures as std::runtime_error through CUDA_CHECK, runtime/include/types.h:18-26)."""

    def __init__(self, fn: str, status: int, lib: ctypes.CDLL):
        msg = lib.fr_status_string(status).decode()
        extra = ""
        if status == FR_ERR_CUDA:
            extra = f" (cudaError {lib.fr_last_cuda_error()})"
        super().__init__(f"{fn} failed: status {status}: {msg}{extra}")
        self.status = status


_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("FORGERT_B200_LIB", LIB_PATH))
    if not path.exists():
        raise ImportError(
            f"{path} is missing: build the CUDA library first (python -m forgert_b200.build)")
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(fn: str, status: int) -> None:
    if status != FR_OK:
        raise ForgeRTError(fn, status, load())
