"""ctypes binding of the C ABI declared in ``include/logitfill_b200.h``.

The library is prebuilt in-tree (``python -m logitfill_b200.build``).  There
is no fallback: if it is missing or a call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "liblogitfill_b200.so"

(LF_OK, LF_ERR_INVALID_ARGUMENT, LF_ERR_UNSUPPORTED, LF_ERR_LAUNCH, LF_ERR_DEVICE_TIMEOUT, LF_ERR_OUT_OF_RANGE,
 LF_ERR_CUDA) = range(7)
LF_F32, LF_F16, LF_BF16 = 0, 1, 2

EXPORTS = (
    "lf_layout_init", "lf_pack_pages", "lf_dequantize", "lf_decode_workspace_bytes",
    "lf_decode_max_splits", "lf_decode_occupancy", "lf_decode_partial", "lf_decode_noalloc", "lf_decode_merge",
    "lf_decode", "lf_decode_multi", "lf_decode_max_splits_multi", "lf_commit_token", "lf_selftest_wait", "lf_selftest_divide",
    "lf_ipc_alloc", "lf_ipc_free", "lf_ipc_handle", "lf_ipc_open", "lf_ipc_close", "lf_decode_merge_gather",
    "lf_gather_signals", "lf_gather_wait", "lf_status_string", "lf_last_error",
)


class LfLayout(ctypes.Structure):
    """Mirror of ``struct lf_layout``."""

    _fields_ = [
        ("kv_heads", c_int32), ("head_dim", c_int32), ("page_size", c_int32), ("k_group", c_int32),
        ("v_group", c_int32), ("bit_v", c_int32), ("width", c_int32 * 4), ("words", c_int32 * 3),
        ("code_off", c_int32 * 3), ("vcode_off", c_int32), ("vcode_words", c_int32),
        ("half_off", c_int32), ("row_words", c_int32), ("meta_halves", c_int32),
        ("scale_off", c_int32 * 3), ("min_off", c_int32 * 3), ("kmax_off", c_int32), ("row_cap", c_int64),
        ("group_cap", c_int64),
    ]


_LIB = None


def lib() -> ctypes.CDLL:
    """Load the native library once; raise if it has not been built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"logitfill_b200 native library missing at {LIB_PATH}; build it with "
            "`python -m logitfill_b200.build` (there is no CPU or Python fallback)")
    so = ctypes.CDLL(str(LIB_PATH))
    P, L = c_void_p, POINTER(LfLayout)
    sig = {
        "lf_layout_init": (c_int, [L, c_int, c_int, c_int, c_int, c_int, c_int, P, c_int64, c_int64]),
        "lf_pack_pages": (c_int, [L, P, P, c_int, c_int64, c_int64, c_int64, P, c_int, c_int, P, P, P, P, P]),
        "lf_dequantize": (c_int, [L, P, P, P, c_int, c_int64, P, P, P]),
        "lf_decode_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
        "lf_decode_max_splits": (c_int, [c_int64, c_int, c_int]),
        "lf_decode_occupancy": (c_int, [L, c_int, c_int]),
        "lf_decode_partial": (c_int, [L, P, P, P, P, P, P, c_int64, c_int64, P, c_int, P, P, c_int64, c_int64,
                                      P, c_int, c_int64, c_int64, c_int, c_int, c_float, c_int, c_int, P, P, P]),
        "lf_decode_merge": (c_int, [P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int, P, c_int,
                                    c_int64, c_int64, P]),
        "lf_decode_noalloc": (c_int, [L, P, P, P, P, P, P, c_int64, c_int64, P, c_int, P, P, c_int64, c_int64,
                                      P, c_int, c_int64, c_int64, c_int, c_int, c_float, c_int, c_int, P, c_int,
                                      c_int64, c_int64, P, P]),
        "lf_decode": (c_int, [L, P, P, P, P, P, P, c_int64, c_int64, P, c_int, P, P, c_int64, c_int64,
                              P, c_int, c_int64, c_int64, c_int, c_int, c_float, c_int, c_int, P, P, c_int,
                              c_int64, c_int64, P, P]),
        "lf_decode_multi": (c_int, [L, P, P, P, P, P, P, c_int64, c_int64, P, c_int, P, P, c_int64, c_int64, c_int64,
                                    P, c_int, c_int64, c_int64, c_int64, c_int, c_int, c_int, c_float, c_int, c_int,
                                    P, P, c_int, c_int64, c_int64, c_int64, P, P]),
        "lf_decode_max_splits_multi": (c_int, [c_int64, c_int, c_int, c_int]),
        "lf_commit_token": (c_int, [L, P, P, P, P, P, c_int64, c_int64, P, P, c_int, P, P, c_int64, c_int64, c_int,
                                    P, P, P]),
        "lf_selftest_wait": (c_int, [P, c_int64, c_int, P]),
        "lf_selftest_divide": (c_int, [P, P, P, c_int64, c_int, P, P, P]),
        "lf_ipc_alloc": (c_int, [c_size_t, P]),
        "lf_ipc_free": (c_int, [P]),
        "lf_ipc_handle": (c_int, [P, P]),
        "lf_ipc_open": (c_int, [P, P]),
        "lf_ipc_close": (c_int, [P]),
        "lf_decode_merge_gather": (c_int, [P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int, P, P, c_int,
                                           c_int, c_int, c_int, P]),
        "lf_gather_signals": (c_int, [c_int, c_int, c_int]),
        "lf_gather_wait": (c_int, [P, c_int, ctypes.c_uint32, ctypes.c_uint64, P, P]),
        "lf_status_string": (c_char_p, [c_int]),
        "lf_last_error": (c_char_p, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(so, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = so
    return so


def check(status: int, what: str) -> None:
    """Raise on a non-zero lf_status, with the library's detail message."""
    if status == LF_OK:
        return
    so = lib()
    text = so.lf_status_string(status).decode()
    detail = so.lf_last_error().decode()
    msg = f"{what}: {text}: {detail}"
    if status == LF_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if status == LF_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    raise RuntimeError(msg)


def dtype_code(dtype) -> int:
    import torch

    codes = {torch.float32: LF_F32, torch.float16: LF_F16, torch.bfloat16: LF_BF16}
    if dtype not in codes:
        raise NotImplementedError(f"dtype {dtype} is not supported (float32, float16, bfloat16)")
    return codes[dtype]


def ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


def stream_handle(device) -> int:
    import torch

    return int(torch.cuda.current_stream(device).cuda_stream)
