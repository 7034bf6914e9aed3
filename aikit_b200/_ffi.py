"""ctypes binding of the C ABI declared in include/fi8.h."""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libfi8_b200.so")

FI8_OK = 0
FI8_ERR_ARG = 1
FI8_ERR_DECLINED = 2
FI8_ERR_CUDA = 3
FI8_ERR_OOM = 4
FI8_ERR_DEVICE = 5

FI8_OPT_GEMM_MIN_BATCH = 1
FI8_OPT_KERNEL_TIMING = 2
FI8_OPT_GEMM_CTAS = 3
FI8_OPT_GEMM_PAIR = 4
# kernel classes of fi8_index_kernel_times, in index order
KERNEL_KINDS = ("scan_kernel", "gemm_kernel", "select_kernel", "quantize_kernel", "rerank_kernel",
                "redo_gated")

_P = C.c_void_p
_I32 = C.c_int32
_I64 = C.c_int64

# name -> (restype, argtypes); the complete exported surface of include/fi8.h
SIGNATURES = {
    "fi8_last_error": (C.c_char_p, []),
    "fi8_device_count": (C.c_int, [_P]),
    "fi8_ctx_create": (C.c_int, [C.c_int, _P]),
    "fi8_ctx_destroy": (C.c_int, [_P]),
    "fi8_ctx_sm_count": (C.c_int, [_P, _P]),
    "fi8_probe_tensor_i8": (C.c_int, [_P, _I64, _P, _P]),
    "fi8_index_create": (C.c_int, [_P, _P, _P, _I64, _I32, _I64, _P]),
    "fi8_index_destroy": (C.c_int, [_P]),
    "fi8_index_info": (C.c_int, [_P, _P, _P]),
    "fi8_score": (C.c_int, [_P, _P, _P]),
    "fi8_score_batch": (C.c_int, [_P, _P, _I32, _P]),
    "fi8_topk_batch": (C.c_int, [_P, _P, _I32, _I32, _P, _P]),
    "fi8_topk_max_k": (C.c_int, [_P, _P]),
    "fi8_gemm_plan": (C.c_int, [_I64, C.c_int32, C.c_int32, _P, C.c_int32, _P]),
    "fi8_topk_batch_async": (C.c_int, [_P, _P, _I32, _I32, _P, _P]),
    "fi8_index_set_option": (C.c_int, [_P, C.c_int, _I64]),
    "fi8_index_last_launch_count": (C.c_int, [_P, _P]),
    "fi8_index_kernel_times": (C.c_int, [_P, _P, _P, _P, C.c_int]),
    "fi8_index_kernel_log": (C.c_int, [_P, _I32, _P, _P, _P, _P]),
    "fi8_index_sync": (C.c_int, [_P]),
    "fi8_keys_unpack": (C.c_int, [_P, _I64, _P, _P]),
    "fi8_merge_keys_async": (C.c_int, [_P, _P, _I32, _I32, _I32, _P, _P]),
    "fi8_topk1_noalloc": (C.c_int, [_P, _P, _I32, _P, _P]),
    "fi8_bin_index_create": (C.c_int, [_P, _P, _I32, _P, _P, _P, _I64, _I32, _I32, _I64, _P]),
    "fi8_bin_index_destroy": (C.c_int, [_P]),
    "fi8_bin_index_handle": (C.c_int, [_P, _P]),
    "fi8_bin_query_topk": (C.c_int, [_P, _P, _I32, _I32, _P, _P]),
    "fi8_bin_prefilter_async": (C.c_int, [_P, _P, _I32, _I32, _P, _I32, _P]),
    "fi8_bin_rerank_async": (C.c_int, [_P, _P, _I32, _P, _I32, _I32, _P, _P]),
    "fi8_topk_batch_keep": (C.c_int, [_P, _P, _I32, _I32, _P, _I64, _P, _P]),
    "fi8_index_create_f32": (C.c_int, [_P, _P, _I64, _I32, _I64, _P]),
    "fi8_index_read_rows": (C.c_int, [_P, _P, _P]),
    "fi8_bin_index_create_f32": (C.c_int, [_P, _P, _P, _I64, _I32, _I32, _I32, _P, _I64, _P]),
    "fi8_bin_center": (C.c_int, [_P, _P, _P]),
    "fi8_bin_read_codes": (C.c_int, [_P, _P]),
    "fi8_topk_batch_async_keep": (C.c_int, [_P, _P, _I32, _I32, _P, _I64, _P, _P]),
    "fi8_bin_query_topk_keep": (C.c_int, [_P, _P, _I32, _I32, _P, _I64, _P, _P]),
    "fi8_bin_prefilter_async_keep": (C.c_int, [_P, _P, _I32, _I32, _P, _I64, _P, _I32, _P]),
    "fi8_bin_set_tensor_prefilter": (C.c_int, [_P, _I32]),
    "fi8_index_create_empty": (C.c_int, [_P, _I64, _I32, _I64, _P]),
    "fi8_index_upload_rows": (C.c_int, [_P, _I64, _P, _P, _I64]),
    "fi8_index_upload_finish": (C.c_int, [_P]),
    "fi8_bin_index_create_empty": (C.c_int, [_P, _I64, _I32, _I32, _P, _I32, _I64, _P]),
    "fi8_bin_upload_rows": (C.c_int, [_P, _I64, _P, _P, _P, _I64]),
    "fi8_bin_upload_finish": (C.c_int, [_P]),
}


class Fi8Error(RuntimeError):
    """A failing C-ABI call (the Go seam's `error`)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[fi8 {code}] {msg}")
        self.code = code


class DeclinedError(Fi8Error):
    """The device path declined the request (gpu/anncuda/backend.go:577)."""


_lib = None


def lib() -> C.CDLL:
    """Load libfi8_b200.so. Raises if it has not been built: there is no
    fallback implementation."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is missing; build it with `python -m aikit_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc == FI8_OK:
        return
    msg = lib().fi8_last_error().decode(errors="replace")
    if rc == FI8_ERR_DECLINED:
        raise DeclinedError(rc, msg)
    raise Fi8Error(rc, msg)
