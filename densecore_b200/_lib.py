"""ctypes binding of libdcgpu.so (declarations: include/dcgpu.h).

The product path has no CPU fallback: if the library is missing, loading fails with an error.
"""
from __future__ import annotations

import ctypes
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB_PATH = os.environ.get("DCG_LIB_PATH") or os.path.join(PKG, "libdcgpu.so")
HEADER = os.path.join(ROOT, "include", "dcgpu.h")

_lib = None

vp, i32, i64, sz, f32 = (ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t,
                         ctypes.c_float)

# argtypes / restype of every exported symbol (kept in sync with include/dcgpu.h by a test)
SIGNATURES = {
    "dcg_version": (i32, []),
    "dcg_set_programmatic_launch": (i32, [i32]),
    "dcg_strerror": (ctypes.c_char_p, [i32]),
    "dcg_last_error": (ctypes.c_char_p, []),
    "dcg_device_error": (i32, [ctypes.POINTER(i32), i32]),
    "dcg_row_size": (sz, [i32, i64]),
    "dcg_packed_weight_size": (sz, [i32, i64, i64]),
    "dcg_mul_mat_scratch_size": (sz, [i32, i64, i64, i64]),
    "dcg_mul_mat_q_scratch_size": (sz, [i32, i64, i64, i64]),
    "dcg_quantize_row_q8_0": (i32, [vp, vp, i64, i64, vp]),
    "dcg_quantize_row_q8_K": (i32, [vp, vp, i64, i64, vp]),
    "dcg_quantize_weights": (i32, [i32, vp, vp, i64, i64, vp]),
    "dcg_weight_pack": (i32, [i32, vp, sz, i64, i64, vp, vp]),
    "dcg_weight_unpack": (i32, [i32, vp, i64, i64, vp, sz, vp]),
    "dcg_mul_mat": (i32, [i32, vp, i64, i64, vp, i64, vp, vp, sz, vp]),
    "dcg_act_size": (sz, [i32, i64, i64]),
    "dcg_quantize_act": (i32, [i32, vp, vp, i64, i64, vp]),
    "dcg_mul_mat_q": (i32, [i32, vp, i64, i64, vp, i64, vp, vp, sz, vp]),
    "dcg_mul_mat_noalloc": (i32, [i32, vp, i64, i64, vp, i64, vp, vp]),
    "dcg_paged_attn_scratch_size": (sz, [i32, i32, i32, i32, i32]),
    "dcg_paged_attn_decode": (i32, [vp, vp, vp, i64, i32, i32, vp, i32, vp, i32, i32, i32, i32, i32,
                                    f32, vp, vp, sz, vp]),
    "dcg_paged_attn_prefill": (i32, [vp, vp, vp, i64, i32, i32, vp, i32, vp, vp, i32, i32, i32, i32, i32, i32,
                                     f32, vp, vp]),
    "dcg_qk_norm_rope_kv_append_tokens": (i32, [vp, i64, vp, i64, vp, i64, i32, i32, i32, i32, vp, vp, f32, f32,
                                                vp, vp, vp, vp, vp, i32, i32, vp, i32, vp]),
    "dcg_kv_append": (i32, [vp, vp, vp, vp, i32, i32, vp, i32, vp, vp, i32, i32, i32, vp]),
    "dcg_add_rmsnorm_quantize": (i32, [vp, vp, vp, f32, i64, i64, i32, vp, vp]),
    "dcg_swiglu_quantize": (i32, [vp, vp, i64, i64, i64, i32, vp, vp]),
    "dcg_qk_norm_rope_kv_append": (i32, [vp, i64, vp, i64, vp, i64, i32, i32, i32, i32, vp, vp, f32, f32,
                                         vp, vp, vp, vp, i32, i32, vp, i32, vp]),
    "dcg_ctx_create": (i32, [i32, ctypes.POINTER(vp)]),
    "dcg_ctx_destroy": (i32, [vp]),
    "dcg_ctx_weight_register": (i32, [vp, i32, vp, sz, i64, i64, ctypes.POINTER(vp)]),
    "dcg_ctx_weight_release": (i32, [vp, vp]),
    "dcg_ctx_find_weight": (i32, [vp, vp, ctypes.POINTER(vp)]),
    "dcg_ctx_mul_mat": (i32, [vp, vp, vp, i64, vp]),
}


class DcgError(RuntimeError):
    def __init__(self, code: int, where: str):
        lib = load()
        msg = lib.dcg_last_error().decode(errors="replace")
        super().__init__(f"{where}: {lib.dcg_strerror(code).decode()} ({code}): {msg}")
        self.code = code


def load():
    """Load libdcgpu.so (raises if it was never built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m densecore_b200.build`"
                              " (there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int, where: str) -> None:
    if rc != 0:
        raise DcgError(rc, where)


def header_symbols() -> list[str]:
    """Function names declared in include/dcgpu.h."""
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(dcg_\w+)\s*\(", txt, re.M)))
