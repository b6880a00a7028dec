"""ctypes binding of libelffuss_cuda.so (include/elffuss_cuda.h).

The library is the product path; there is no fallback. Importing this module
without the built library raises ImportError naming the build command.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libelffuss_cuda.so")
HEADER = os.path.join(HERE, "..", "include", "elffuss_cuda.h")

EF_OK, EF_NOT_APPLICABLE = 0, 1
ERRORS = {-1: "EF_ERR_INVALID", -2: "EF_ERR_TYPE", -3: "EF_ERR_SHAPE", -4: "EF_ERR_CUDA",
          -5: "EF_ERR_OOM", -6: "EF_ERR_MISMATCH", -7: "EF_ERR_RANGE", -8: "EF_ERR_TIMEOUT"}
F32, F16, Q4_0, Q8_0, Q2_K, Q4_K, Q5_K, Q6_K, IQ2_XXS, IQ1_S = 0, 1, 2, 8, 10, 12, 13, 14, 16, 19
TYPE_IDS = {"F32": F32, "F16": F16, "Q4_0": Q4_0, "Q8_0": Q8_0, "Q2_K": Q2_K, "Q4_K": Q4_K, "Q5_K": Q5_K,
            "Q6_K": Q6_K, "IQ2_XXS": IQ2_XXS, "IQ1_S": IQ1_S}
TYPE_NAMES = {v: k for k, v in TYPE_IDS.items()}


class EfError(RuntimeError):
    """A negative status from the library (the reference's `throw`)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{ERRORS.get(code, code)}: {message}")
        self.code = code


_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
_PP = ctypes.POINTER(ctypes.c_void_p)

_SIGS = {
    "ef_version": ([], _I),
    "ef_type_info": ([_I, ctypes.POINTER(_I), ctypes.POINTER(_I)], _I),
    "ef_ctx_create": ([_I, _PP], _I),
    "ef_ctx_destroy": ([_P], _I),
    "ef_ctx_set_stream": ([_P, _P], _I),
    "ef_ctx_stream": ([_P], _P),
    "ef_stream_sync": ([_P], _I),
    "ef_last_error": ([_P], ctypes.c_char_p),
    "ef_ctx_launch_count": ([_P], ctypes.c_uint64),
    "ef_alloc": ([_P, _SZ, _PP], _I),
    "ef_free": ([_P, _P], _I),
    "ef_buf_ptr": ([_P], _P),
    "ef_buf_size": ([_P], _SZ),
    "ef_upload": ([_P, _P, _SZ, _P, _SZ], _I),
    "ef_download": ([_P, _P, _SZ, _P, _SZ], _I),
    "ef_scratch_mark": ([_P, ctypes.POINTER(ctypes.c_uint64)], _I),
    "ef_scratch_release": ([_P, ctypes.c_uint64, _PP, _I], _I),
    "ef_weight_load": ([_P, _I, _P, _I64, _I64, _PP], _I),
    "ef_weight_load_device": ([_P, _I, _P, _I64, _I64, _PP], _I),
    "ef_weight_load_slice": ([_P, _I, _P, _I64, _I64, _I64, _I64, _I64, _I64, _PP], _I),
    "ef_weight_load_shard": ([_P, _I, _P, _I64, _I64, _I, _I, _I, _PP], _I),
    "ef_weight_free": ([_P, _P], _I),
    "ef_weight_info": ([_P, ctypes.POINTER(_I), ctypes.POINTER(_I64), ctypes.POINTER(_I64),
                        ctypes.POINTER(_SZ)], _I),
    "ef_weight_unpack": ([_P, _P, _P], _I),
    "ef_dequant": ([_P, _P, _I64, _I64, _P], _I),
    "ef_gemv": ([_P, _P, _P, _I, _P], _I),
    "ef_gemv_swiglu": ([_P, _P, _P, _P, _I, _P], _I),
    "ef_gemv_sections": ([_P, _PP, _I, _P, _I, _PP], _I),
    "ef_gemm": ([_P, _P, _P, _I, _I, _P, ctypes.c_uint32], _I),
    "ef_matmul": ([_P, _P, _P, _I, _P], _I),
    "ef_gemv_noalloc": ([_P, _P, _I, _P, _P], _I),
    "ef_gather": ([_P, _P, _P, _I, _P], _I),
    "ef_rmsnorm": ([_P, _P, _P, _I, _I, ctypes.c_float, _P], _I),
    "ef_norm_add_norm": ([_P, _P, _P, _P, _P, _I, _I, ctypes.c_float, _P], _I),
    "ef_shortconv": ([_P, _P, _P, _P, _I, _I, _I, _P], _I),
    "ef_qk_norm_rope_cache": ([_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, ctypes.c_float, ctypes.c_float,
                               _P, _P], _I),
    "ef_attn_decode": ([_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P], _I),
    "ef_argmax_step": ([_P, _P, _I, _P, _P, _P, _I, _I], _I),
    "ef_ctx_set_pdl": ([_P, _I], _I),
    "ef_gather_rmsnorm": ([_P, _P, _P, _I, _P, ctypes.c_float, _P, _P], _I),
    "ef_argmax_rows": ([_P, _P, _I, _I, _P, _P, _P, _I, _I], _I),
    "ef_argmax_partial": ([_P, _P, _I, _I, _I, _P], _I),
    "ef_argmax_select": ([_P, _P, _I, _I, _P, _P, _P, _I, _I], _I),
    "ef_rope_cache": ([_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, ctypes.c_float, ctypes.c_float,
                       _P, _P], _I),
    "ef_attention": ([_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P], _I),
    "ef_qk_norm_rope_cache_f16": ([_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, ctypes.c_float, ctypes.c_float,
                                   _P, _P], _I),
    "ef_attn_decode_f16": ([_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P], _I),
    "ef_rope_cache_f16": ([_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, ctypes.c_float, ctypes.c_float,
                           _P, _P], _I),
    "ef_attention_f16": ([_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P], _I),
    "ef_swiglu": ([_P, _P, _P, ctypes.c_int64, _P], _I),
    "ef_topk": ([_P, _P, _I, _I, _I, _P, _P, _P], _I),
    "ef_tp_create": ([_P, _I, _I, ctypes.c_size_t, ctypes.c_double, _P], _I),
    "ef_tp_handle": ([_P, _P, _P], _I),
    "ef_tp_connect": ([_P, _P, _P], _I),
    "ef_allreduce_sum": ([_P, _P, _P, ctypes.c_int64], _I),
    "ef_allgather": ([_P, _P, _P, ctypes.c_int64, _P], _I),
    "ef_tp_status": ([_P, _P], _I),
    "ef_gemm_status": ([_P], _I),
    "ef_gemm_set_wait_limit": ([_P, _I], _I),
    "ef_gguf_open": ([ctypes.c_char_p, _P, ctypes.c_char_p, ctypes.c_size_t], _I),
    "ef_gguf_close": ([_P], _I),
    "ef_gguf_header": ([_P, _P, _P, _P, _P, _P], _I),
    "ef_gguf_tensor": ([_P, ctypes.c_int64, _P, _P, _P, _P, _P, _P], _I),
    "ef_gguf_find_tensor": ([_P, ctypes.c_char_p], ctypes.c_int64),
    "ef_gguf_tensor_data": ([_P, ctypes.c_int64], _P),
    "ef_gguf_find_key": ([_P, ctypes.c_char_p], ctypes.c_int64),
    "ef_gguf_meta": ([_P, ctypes.c_int64, _P, _P, _P, _P, _P], _I),
    "ef_gguf_load_weight": ([_P, _P, ctypes.c_char_p, _P], _I),
    "ef_gemv_allreduce_norm": ([_P, _P, _P, _P, _I, _P, _P, _P, ctypes.c_float, _P], _I),
    "ef_gemv_allgather": ([_P, _P, _P, _P, _I, _P], _I),
    "ef_tp_destroy": ([_P, _P], _I),
}


def header_symbols() -> list[str]:
    """Every function the public header declares."""
    src = open(HEADER, encoding="utf-8").read()
    return sorted(set(re.findall(r"EF_API\s+[\w\s\*]*?\b(ef_\w+)\s*\(", src)))


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with "
                              f"`python elffuss-engine_b200/build.py` (or __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def check(rc: int, ctx=None) -> int:
    """Raise EfError for a negative status; return 0 or EF_NOT_APPLICABLE."""
    if rc < 0:
        msg = lib().ef_last_error(ctx).decode(errors="replace") if ctx else ""
        raise EfError(rc, msg)
    return rc
