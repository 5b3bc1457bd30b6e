"""ctypes binding of libbramha_cuda.so (the C ABI in include/bramha_cuda.h).

There is no CPU fallback: if the library is missing this module raises, so a
product call can never silently run somewhere other than the CUDA kernels.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "libbramha_cuda.so")
HEADER = os.path.join(ROOT, "include", "bramha_cuda.h")

FMT = {"f32": 0, "w8": 1, "w4zp8": 2, "log4": 3, "sp24_f32": 4, "sp24_w8": 5, "sp24_w4zp8": 6}
DTYPE = {"f32": 0, "bf16": 1}
STATUS = {
    0: "BRAMHA_OK", -1: "BRAMHA_ERR_INVALID", -2: "BRAMHA_ERR_SIZE", -3: "BRAMHA_ERR_CUDA",
    -4: "BRAMHA_ERR_OOM", -5: "BRAMHA_ERR_UNSUPPORTED", -6: "BRAMHA_ERR_NOT_FOUND",
    -7: "BRAMHA_ERR_TIMEOUT", -8: "BRAMHA_ERR_NCCL",
}


class BramhaError(RuntimeError):
    """A non-zero status from the C ABI (the reference's `Err(String)`)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{STATUS.get(code, code)}: {message}")
        self.code = code
        self.message = message


_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t
_int = ctypes.c_int
_pp = ctypes.POINTER(ctypes.c_void_p)

_SIGNATURES = {
    "bramha_cuda_init": [_int, ctypes.POINTER(_vp)],
    "bramha_cuda_destroy": [_vp],
    "bramha_cuda_last_error": [],
    "bramha_cuda_abi_version": [],
    "bramha_cuda_set_memory_cap": [_vp, _sz],
    "bramha_cuda_memory_used": [_vp, ctypes.POINTER(_sz)],
    "bramha_cuda_register_weight": [_vp, ctypes.c_char_p, _int, _i64, _i64, _vp, _sz, _vp, _sz, ctypes.POINTER(_vp)],
    "bramha_cuda_register_weight_dev": [_vp, ctypes.c_char_p, _int, _i64, _i64, _vp, _sz, _vp, _sz, _vp,
                                        ctypes.POINTER(_vp)],
    "bramha_cuda_lookup_weight": [_vp, ctypes.c_char_p, ctypes.POINTER(_vp)],
    "bramha_cuda_evict_weight": [_vp, ctypes.c_char_p],
    "bramha_cuda_clear": [_vp],
    "bramha_cuda_weight_info": [_vp, ctypes.POINTER(_int), ctypes.POINTER(_i64), ctypes.POINTER(_i64),
                                ctypes.POINTER(_sz)],
    "bramha_cuda_gemv": [_vp, _vp, _vp, _i64, _vp],
    "bramha_cuda_gemv_dev": [_vp, _vp, _vp, _i64, _vp, _vp],
    "bramha_cuda_gemv_multi_dev": [_vp, _int, _pp, _vp, _i64, _pp, _vp],
    "bramha_cuda_matvec": [_vp, _int, _vp, _i64, _vp, _sz, _vp, _sz, _i64, ctypes.c_char_p, ctypes.c_char_p, _vp],
    "bramha_cuda_register_sparse24": [_vp, ctypes.c_char_p, _int, _i64, _i64, _vp, _sz, _vp, _sz,
                                      ctypes.POINTER(_vp)],
    "bramha_cuda_register_sparse24_dev": [_vp, ctypes.c_char_p, _int, _i64, _i64, _vp, _sz, _vp, _sz, _vp,
                                          ctypes.POINTER(_vp)],
    "bramha_cuda_register_sparse24_compressed": [_vp, ctypes.c_char_p, _i64, _i64, _vp, _sz, _vp, _sz,
                                                 ctypes.POINTER(_vp)],
    "bramha_cuda_sparse_matvec_2_4": [_vp, _int, _vp, _i64, _vp, _sz, _vp, _sz, _i64, ctypes.c_char_p,
                                      ctypes.c_char_p, _vp],
    "bramha_cuda_sparse_matvec_2_4_compressed": [_vp, _vp, _i64, _vp, _sz, _vp, _sz, _i64, ctypes.c_char_p,
                                                 ctypes.c_char_p, _vp],
    "bramha_cuda_gemv_swiglu_dev": [_vp, _vp, _vp, _vp, _i64, _vp, _vp],
    "bramha_cuda_gemv_rmsnorm_dev": [_vp, _int, _vp, _vp, _vp, _vp, ctypes.c_float, _vp, _vp, _vp],
    "bramha_cuda_moe_mlp_dev": [_vp, _vp, _vp, _int, _int, _vp, _vp, _i64, _vp, _vp, _vp],
    "bramha_cuda_moe_mlp": [_vp, _vp, _vp, _int, _int, _vp, _vp, _i64, _vp, _vp],
    "bramha_cuda_moe_route_dev": [_vp, _vp, _i64, _int, _int, _vp, _vp, _vp],
    "bramha_cuda_moe_experts_dev": [_vp, _vp, _vp, _int, _vp, _vp, _i64, _vp, _vp],
    "bramha_cuda_gemm": [_vp, _vp, _vp, _i64, _vp],
    "bramha_cuda_gemm_dev": [_vp, _vp, _vp, _int, _i64, _vp, _vp],
    "bramha_cuda_quantize_dev": [_vp, _int, _i64, _i64, _vp, _vp, _vp, _vp],
    "bramha_cuda_stream_sync": [_vp, _vp],
    "bramha_cuda_gemm_noalloc_dev": [_vp, _vp, _vp, _i64, _vp, _vp],
    "bramha_cuda_set_gemv_kernel": [_vp, _int],
    "bramha_cuda_set_wait_timeout": [_vp, ctypes.c_uint64],
    "bramha_cuda_test_fault": [_vp, _int],
    "bramha_cuda_set_prefetch": [_vp, _i64, _i64],
    "bramha_cuda_set_gemv_tuning": [_vp, _int, _i64],
    "bramha_cuda_shard_handle": [_vp, _sz, _vp],
    "bramha_cuda_shard_init": [_vp, _int, _int, _vp],
    "bramha_cuda_shard_malloc": [_vp, _sz, ctypes.POINTER(_vp)],
    "bramha_cuda_register_weight_shard": [_vp, ctypes.c_char_p, _int, _i64, _i64, _vp, _sz, _vp, _sz,
                                          ctypes.POINTER(_vp)],
    "bramha_cuda_register_weight_shard_dev": [_vp, ctypes.c_char_p, _int, _i64, _i64, _vp, _sz, _vp, _sz, _vp,
                                              ctypes.POINTER(_vp)],
    "bramha_cuda_shard_rows": [_vp, _i64, ctypes.POINTER(_i64), ctypes.POINTER(_i64)],
    "bramha_cuda_shard_sync_dev": [_vp, _vp],
    "bramha_cuda_gemv_chain_dev": [_vp, _int, _vp, _i64, _vp],
    "bramha_cuda_gemv_chain": [_vp, _int, _vp, _i64],
    "bramha_cuda_host_chain_create": [_vp, _int, _vp, _i64, ctypes.POINTER(_vp)],
    "bramha_cuda_host_chain_run": [_vp, _vp],
    "bramha_cuda_host_chain_uses_graph": [_vp, _vp, ctypes.POINTER(_int)],
    "bramha_cuda_host_chain_destroy": [_vp, _vp],
    "bramha_cuda_gemv_program_create": [_vp, _int, _vp, _i64, ctypes.POINTER(_vp)],
    "bramha_cuda_gemv_program_run_dev": [_vp, _vp, _vp],
    "bramha_cuda_gemv_program_destroy": [_vp, _vp],
    "bramha_cuda_gemv_program_trace": [_vp, _vp, _int],
    "bramha_cuda_gemv_program_read_trace": [_vp, _vp, _vp, _sz, ctypes.POINTER(_int)],
    "bramha_cuda_op_embed": [_vp, _vp, _i64, _i64, _vp, _vp, _vp],
    "bramha_cuda_op_rmsnorm": [_vp, _vp, _vp, _vp, _i64, ctypes.c_float, _vp, _vp],
    "bramha_cuda_op_qkv_rope": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _int, _int, _int, ctypes.c_float, _vp, _i64,
                                _vp, _vp, _vp],
    "bramha_cuda_op_attention": [_vp, _vp, _vp, _vp, _vp, _int, _int, _int, _i64, _vp, _vp],
    "bramha_cuda_op_rope_attention": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _int, _int, _int, ctypes.c_float, _vp,
                                      _i64, _vp, _vp, _vp, _vp],
    "bramha_cuda_op_silu_mul": [_vp, _vp, _vp, _i64, _vp, _vp],
    "bramha_cuda_op_select": [_vp, _vp, _i64, _vp, _vp, _i64, ctypes.c_float, _int, _vp, _vp, _vp],
}



class GemvOp(ctypes.Structure):
    """`bramha_gemv_op` of include/bramha_cuda.h (one launch of a GEMV chain)."""
    _fields_ = [("n_weights", ctypes.c_int), ("weights", ctypes.POINTER(ctypes.c_void_p)),
                ("x", ctypes.c_void_p), ("x_up", ctypes.c_void_p), ("y", ctypes.POINTER(ctypes.c_void_p))]


_lib = None


def header_symbols() -> list[str]:
    """Every function the public header declares."""
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(bramha_cuda_\w+)\s*\(", src)))


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m bramha_b200.build` "
                "(there is no CPU fallback for the CUDA plane)")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_char_p if name == "bramha_cuda_last_error" else ctypes.c_int
        _lib = L
    return _lib


def last_error() -> str:
    return lib().bramha_cuda_last_error().decode(errors="replace")


def check(rc: int) -> None:
    if rc != 0:
        raise BramhaError(rc, last_error())
