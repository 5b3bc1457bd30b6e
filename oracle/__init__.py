"""CPU oracle for the quantized linear-layer path -- TEST INFRASTRUCTURE ONLY.

numpy/ctypes wrappers around ``liboracle.so``, the plain-C restatement of the
reference's CPU arithmetic (akshaybhlrp/bramha):

* packers / dequantizers: ``src/models/quantization.rs:7-122``
* log4 decoder: ``spanda-engine/src/lib.rs:332-342`` (encoder defined here)
* decode GEMV ``matvec_mul_into``: ``src/inference/cpu_engine.rs:1307-1444``
* allocating GEMV ``matvec_mul``: ``src/inference/cpu_engine.rs:355-562``
* prefill GEMM ``gemm_cpu``: ``src/inference/cpu_engine.rs:565-706``
* 2:4 sparse GEMVs and compression: ``spanda-engine/src/sparse.rs:19-138``,
  ``src/inference/cpu_engine.rs:1532-1640``, ``spanda-engine/src/bin/convert.rs:55-92``
* MoE expert MLP (router softmax, stable top-k, SwiGLU experts, weighted sum):
  ``src/inference/cpu_engine.rs:1799-1989``
* decode-step operations (RMSNorm, RoPE, single-token attention, SwiGLU,
  repetition penalty + argmax): ``src/inference/cpu_engine.rs:1292-1302,
  1450-1530, 1682-1698, 2023-2026, 2985-3031``; the step itself is in
  ``oracle/decode.py``

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline and
reference legs may import this package.  The product path (``bramha_b200``)
never does: it fails loudly when its CUDA library is missing.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i8p = ctypes.POINTER(ctypes.c_int8)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_i64 = ctypes.c_int64


def build(force: bool = False) -> str:
    """Compile liboracle.so with its Makefile (gcc, no fast-math, no FMA contraction)."""
    target = os.path.basename(_LIB_PATH)
    if force or not os.path.exists(_LIB_PATH) or (
        os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "bramha_oracle.c"))
    ):
        subprocess.run(["make", "-s", "-C", _HERE] + (["-B"] if force else []) + [target], check=True)
    return _LIB_PATH


def use_native_build() -> bool:
    """Switch this process to a ``-march=native`` build of the same source, for
    the timed CPU legs of bench.py only: the reference compiles with
    ``target-cpu=native`` (.cargo/config.toml:2).  The build is redone on the
    host that runs it (a native binary does not travel); on failure the
    portable build stays in use and False is returned."""
    global _lib, _LIB_PATH
    native = os.path.join(_HERE, "liboracle_native.so")
    try:
        subprocess.run(["make", "-s", "-B", "-C", _HERE, "liboracle_native.so"], check=True, capture_output=True)
    except Exception:
        return False
    _lib = None
    _LIB_PATH = native
    return True


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        sig = {
            "bro_quantize_to_int8": (None, [_f32p, _i64, _i64, _i8p, _f32p]),
            "bro_quantize_to_int4": (ctypes.c_int, [_f32p, _i64, _i64, _u8p, _f32p]),
            "bro_quantize_to_log4": (ctypes.c_int, [_f32p, _i64, _i64, _u8p, _f32p]),
            "bro_dequantize_int8": (None, [_i8p, _f32p, _i64, _i64, _f32p]),
            "bro_dequantize_int4": (None, [_u8p, _f32p, _i64, _i64, _f32p]),
            "bro_dequantize_log4": (None, [_u8p, _i64, ctypes.c_float, _f32p]),
            "bro_dequantize_log4_rows": (None, [_u8p, _f32p, _i64, _i64, _f32p]),
            "bro_matvec_into_f32": (None, [_f32p, _i64, _f32p, _i64, _f32p, ctypes.c_int]),
            "bro_matvec_into_i8": (None, [_f32p, _i64, _i8p, _f32p, _i64, _f32p, ctypes.c_int]),
            "bro_matvec_into_u4": (None, [_f32p, _i64, _u8p, _f32p, _i64, _f32p, ctypes.c_int]),
            "bro_matvec_into_log4": (None, [_f32p, _i64, _u8p, _f32p, _i64, _f32p, ctypes.c_int]),
            "bro_matvec_fused_log4": (None, [_f32p, _i64, _u8p, _f32p, _i64, _f32p, ctypes.c_int]),
            "bro_matvec_f32": (None, [_f32p, _i64, _f32p, _i64, _f32p]),
            "bro_matvec_i8": (None, [_f32p, _i64, _i8p, _f32p, _i64, _f32p]),
            "bro_matvec_u4": (None, [_f32p, _i64, _u8p, _f32p, _i64, _f32p]),
            "bro_gemm_f32": (None, [_f32p, _i64, _i64, _f32p, _i64, _f32p]),
            "bro_gemm_i8": (None, [_f32p, _i64, _i64, _i8p, _f32p, _i64, _f32p]),
            "bro_gemm_u4": (None, [_f32p, _i64, _i64, _u8p, _f32p, _i64, _f32p]),
            "bro_gemm_log4": (None, [_f32p, _i64, _i64, _u8p, _f32p, _i64, _f32p]),
            "bro_gemm_u4_par": (None, [_f32p, _i64, _i64, _u8p, _f32p, _i64, _f32p, ctypes.c_int]),
            "bro_max_threads": (ctypes.c_int, []),
            "bro_rms_norm": (None, [_f32p, _f32p, _i64, ctypes.c_float, _f32p]),
            "bro_rope": (None, [_f32p, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_float]),
            "bro_attention": (None, [_f32p, _f32p, _f32p, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]),
            "bro_silu_mul": (None, [_f32p, _f32p, _i64, _f32p]),
            "bro_penalty_argmax": (ctypes.c_int64, [_f32p, _i64, ctypes.POINTER(ctypes.c_int32), _i64,
                                                    ctypes.c_float]),
            "bro_sparse_matvec_2_4": (None, [ctypes.c_int, _f32p, _i64, ctypes.c_void_p, _f32p, _i64, _f32p,
                                             ctypes.c_int]),
            "bro_sparse_matvec_2_4_compressed": (None, [_f32p, _u16p, _f32p, _i64, _i64, _i64, _f32p, ctypes.c_int]),
            "bro_compress_2_4": (_i64, [_f32p, _i64, _u16p, _f32p]),
            "bro_moe_mlp": (None, [ctypes.c_int, _f32p, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int, _f32p,
                                   ctypes.c_void_p, _f32p, ctypes.c_void_p, _f32p, ctypes.c_void_p, _f32p, _f32p,
                                   ctypes.POINTER(ctypes.c_int32), _f32p, ctypes.c_int]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ----------------------------------------------------------------------------- packers
def quantize_to_int8(w: np.ndarray, out_features: int, in_features: int):
    w = _c(w, np.float32)
    q = np.empty(out_features * in_features, np.int8)
    s = np.empty(out_features, np.float32)
    lib().bro_quantize_to_int8(_p(w, _f32p), out_features, in_features, _p(q, _i8p), _p(s, _f32p))
    return q, s


def quantize_to_int4(w: np.ndarray, out_features: int, in_features: int):
    w = _c(w, np.float32)
    q = np.empty(out_features * (in_features // 2), np.uint8)
    s = np.empty(out_features, np.float32)
    rc = lib().bro_quantize_to_int4(_p(w, _f32p), out_features, in_features, _p(q, _u8p), _p(s, _f32p))
    if rc != 0:
        raise ValueError("in_features must be a multiple of 2 for INT4 packing")
    return q, s


def quantize_to_log4(w: np.ndarray, out_features: int, in_features: int):
    w = _c(w, np.float32)
    q = np.empty(out_features * (in_features // 2), np.uint8)
    s = np.empty(out_features, np.float32)
    rc = lib().bro_quantize_to_log4(_p(w, _f32p), out_features, in_features, _p(q, _u8p), _p(s, _f32p))
    if rc != 0:
        raise ValueError("in_features must be a multiple of 2 for LOG4 packing")
    return q, s


def dequantize_int8(q, scales, in_features: int):
    q = _c(q, np.int8)
    scales = _c(scales, np.float32)
    n = scales.size
    out = np.empty(n * in_features, np.float32)
    lib().bro_dequantize_int8(_p(q, _i8p), _p(scales, _f32p), n, in_features, _p(out, _f32p))
    return out


def dequantize_int4(q, scales, in_features: int):
    q = _c(q, np.uint8)
    scales = _c(scales, np.float32)
    n = scales.size
    out = np.zeros(n * in_features, np.float32)
    lib().bro_dequantize_int4(_p(q, _u8p), _p(scales, _f32p), n, in_features, _p(out, _f32p))
    return out


def dequantize_log4(data, scale: float):
    data = _c(data, np.uint8)
    out = np.empty(data.size * 2, np.float32)
    lib().bro_dequantize_log4(_p(data, _u8p), data.size, ctypes.c_float(scale), _p(out, _f32p))
    return out


def dequantize_log4_rows(q, scales, in_features: int):
    q = _c(q, np.uint8)
    scales = _c(scales, np.float32)
    n = scales.size
    out = np.zeros(n * in_features, np.float32)
    lib().bro_dequantize_log4_rows(_p(q, _u8p), _p(scales, _f32p), n, in_features, _p(out, _f32p))
    return out


# ----------------------------------------------------------------------------- GEMV / GEMM
FORMATS = ("f32", "w8", "w4zp8", "log4")


def matvec_mul_into(fmt: str, h, q, scales, out_features: int, threads: int = 0):
    """Decode GEMV as `matvec_mul_into` computes it (4 interleaved accumulators)."""
    h = _c(h, np.float32)
    K = h.size
    out = np.empty(out_features, np.float32)
    L = lib()
    if fmt == "f32":
        w = _c(q, np.float32)
        L.bro_matvec_into_f32(_p(h, _f32p), K, _p(w, _f32p), out_features, _p(out, _f32p), threads)
        return out
    scales = _c(scales, np.float32)
    if fmt == "w8":
        L.bro_matvec_into_i8(_p(h, _f32p), K, _p(_c(q, np.int8), _i8p), _p(scales, _f32p), out_features,
                             _p(out, _f32p), threads)
    elif fmt == "w4zp8":
        L.bro_matvec_into_u4(_p(h, _f32p), K, _p(_c(q, np.uint8), _u8p), _p(scales, _f32p), out_features,
                             _p(out, _f32p), threads)
    elif fmt == "log4":
        L.bro_matvec_into_log4(_p(h, _f32p), K, _p(_c(q, np.uint8), _u8p), _p(scales, _f32p), out_features,
                               _p(out, _f32p), threads)
    else:
        raise ValueError(fmt)
    return out


def matvec_fused_log4(h, q, scales, out_features: int, threads: int = 0):
    h = _c(h, np.float32)
    out = np.empty(out_features, np.float32)
    lib().bro_matvec_fused_log4(_p(h, _f32p), h.size, _p(_c(q, np.uint8), _u8p), _p(_c(scales, np.float32), _f32p),
                                out_features, _p(out, _f32p), threads)
    return out


def matvec_mul(fmt: str, h, q, scales, out_features: int):
    """`matvec_mul` (single accumulator, cpu_engine.rs:456-561)."""
    h = _c(h, np.float32)
    K = h.size
    out = np.empty(out_features, np.float32)
    L = lib()
    if fmt == "f32":
        L.bro_matvec_f32(_p(h, _f32p), K, _p(_c(q, np.float32), _f32p), out_features, _p(out, _f32p))
    elif fmt == "w8":
        L.bro_matvec_i8(_p(h, _f32p), K, _p(_c(q, np.int8), _i8p), _p(_c(scales, np.float32), _f32p),
                        out_features, _p(out, _f32p))
    elif fmt == "w4zp8":
        L.bro_matvec_u4(_p(h, _f32p), K, _p(_c(q, np.uint8), _u8p), _p(_c(scales, np.float32), _f32p),
                        out_features, _p(out, _f32p))
    else:
        raise ValueError(fmt)
    return out


def gemm_cpu(fmt: str, h_block, q, scales, block_size: int, in_features: int, out_features: int):
    """`gemm_cpu` sequential branch: out[b][j] = s_j * sum_i h[b][i] * dq(w_ji)."""
    hb = _c(h_block, np.float32)
    out = np.empty(block_size * out_features, np.float32)
    L = lib()
    args = (_p(hb, _f32p), block_size, in_features)
    if fmt == "f32":
        L.bro_gemm_f32(*args, _p(_c(q, np.float32), _f32p), out_features, _p(out, _f32p))
    elif fmt == "w8":
        L.bro_gemm_i8(*args, _p(_c(q, np.int8), _i8p), _p(_c(scales, np.float32), _f32p), out_features,
                      _p(out, _f32p))
    elif fmt == "w4zp8":
        L.bro_gemm_u4(*args, _p(_c(q, np.uint8), _u8p), _p(_c(scales, np.float32), _f32p), out_features,
                      _p(out, _f32p))
    elif fmt == "log4":
        L.bro_gemm_log4(*args, _p(_c(q, np.uint8), _u8p), _p(_c(scales, np.float32), _f32p), out_features,
                        _p(out, _f32p))
    else:
        raise ValueError(fmt)
    return out


def quantize(fmt: str, w, out_features: int, in_features: int):
    if fmt == "w8":
        return quantize_to_int8(w, out_features, in_features)
    if fmt == "w4zp8":
        return quantize_to_int4(w, out_features, in_features)
    if fmt == "log4":
        return quantize_to_log4(w, out_features, in_features)
    if fmt == "f32":
        return _c(w, np.float32).reshape(-1).copy(), None
    raise ValueError(fmt)


def dequantize(fmt: str, q, scales, in_features: int):
    if fmt == "w8":
        return dequantize_int8(q, scales, in_features)
    if fmt == "w4zp8":
        return dequantize_int4(q, scales, in_features)
    if fmt == "log4":
        return dequantize_log4_rows(q, scales, in_features)
    if fmt == "f32":
        return _c(q, np.float32)
    raise ValueError(fmt)


def max_threads() -> int:
    return int(lib().bro_max_threads())


# ---- decode-step operations (cpu_engine.rs; see bramha_oracle.c) -------------
def rms_norm(x, w, eps: float):
    x = _c(x, np.float32)
    w = _c(w, np.float32)
    out = np.empty_like(x)
    lib().bro_rms_norm(_p(x, _f32p), _p(w, _f32p), x.size, eps, _p(out, _f32p))
    return out


def rope_(v, pos: int, num_heads: int, head_dim: int, rope_theta: float):
    """In-place RoPE of a float32 vector of num_heads * head_dim values."""
    assert v.dtype == np.float32 and v.flags.c_contiguous
    lib().bro_rope(_p(v, _f32p), pos, num_heads, head_dim, rope_theta)
    return v


def attention(q, k_cache, v_cache, kv_len: int, num_q_heads: int, num_kv_heads: int, head_dim: int):
    q = _c(q, np.float32)
    k_cache = _c(k_cache, np.float32)
    v_cache = _c(v_cache, np.float32)
    out = np.empty(num_q_heads * head_dim, np.float32)
    lib().bro_attention(_p(q, _f32p), _p(k_cache, _f32p), _p(v_cache, _f32p), kv_len, num_q_heads,
                        num_kv_heads, head_dim, _p(out, _f32p))
    return out


def silu_mul(g, u):
    g = _c(g, np.float32)
    u = _c(u, np.float32)
    out = np.empty_like(g)
    lib().bro_silu_mul(_p(g, _f32p), _p(u, _f32p), g.size, _p(out, _f32p))
    return out


def penalty_argmax(logits, generated, penalty: float = 1.15):
    """Applies the repetition penalty to `logits` in place; returns the argmax."""
    assert logits.dtype == np.float32 and logits.flags.c_contiguous
    gen = np.ascontiguousarray(np.asarray(generated, dtype=np.int32))
    return int(lib().bro_penalty_argmax(_p(logits, _f32p), logits.size,
                                        gen.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), gen.size, penalty))


# ---- 2:4 structured sparsity (sparse.rs, cpu_engine.rs:1532-1640) ------------
_SP_FMT = {"f32": 0, "w8": 1, "w4zp8": 2}


def sparse_matvec_2_4(fmt: str, h, q, scales, out_features: int, threads: int = 0):
    """sparse_matvec_mul_2_4_tensor_into: top-2-of-4 products per group, the
    K % 4 trailing columns densely, times the row scale (i8 / int4)."""
    h = _c(h, np.float32)
    qa = np.ascontiguousarray(q)
    sa = None if scales is None else _c(scales, np.float32)
    out = np.empty(out_features, np.float32)
    lib().bro_sparse_matvec_2_4(_SP_FMT[fmt], _p(h, _f32p), h.size, qa.ctypes.data,
                                None if sa is None else _p(sa, _f32p), out_features, _p(out, _f32p), threads)
    return out


def sparse_matvec_2_4_compressed(x, masks, values, rows: int, cols: int, threads: int = 0):
    x = _c(x, np.float32)
    m = _c(masks, np.uint16)
    v = _c(values, np.float32)
    assert m.size >= rows * (cols // 4) and x.size >= (cols // 4) * 4
    out = np.empty(rows, np.float32)
    lib().bro_sparse_matvec_2_4_compressed(_p(x, _f32p), _p(m, _u16p), _p(v, _f32p), v.size, rows, cols,
                                           _p(out, _f32p), threads)
    return out


def compress_2_4(w):
    """convert.rs:55-92 over a flat f32 tensor (length a multiple of 4):
    (masks u16 [n/4], values f32 [n/2])."""
    w = _c(w, np.float32).reshape(-1)
    assert w.size % 4 == 0
    masks = np.empty(w.size // 4, np.uint16)
    values = np.empty(w.size // 2, np.float32)
    nv = lib().bro_compress_2_4(_p(w, _f32p), w.size, _p(masks, _u16p), _p(values, _f32p))
    assert nv == values.size
    return masks, values


# ---- MoE expert MLP (run_mlp_into's MoE branch, cpu_engine.rs:1799-1989) -----
_MOE_FMT = {"f32": 0, "w8": 1, "w4zp8": 2, "log4": 3}


def moe_mlp(fmt: str, h, logits, top_k: int, gate, up, down, threads: int = 0):
    """h [T][H], logits [T][E]; gate / up = (codes of the E stacked [I][H]
    weights, scales [E*I] or None for f32), down = (codes of [E][H][I], scales
    [E*H]).  Returns (out [T][H], selected expert ids [T][k], their weights
    [T][k]) -- the first k of the sorted order, including experts skipped for
    a weight <= 0."""
    h = _c(h, np.float32)
    lg = _c(logits, np.float32)
    T, H = h.shape
    E = lg.shape[1]
    gq, gs = gate
    uq, us = up
    dq, ds = down
    gq, uq, dq = (np.ascontiguousarray(a) for a in (gq, uq, dq))
    I = (gs.size if gs is not None else gq.size // (4 * H)) // E
    k = min(top_k, E)
    out = np.empty((T, H), np.float32)
    ids = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    sp = lambda a: None if a is None else _p(_c(a, np.float32), _f32p)
    lib().bro_moe_mlp(_MOE_FMT[fmt], _p(h, _f32p), T, H, I, E, top_k, _p(lg, _f32p), gq.ctypes.data, sp(gs),
                      uq.ctypes.data, sp(us), dq.ctypes.data, sp(ds), _p(out, _f32p),
                      ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), _p(w, _f32p), threads)
    return out, ids, w
