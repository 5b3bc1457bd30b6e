"""`CudaComputePlane`: the reference's GPU compute-plane interface on the C ABI.

Mirrors `WgpuComputePlane` (src/compute/wgpu_backend.rs:100-1728) method by
method, same argument meaning and error behaviour:

* ``matvec_mul(h, weight, out_features, model_name=None, layer_name=None)``  (:734)
* ``matvec_mul_int8(h, q_weight, scales, out_features, model_name, layer_name)``  (:906)
* ``matvec_mul_int4(h, q_weight, scales, out_features, model_name, layer_name)``  (:1083)
* ``matvec_mul_log4(...)``: the same for SPANDA 4-bit log codes
  (decoder spanda-engine/src/lib.rs:332-342; no GPU arm exists in the reference)
* ``gemm(fmt, h_block, q, scales, block_size, in_features, out_features)``:
  the prefill GEMM that `gemm_cpu` (src/inference/cpu_engine.rs:565) computes
* ``clear_persistent_buffers()`` (:725)
* ``moe_mlp(gate_up, down, num_experts, top_k, x, logits)``: the MoE branch
  of run_mlp_into (src/inference/cpu_engine.rs:1799-1989) for a batch of
  tokens; ``stack_gate_up`` builds its stacked expert weight
* ``sparse_matvec_mul_2_4(x, w, cols)`` / ``sparse_matvec_2_4_compressed(x,
  masks, nonzero_values, rows, cols)`` (spanda-engine/src/sparse.rs:19, 100)
  and ``sparse_matvec_mul_2_4_tensor(h, fmt, q, scales, out_features, ...)``
  (sparse_matvec_mul_2_4_tensor_into, src/inference/cpu_engine.rs:1532): the
  2:4 structured-sparse GEMVs; ``register_sparse24`` /
  ``register_sparse24_compressed`` register 2:4 weights for ``gemv``

Where the reference returns ``Err(String)`` this raises :class:`BramhaError`;
``Ok(vec![0; N])`` for an empty input or output becomes a zero array.  When both
``model_name`` and ``layer_name`` are given, the weight is cached on the device
under ``"model:layer"`` (get_or_create_op, :603-722) and later calls skip the
upload.  ``get_cuda_plane()`` mirrors ``get_wgpu_plane()`` (:1710-1728): it
returns ``None`` when ``BRAMHA_CPU`` is set or the device cannot be opened.

The device-pointer methods (``register_dev``, ``gemv_dev``, ``quantize_dev``)
take torch CUDA tensors; torch only supplies memory and streams.
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional, Sequence

import numpy as np

from ._lib import DTYPE, FMT, BramhaError, GemvOp, check, lib

_vp = ctypes.c_void_p


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


class Weight:
    """A weight registered on the device (an opaque `bramha_weight*`)."""

    def __init__(self, plane: "CudaComputePlane", handle: int, key: str, fmt: str, n: int, k: int):
        self.plane, self.handle, self.key, self.fmt, self.N, self.K = plane, handle, key, fmt, n, k
        self.n_full, self.row0 = n, 0  # a column shard holds rows [row0, row0 + N) of n_full

    @property
    def device_bytes(self) -> int:
        nb = ctypes.c_size_t()
        check(lib().bramha_cuda_weight_info(self.handle, None, None, None, ctypes.byref(nb)))
        return nb.value

    def __repr__(self):
        return f"Weight({self.key!r}, {self.fmt}, N={self.N}, K={self.K})"


class CudaComputePlane:
    def __init__(self, device: int = 0):
        ctx = _vp()
        check(lib().bramha_cuda_init(device, ctypes.byref(ctx)))
        self._ctx = ctx
        self.device = device

    # ------------------------------------------------------------------ life
    def close(self):
        if getattr(self, "_ctx", None):
            lib().bramha_cuda_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def ctx(self):
        return self._ctx

    def set_memory_cap(self, nbytes: int):
        check(lib().bramha_cuda_set_memory_cap(self._ctx, nbytes))

    def memory_used(self) -> int:
        v = ctypes.c_size_t()
        check(lib().bramha_cuda_memory_used(self._ctx, ctypes.byref(v)))
        return v.value

    def clear_persistent_buffers(self):
        check(lib().bramha_cuda_clear(self._ctx))

    # ------------------------------------------------------------ registry
    def register(self, key: str, fmt: str, out_features: int, in_features: int, q, scales=None) -> Weight:
        """Upload packed host weights (numpy) under `key` (idempotent)."""
        qa = np.ascontiguousarray(q)
        sa = None if scales is None else _f32(scales)
        h = _vp()
        check(lib().bramha_cuda_register_weight(
            self._ctx, key.encode(), FMT[fmt], out_features, in_features, qa.ctypes.data, qa.nbytes,
            None if sa is None else sa.ctypes.data, 0 if sa is None else sa.size, ctypes.byref(h)))
        return Weight(self, h.value, key, fmt, out_features, in_features)

    def register_dev(self, key: str, fmt: str, out_features: int, in_features: int, q, scales=None,
                     stream=None) -> Weight:
        """Register from torch CUDA tensors (device-to-device copy)."""
        h = _vp()
        check(lib().bramha_cuda_register_weight_dev(
            self._ctx, key.encode(), FMT[fmt], out_features, in_features, q.data_ptr(),
            q.numel() * q.element_size(), None if scales is None else scales.data_ptr(),
            0 if scales is None else scales.numel(), _stream(stream), ctypes.byref(h)))
        return Weight(self, h.value, key, fmt, out_features, in_features)

    def register_sparse24(self, key: str, fmt: str, out_features: int, in_features: int, q, scales=None) -> Weight:
        """Registers a dense f32 / w8 / w4zp8 weight as 2:4 (the top two of every
        group of four columns kept, selected once on the device)."""
        qa = np.ascontiguousarray(q)
        sa = None if scales is None else _f32(scales)
        h = _vp()
        check(lib().bramha_cuda_register_sparse24(
            self._ctx, key.encode(), FMT[fmt], out_features, in_features, qa.ctypes.data, qa.nbytes,
            None if sa is None else sa.ctypes.data, 0 if sa is None else sa.size, ctypes.byref(h)))
        return Weight(self, h.value, key, "sp24_" + fmt, out_features, in_features)

    def register_sparse24_dev(self, key: str, fmt: str, out_features: int, in_features: int, q, scales=None,
                              stream=None) -> Weight:
        h = _vp()
        check(lib().bramha_cuda_register_sparse24_dev(
            self._ctx, key.encode(), FMT[fmt], out_features, in_features, q.data_ptr(),
            q.numel() * q.element_size(), None if scales is None else scales.data_ptr(),
            0 if scales is None else scales.numel(), _stream(stream), ctypes.byref(h)))
        return Weight(self, h.value, key, "sp24_" + fmt, out_features, in_features)

    def register_sparse24_compressed(self, key: str, rows: int, cols: int, masks, nonzero_values) -> Weight:
        """Registers a compressed 2:4 tensor (.spanda BlockSparse2_4: u16 masks
        per group of four, kept values in column order)."""
        m = np.ascontiguousarray(masks, dtype=np.uint16)
        v = _f32(nonzero_values)
        h = _vp()
        check(lib().bramha_cuda_register_sparse24_compressed(self._ctx, key.encode(), rows, cols, m.ctypes.data,
                                                             m.size, v.ctypes.data, v.size, ctypes.byref(h)))
        return Weight(self, h.value, key, "sp24_f32", rows, cols)

    def sparse_matvec_mul_2_4_tensor(self, h, fmt: str, q_weight, scales, out_features: int, model_name=None,
                                     layer_name=None) -> np.ndarray:
        h = _f32(h).reshape(-1)
        qa = np.ascontiguousarray(q_weight)
        sa = None if scales is None else _f32(scales)
        out = np.zeros(out_features, np.float32)
        check(lib().bramha_cuda_sparse_matvec_2_4(
            self._ctx, FMT[fmt], h.ctypes.data, h.size, qa.ctypes.data, qa.nbytes,
            None if sa is None else sa.ctypes.data, 0 if sa is None else sa.size, out_features,
            None if model_name is None else model_name.encode(),
            None if layer_name is None else layer_name.encode(), out.ctypes.data))
        return out

    def sparse_matvec_mul_2_4(self, x, w, cols: int, model_name=None, layer_name=None) -> np.ndarray:
        """sparse.rs:19: rows = len(w) / cols, f32 weights."""
        w = _f32(w).reshape(-1)
        rows = w.size // cols if cols else 0
        return self.sparse_matvec_mul_2_4_tensor(_f32(x)[:cols], "f32", w[:rows * cols], None, rows, model_name,
                                                 layer_name)

    def sparse_matvec_2_4_compressed(self, x, masks, nonzero_values, rows: int, cols: int, model_name=None,
                                     layer_name=None) -> np.ndarray:
        x = _f32(x).reshape(-1)
        if x.size < cols:
            raise BramhaError(-2, f"x has {x.size} elements, expected {cols}")
        m = np.ascontiguousarray(masks, dtype=np.uint16)
        v = _f32(nonzero_values)
        out = np.zeros(rows, np.float32)
        check(lib().bramha_cuda_sparse_matvec_2_4_compressed(
            self._ctx, x.ctypes.data, cols, m.ctypes.data, m.size, v.ctypes.data, v.size, rows,
            None if model_name is None else model_name.encode(),
            None if layer_name is None else layer_name.encode(), out.ctypes.data))
        return out

    def moe_mlp(self, gate_up: Weight, down: Weight, num_experts: int, top_k: int, x, logits):
        """MoE expert MLP of T tokens (run_mlp_into's MoE branch): x [T][H],
        logits [T][E] -> (out [T][H], selected expert ids [T][min(k, E)])."""
        x = _f32(x)
        lg = _f32(logits)
        T = x.shape[0]
        k = min(top_k, num_experts)
        out = np.empty_like(x)
        sel = np.empty((T, k), np.int32)
        check(lib().bramha_cuda_moe_mlp(self._ctx, gate_up.handle, down.handle, num_experts, top_k, x.ctypes.data,
                                        lg.ctypes.data, T, out.ctypes.data, sel.ctypes.data))
        return out, sel

    def moe_mlp_dev(self, gate_up: Weight, down: Weight, num_experts: int, top_k: int, x, logits, out,
                    selected=None, stream=None):
        check(lib().bramha_cuda_moe_mlp_dev(self._ctx, gate_up.handle, down.handle, num_experts, top_k, x.data_ptr(),
                                            logits.data_ptr(), x.shape[0], out.data_ptr(),
                                            None if selected is None else selected.data_ptr(), _stream(stream)))

    def moe_route_dev(self, logits, top_k: int, ids, weights, stream=None):
        """Routing alone: logits [T][E] -> ids [T][k] int32, weights [T][k] f32 (CUDA tensors)."""
        T, E = logits.shape
        check(lib().bramha_cuda_moe_route_dev(self._ctx, logits.data_ptr(), T, E, top_k, ids.data_ptr(),
                                              weights.data_ptr(), _stream(stream)))

    def moe_experts_dev(self, gate_up: Weight, down: Weight, num_experts: int, x, ids, y, stream=None):
        """y[r] = expert ids[r]'s SwiGLU MLP of x[r] (CUDA tensors, x/y [R][H], ids [R] int32)."""
        check(lib().bramha_cuda_moe_experts_dev(self._ctx, gate_up.handle, down.handle, num_experts, x.data_ptr(),
                                                ids.data_ptr(), x.shape[0], y.data_ptr(), _stream(stream)))

    def lookup(self, key: str) -> Weight:
        h = _vp()
        check(lib().bramha_cuda_lookup_weight(self._ctx, key.encode(), ctypes.byref(h)))
        f, n, k = ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64()
        check(lib().bramha_cuda_weight_info(h, ctypes.byref(f), ctypes.byref(n), ctypes.byref(k), None))
        return Weight(self, h.value, key, {v: s for s, v in FMT.items()}[f.value], n.value, k.value)

    def evict(self, key: str):
        check(lib().bramha_cuda_evict_weight(self._ctx, key.encode()))

    # ------------------------------------------------- reference-shaped API
    def _matvec(self, fmt, h, q, scales, out_features, model_name, layer_name):
        h = _f32(h).reshape(-1)
        qa = np.ascontiguousarray(q)
        sa = None if scales is None else _f32(scales)
        out = np.zeros(out_features, np.float32)
        check(lib().bramha_cuda_matvec(
            self._ctx, FMT[fmt], h.ctypes.data, h.size, qa.ctypes.data, qa.nbytes,
            None if sa is None else sa.ctypes.data, 0 if sa is None else sa.size, out_features,
            None if model_name is None else model_name.encode(),
            None if layer_name is None else layer_name.encode(), out.ctypes.data))
        return out

    def matvec_mul(self, h, weight, out_features, model_name: Optional[str] = None,
                   layer_name: Optional[str] = None) -> np.ndarray:
        return self._matvec("f32", h, _f32(weight), None, out_features, model_name, layer_name)

    def matvec_mul_int8(self, h, q_weight, scales, out_features, model_name=None, layer_name=None):
        return self._matvec("w8", h, np.ascontiguousarray(q_weight, np.int8), scales, out_features,
                            model_name, layer_name)

    def matvec_mul_int4(self, h, q_weight, scales, out_features, model_name=None, layer_name=None):
        return self._matvec("w4zp8", h, np.ascontiguousarray(q_weight, np.uint8), scales, out_features,
                            model_name, layer_name)

    def matvec_mul_log4(self, h, q_weight, scales, out_features, model_name=None, layer_name=None):
        return self._matvec("log4", h, np.ascontiguousarray(q_weight, np.uint8), scales, out_features,
                            model_name, layer_name)

    # ------------------------------------------------------- host-buffer ops
    def gemv(self, w: Weight, x) -> np.ndarray:
        """y[b] = W x[b] for x of shape [batch, K] (or [K]); synchronous."""
        x = _f32(x)
        batch = 1 if x.ndim == 1 else x.shape[0]
        if x.size != batch * w.K:
            raise BramhaError(-2, f"input has {x.size} elements, expected {batch} x {w.K}")
        y = np.empty((batch, w.N), np.float32)
        check(lib().bramha_cuda_gemv(self._ctx, w.handle, x.ctypes.data, batch, y.ctypes.data))
        return y.reshape(-1) if x.ndim == 1 else y

    def gemm(self, w: Weight, h_block, block_size: int) -> np.ndarray:
        """gemm_cpu(h_block, weight, block_size, in_features, out_features) -> [M*N]."""
        hb = _f32(h_block).reshape(-1)
        if hb.size != block_size * w.K:
            raise BramhaError(-2, f"h_block has {hb.size} elements, expected {block_size} x {w.K}")
        out = np.empty(block_size * w.N, np.float32)
        check(lib().bramha_cuda_gemm(self._ctx, w.handle, hb.ctypes.data, block_size, out.ctypes.data))
        return out

    # ---------------------------------------------------- device-pointer ops
    def gemv_dev(self, w: Weight, x, y, stream=None):
        """x: CUDA f32 [batch, K]; y: CUDA f32 [batch, N]; stream-ordered."""
        batch = 1 if x.dim() == 1 else x.shape[0]
        check(lib().bramha_cuda_gemv_dev(self._ctx, w.handle, x.data_ptr(), batch, y.data_ptr(), _stream(stream)))

    def gemv_multi_dev(self, ws: Sequence[Weight], x, ys, stream=None):
        n = len(ws)
        harr = (ctypes.c_void_p * n)(*[w.handle for w in ws])
        yarr = (ctypes.c_void_p * n)(*[y.data_ptr() for y in ys])
        batch = 1 if x.dim() == 1 else x.shape[0]
        check(lib().bramha_cuda_gemv_multi_dev(self._ctx, n, harr, x.data_ptr(), batch, yarr, _stream(stream)))

    def gemm_dev(self, w: Weight, x, y, stream=None):
        dt = DTYPE["bf16"] if str(x.dtype) == "torch.bfloat16" else DTYPE["f32"]
        check(lib().bramha_cuda_gemm_dev(self._ctx, w.handle, x.data_ptr(), dt, x.shape[0], y.data_ptr(),
                                         _stream(stream)))

    def gemv_rmsnorm_dev(self, ws: Sequence[Weight], x, delta, norm_w, eps: float, x_out, ys, stream=None):
        """ys[i] = W_i rms_norm(x + delta) * norm_w at batch 1, with x + delta stored
        to x_out (None: not stored; it must not overlap x or delta); delta may be
        None.  One launch when the CUDA-core GEMV takes the weights."""
        n = len(ws)
        harr = (ctypes.c_void_p * n)(*[w.handle for w in ws])
        yarr = (ctypes.c_void_p * n)(*[y.data_ptr() for y in ys])
        check(lib().bramha_cuda_gemv_rmsnorm_dev(self._ctx, n, harr, x.data_ptr(), _ptr_or_none(delta),
                                                 norm_w.data_ptr(), float(eps), _ptr_or_none(x_out), yarr,
                                                 _stream(stream)))

    def gemv_swiglu_dev(self, w: Weight, gate, up, y, stream=None):
        """y = W (silu(gate) * up), one launch (CUDA f32 tensors [batch][K])."""
        batch = 1 if gate.dim() == 1 else gate.shape[0]
        check(lib().bramha_cuda_gemv_swiglu_dev(self._ctx, w.handle, gate.data_ptr(), up.data_ptr(), batch,
                                                y.data_ptr(), _stream(stream)))

    GEMV_KERNELS = {"auto": 0, "tensor_core": 1, "cuda_core": 2}

    def set_gemv_kernel(self, kind: str = "auto"):
        """'auto' (default), 'tensor_core' or 'cuda_core' for the quantized GEMVs."""
        check(lib().bramha_cuda_set_gemv_kernel(self._ctx, self.GEMV_KERNELS[kind]))

    TEST_FAULTS = {"none": 0, "gemv": 1, "gemm": 2}

    def set_wait_timeout(self, ns: int = 0):
        """Bound on every device-side wait of the tensor-core kernels (0 = the 2 s default)."""
        check(lib().bramha_cuda_set_wait_timeout(self._ctx, int(ns)))

    def test_fault(self, kind: str = "none"):
        """TEST ONLY: CTA 0 of later tensor-core GEMV ('gemv') or GEMM ('gemm')
        launches withholds one weight copy, so a bounded wait runs out."""
        check(lib().bramha_cuda_test_fault(self._ctx, self.TEST_FAULTS[kind]))

    def set_prefetch(self, lookahead_bytes: int = 0, next_launch_bytes: int = 8 << 20):
        """L2 prefetch of the tensor-core GEMV (tuning only; results do not change)."""
        check(lib().bramha_cuda_set_prefetch(self._ctx, int(lookahead_bytes), int(next_launch_bytes)))

    TUNING = {"lookahead_bytes": 1, "next_launch_bytes": 2, "evict_first": 3, "split_cost": 4,
              "program_lookahead_bytes": 5, "cc_split_depth": 6}

    def set_gemv_tuning(self, **kw):
        """GEMV tuning: lookahead_bytes, next_launch_bytes, evict_first (0/1),
        split_cost, program_lookahead_bytes (tensor-core GEMV; results do not
        change) and cc_split_depth (CUDA-core GEMV; fp32 grouping only)."""
        for k, v in kw.items():
            check(lib().bramha_cuda_set_gemv_tuning(self._ctx, self.TUNING[k], int(v)))

    @staticmethod
    def _chain_ops(ops):
        """[(weights, x, ys[, x_up])] -> (GemvOp array, keep-alive list); x / ys / x_up
        are torch tensors or numpy arrays (pointers taken as they are)."""
        arr = (GemvOp * len(ops))()
        keep = []
        for i, op in enumerate(ops):
            ws, x, ys = op[0], op[1], op[2]
            up = op[3] if len(op) > 3 else None
            wa = (ctypes.c_void_p * len(ws))(*[w.handle for w in ws])
            ya = (ctypes.c_void_p * len(ys))(*[_ptr(y) for y in ys])
            keep += [wa, ya]
            arr[i].n_weights = len(ws)
            arr[i].weights = ctypes.cast(wa, ctypes.POINTER(ctypes.c_void_p))
            arr[i].x = _ptr(x)
            arr[i].x_up = None if up is None else _ptr(up)
            arr[i].y = ctypes.cast(ya, ctypes.POINTER(ctypes.c_void_p))
        return arr, keep

    def gemv_chain_dev(self, ops, batch: int = 1, stream=None):
        """A chain of dependent GEMV launches on CUDA tensors: ops = [(weights, x, ys)
        or (weights, x, ys, x_up)]; launch i prefetches launch i+1's weights into L2."""
        arr, keep = self._chain_ops(ops)
        check(lib().bramha_cuda_gemv_chain_dev(self._ctx, len(ops), arr, batch, _stream(stream)))
        del keep

    def gemv_program(self, ops, batch: int = 1) -> "GemvProgram":
        """The chain `ops` (as gemv_chain_dev takes it) as one persistent launch;
        the ops' tensors are bound now and must outlive the program."""
        return GemvProgram(self, ops, batch)

    def gemv_chain(self, ops, batch: int = 1):
        """The same chain on host buffers (numpy arrays or pinned torch CPU tensors):
        inputs copied in, the chain run, outputs copied back; synchronous.  The
        copies run on their own streams, overlapping the launches block by block."""
        _check_host_buffers(ops)
        arr, keep = self._chain_ops(ops)
        check(lib().bramha_cuda_gemv_chain(self._ctx, len(ops), arr, batch))
        del keep

    def prepare_chain(self, ops, batch: int = 1) -> "HostGemvChain":
        """gemv_chain on fixed host buffers, bound once (bramha_cuda_host_chain_*):
        each run() copies the buffers' current contents in and the outputs back;
        with pinned buffers the copies and launches replay as one CUDA graph."""
        return HostGemvChain(self, ops, batch)

    def stream_sync(self, stream=None):
        """Wait for the stream and raise if a kernel reported a device-side failure."""
        check(lib().bramha_cuda_stream_sync(self._ctx, _stream(stream)))

    def quantize_dev(self, fmt: str, w, q, scales, stream=None):
        n, k = w.shape
        check(lib().bramha_cuda_quantize_dev(self._ctx, FMT[fmt], n, k, w.data_ptr(), q.data_ptr(),
                                             scales.data_ptr(), _stream(stream)))


def _check_host_buffers(ops):
    for op in ops:
        for a in (op[1],) + tuple(op[2]) + ((op[3],) if len(op) > 3 and op[3] is not None else ()):
            if isinstance(a, np.ndarray) and (a.dtype != np.float32 or not a.flags.c_contiguous):
                raise BramhaError(-1, "gemv_chain: host buffers must be contiguous float32")


class HostGemvChain:
    """A host-buffer GEMV chain bound once (bramha_cuda_host_chain_*); the host
    buffers are held here and keep their addresses while it exists."""

    def __init__(self, plane: "CudaComputePlane", ops, batch: int = 1):
        _check_host_buffers(ops)
        self.plane, self.batch, self._ops, self.handle = plane, batch, ops, None
        arr, keep = CudaComputePlane._chain_ops(ops)
        h = ctypes.c_void_p()
        check(lib().bramha_cuda_host_chain_create(plane.ctx, len(ops), arr, batch, ctypes.byref(h)))
        self.handle = h.value

    def run(self):
        check(lib().bramha_cuda_host_chain_run(self.plane.ctx, self.handle))

    def uses_graph(self) -> bool:
        g = ctypes.c_int()
        check(lib().bramha_cuda_host_chain_uses_graph(self.plane.ctx, self.handle, ctypes.byref(g)))
        return bool(g.value)

    def close(self):
        if self.handle is not None and self.plane.ctx:
            lib().bramha_cuda_host_chain_destroy(self.plane.ctx, self.handle)
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GemvProgram:
    """A chain of GEMVs run as one persistent launch (bramha_cuda_gemv_program_*)."""

    def __init__(self, plane: "CudaComputePlane", ops, batch: int = 1):
        arr, keep = CudaComputePlane._chain_ops(ops)
        h = ctypes.c_void_p()
        check(lib().bramha_cuda_gemv_program_create(plane.ctx, len(ops), arr, batch, ctypes.byref(h)))
        self.plane, self.handle, self._ops = plane, h.value, ops

    def run(self, stream=None):
        check(lib().bramha_cuda_gemv_program_run_dev(self.plane.ctx, self.handle, _stream(stream)))

    def trace(self, on: bool = True):
        """Record per-op, per-CTA timestamps in the next runs."""
        check(lib().bramha_cuda_gemv_program_trace(self.plane.ctx, self.handle, int(on)))

    def read_trace(self) -> np.ndarray:
        """[n_ops][grid][8] %globaltimer stamps (ns) of the last traced run: op
        reached, previous op finished everywhere, B area free, activations loaded,
        terms built, last accumulator ready, outputs stored, completion published."""
        n = len(self._ops) * 1024 * 8
        buf = np.zeros(n, np.uint64)
        g = ctypes.c_int()
        check(lib().bramha_cuda_gemv_program_read_trace(self.plane.ctx, self.handle, buf.ctypes.data, n,
                                                        ctypes.byref(g)))
        return buf[:len(self._ops) * g.value * 8].reshape(len(self._ops), g.value, 8)

    def close(self):
        if self.handle:
            lib().bramha_cuda_gemv_program_destroy(self.plane.ctx, self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _ptr(a) -> int:
    """Address of a torch tensor's or numpy array's data."""
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


def _ptr_or_none(a) -> Optional[int]:
    return None if a is None else _ptr(a)


_STREAM_LEGACY = 0x1  # cudaStreamLegacy: the legacy default stream, valid in any CUDA runtime


def _stream(stream) -> Optional[int]:
    """The cudaStream_t to pass: torch's current stream unless one is given.

    torch's default stream has handle 0, which the C ABI reads as "the
    context's own stream" -- a different, non-blocking stream.  The legacy
    default stream is passed explicitly instead so the call stays ordered
    after torch's work on that stream.
    """
    if stream is None:
        try:
            import torch
            if torch.cuda.is_available():
                stream = torch.cuda.current_stream()
        except Exception:
            return None
        if stream is None:
            return None
    handle = getattr(stream, "cuda_stream", stream)
    return _STREAM_LEGACY if handle == 0 else handle


_PLANES: dict = {}
_PLANES_LOCK = threading.Lock()


def get_cuda_plane(device: int = 0) -> Optional[CudaComputePlane]:
    """Process-wide plane for `device`, or None (BRAMHA_CPU set / init failed)."""
    if os.environ.get("BRAMHA_CPU") is not None:
        return None
    with _PLANES_LOCK:
        if device not in _PLANES:
            try:
                _PLANES[device] = CudaComputePlane(device)
            except (BramhaError, RuntimeError):
                _PLANES[device] = None
        return _PLANES[device]


def packed_nbytes(fmt: str, n: int, k: int) -> int:
    return {"f32": n * k * 4, "w8": n * k, "w4zp8": n * (k // 2), "log4": n * (k // 2)}[fmt]


def stack_gate_up(gates, ups):
    """Per-expert packed gate and up weights [(q, scales)] -> the stacked
    gate_up layout of the MoE call: expert e's gate rows, then its up rows."""
    qs, ss = [], []
    for (gq, gs), (uq, us) in zip(gates, ups):
        qs += [np.ascontiguousarray(gq).reshape(-1).view(np.uint8), np.ascontiguousarray(uq).reshape(-1).view(np.uint8)]
        ss += [_f32(gs), _f32(us)]
    return np.concatenate(qs), np.concatenate(ss)
