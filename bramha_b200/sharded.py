"""Column sharding of the quantized linears across the GPUs of one node.

The reference runs every linear on one device (`matvec_mul_into`,
src/inference/cpu_engine.rs:1307-1444; its GPU plane is a single
`WgpuComputePlane`, src/compute/wgpu_backend.rs:1707-1728).  Here a linear's
output rows are split across ranks, one process and one `CudaComputePlane` per
GPU: rank r holds rows ``[N*r//world, N*(r+1)//world)`` of each sharded weight.
A GEMV on sharded weights computes this rank's rows and its epilogue stores
them, over NVLink, into every rank's copy of the full output (a symmetric
arena allocated on every rank; the all-gather is part of the GEMV), then
publishes the launch; the next sharded GEMV waits (bounded) for every rank's
publication before it reads its input.  The process group is used once, to
exchange the arenas' IPC handles; no collective runs on the data path.

:class:`ShardedPlane` owns that set-up.  The row split and the packed-row
slicing are plain functions (:func:`shard_rows`, :func:`shard_slab`) so the
host logic can be checked without a GPU.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import numpy as np

from ._lib import check, lib
from .plane import CudaComputePlane, Weight, _stream


class IpcHandle(ctypes.Structure):
    """`bramha_ipc_handle` of include/bramha_cuda.h."""
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


def shard_rows(n: int, world: int, rank: int):
    """(first row, row count) of rank `rank`'s shard of an n-row weight -- the
    split bramha_cuda_shard_rows makes."""
    r0 = n * rank // world
    return r0, n * (rank + 1) // world - r0


def shard_slab(fmt: str, q, scales, n: int, k: int, world: int, rank: int):
    """This rank's packed rows and scales of a row-major packed weight."""
    r0, rows = shard_rows(n, world, rank)
    rb = {"w8": k, "w4zp8": k // 2, "log4": k // 2}[fmt]
    qa = np.ascontiguousarray(q).reshape(-1)
    return qa[r0 * rb:(r0 + rows) * rb], np.asarray(scales, np.float32)[r0:r0 + rows]


def gather_rows(shards: Sequence[np.ndarray]) -> np.ndarray:
    """The full output from every rank's rows, in rank order (what the sharded
    GEMV's epilogue assembles in every rank's copy)."""
    return np.concatenate([np.asarray(s, np.float32) for s in shards], axis=-1)


class _CudaArray:
    def __init__(self, ptr: int, shape, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class ShardedPlane:
    """A rank of a column-shard group on top of a :class:`CudaComputePlane`."""

    def __init__(self, plane: CudaComputePlane, group=None, arena_bytes: int = 256 << 20):
        import torch.distributed as dist
        self.plane = plane
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        h = IpcHandle()
        check(lib().bramha_cuda_shard_handle(plane.ctx, arena_bytes, ctypes.byref(h)))
        mine = bytes(h.bytes)
        allh = [None] * self.world
        dist.all_gather_object(allh, mine, group=group)
        arr = (IpcHandle * self.world)()
        for r, b in enumerate(allh):
            arr[r].bytes[:] = list(b)
        check(lib().bramha_cuda_shard_init(plane.ctx, self.world, self.rank, arr))

    def rows(self, n: int):
        return shard_rows(n, self.world, self.rank)

    def _weight(self, h, key, fmt, n, k) -> Weight:
        r0, rows = self.rows(n)
        w = Weight(self.plane, h, key, fmt, rows, k)
        w.n_full, w.row0 = n, r0
        return w

    def register(self, key: str, fmt: str, out_features: int, in_features: int, q, scales) -> Weight:
        """This rank's rows of a full packed host weight."""
        qa = np.ascontiguousarray(q)
        sa = np.ascontiguousarray(scales, np.float32)
        h = ctypes.c_void_p()
        check(lib().bramha_cuda_register_weight_shard(
            self.plane.ctx, key.encode(), {"w8": 1, "w4zp8": 2, "log4": 3}[fmt], out_features, in_features,
            qa.ctypes.data, qa.nbytes, sa.ctypes.data, sa.size, ctypes.byref(h)))
        return self._weight(h.value, key, fmt, out_features, in_features)

    def register_dev(self, key: str, fmt: str, out_features: int, in_features: int, q, scales,
                     stream=None) -> Weight:
        """This rank's rows of a full packed weight held in device memory (torch)."""
        h = ctypes.c_void_p()
        check(lib().bramha_cuda_register_weight_shard_dev(
            self.plane.ctx, key.encode(), {"w8": 1, "w4zp8": 2, "log4": 3}[fmt], out_features, in_features,
            q.data_ptr(), q.numel() * q.element_size(), scales.data_ptr(), scales.numel(), _stream(stream),
            ctypes.byref(h)))
        return self._weight(h.value, key, fmt, out_features, in_features)

    def empty(self, shape, device: Optional[int] = None):
        """A float32 tensor in the symmetric arena (allocate in the same order and
        sizes on every rank); sharded GEMV outputs must live here."""
        import torch
        n = int(np.prod(shape))
        p = ctypes.c_void_p()
        check(lib().bramha_cuda_shard_malloc(self.plane.ctx, 4 * n, ctypes.byref(p)))
        dev = self.plane.device if device is None else device
        return torch.as_tensor(_CudaArray(p.value, shape), device=f"cuda:{dev}")

    def sync(self, stream=None):
        """Stream-ordered: later work sees every rank's rows of every sharded GEMV issued so far."""
        check(lib().bramha_cuda_shard_sync_dev(self.plane.ctx, _stream(stream)))

    def gemv(self, w: Weight, x) -> np.ndarray:
        """Host buffers: the full output [batch][N] of a sharded weight (every rank calls it)."""
        x = np.ascontiguousarray(x, np.float32)
        batch = 1 if x.ndim == 1 else x.shape[0]
        y = np.empty((batch, w.n_full), np.float32)
        check(lib().bramha_cuda_gemv(self.plane.ctx, w.handle, x.ctypes.data, batch, y.ctypes.data))
        return y.reshape(-1) if x.ndim == 1 else y
