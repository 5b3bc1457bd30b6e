"""B200-native (sm_100a) dequantize-fused linear-layer path for Bramha.

The product is the C ABI in ``include/bramha_cuda.h`` (``libbramha_cuda.so``,
built by ``python -m bramha_b200.build``); this package is its Python host
side, mirroring the reference's compute-plane interface.
"""
from ._lib import FMT, BramhaError, header_symbols, last_error, lib
from .plane import CudaComputePlane, GemvProgram, HostGemvChain, Weight, get_cuda_plane, packed_nbytes, stack_gate_up
from .decode import DecodeConfig, DecodeLayer, DecodeModel
from .sharded import ShardedPlane, gather_rows, shard_rows, shard_slab

__all__ = [
    "FMT", "BramhaError", "CudaComputePlane", "DecodeConfig", "DecodeLayer", "DecodeModel", "GemvProgram",
    "HostGemvChain", "Weight",
    "get_cuda_plane", "header_symbols", "last_error", "lib", "packed_nbytes", "stack_gate_up",
    "ShardedPlane", "gather_rows", "shard_rows", "shard_slab",
]
