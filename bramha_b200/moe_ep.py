"""Expert-parallel MoE layer: the experts of a layer spread over the ranks of a
process group, tokens kept on the rank that owns them.

The reference runs every routed expert of a token on one CPU
(run_mlp_into's MoE branch, src/inference/cpu_engine.rs:1799-1989).  Here
rank r holds experts [r E/W, (r+1) E/W) and, for its own T tokens:

1. routes them (softmax, stable top-k: ``route_fn``);
2. dispatches: the (token, choice) pairs with a positive weight, grouped by
   the rank owning the expert (token order inside each group), go out with
   one ``all_to_all_single`` of activations and one of local expert ids, after
   an ``all_to_all_single`` of the pair counts (the sizes of the exchanges: the
   layer's only host synchronisation);
3. computes its experts on the rows it received (``experts_fn``);
4. returns the expert outputs with the reverse ``all_to_all_single``;
5. combines: out[t] = sum over j of y(t, j) * weight[t][j] in the sorted
   order, skipping weights <= 0, one rounding per product and per sum from 0
   (cpu_engine.rs:1944-1946).

The exchange is NCCL over NVLink on GPUs (the backend of the process group);
the same code runs on ``gloo`` with CPU tensors, which is how its host logic is
tested.  Every rank takes the same collective steps in the same order.
"""
from __future__ import annotations

from typing import Callable, Tuple

import torch
import torch.distributed as dist


class ExpertParallelMoE:
    def __init__(self, num_experts: int, top_k: int, route_fn: Callable, experts_fn: Callable, group=None):
        """route_fn(logits [T][E]) -> (ids [T][k] int32, weights [T][k] f32);
        experts_fn(x [R][H], local_ids [R] int32) -> y [R][H] for this rank's
        experts (local ids 0 .. E/W - 1)."""
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split over {self.world} ranks")
        self.E, self.k = num_experts, top_k
        self.e_local = num_experts // self.world
        self.route_fn, self.experts_fn = route_fn, experts_fn

    def expert_range(self) -> Tuple[int, int]:
        return self.rank * self.e_local, (self.rank + 1) * self.e_local

    def forward(self, x: torch.Tensor, logits: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        dev = x.device
        ids, w = self.route_fn(logits)
        k = ids.shape[1]
        valid = w > 0
        dest = torch.where(valid, ids.long() // self.e_local, torch.full_like(ids, self.world, dtype=torch.long))
        flat_dest = dest.reshape(-1)
        order = torch.argsort(flat_dest, stable=True)           # grouped by rank, (t, j) order inside
        # pairs per destination rank (index world: skipped pairs, sorted last)
        send_counts = torch.bincount(flat_dest, minlength=self.world + 1)[:self.world].to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        counts = torch.cat([send_counts, recv_counts]).tolist()  # the layer's one host synchronisation
        send_splits, recv_splits = counts[:self.world], counts[self.world:]
        n_send, n_recv = sum(send_splits), sum(recv_splits)
        order = order[:n_send]
        send_x = x.index_select(0, order // k).contiguous()
        send_e = (ids.reshape(-1).long()[order] - flat_dest[order] * self.e_local).to(torch.int32).contiguous()
        recv_x = torch.empty((n_recv, H), dtype=x.dtype, device=dev)
        recv_e = torch.empty(n_recv, dtype=torch.int32, device=dev)
        dist.all_to_all_single(recv_x, send_x, recv_splits, send_splits, group=self.group)
        dist.all_to_all_single(recv_e, send_e, recv_splits, send_splits, group=self.group)
        y_recv = self.experts_fn(recv_x, recv_e) if n_recv else torch.empty((0, H), dtype=x.dtype, device=dev)
        y_back = torch.empty((n_send, H), dtype=x.dtype, device=dev)
        dist.all_to_all_single(y_back, y_recv.contiguous(), send_splits, recv_splits, group=self.group)
        y_pairs = torch.zeros((T * k, H), dtype=x.dtype, device=dev)
        y_pairs.index_copy_(0, order, y_back)
        y_pairs = y_pairs.view(T, k, H)
        out = torch.zeros((T, H), dtype=x.dtype, device=dev)
        for j in range(k):
            prod = y_pairs[:, j] * w[:, j:j + 1]
            out = torch.where(valid[:, j:j + 1], out + prod, out)
        return out


def cuda_moe_fns(plane, gate_up_local, down_local, e_local: int, top_k: int):
    """route_fn / experts_fn on the CUDA plane: routing by
    bramha_cuda_moe_route_dev, the local experts by bramha_cuda_moe_experts_dev
    (gate_up_local / down_local: this rank's stacked expert weights)."""

    def route_fn(logits):
        T, E = logits.shape
        k = min(top_k, E)
        ids = torch.empty((T, k), dtype=torch.int32, device=logits.device)
        w = torch.empty((T, k), dtype=torch.float32, device=logits.device)
        plane.moe_route_dev(logits.contiguous(), top_k, ids, w)
        return ids, w

    def experts_fn(x, ids):
        y = torch.empty_like(x)
        plane.moe_experts_dev(gate_up_local, down_local, e_local, x, ids, y)
        return y

    return route_fn, experts_fn
