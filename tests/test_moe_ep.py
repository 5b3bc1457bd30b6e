"""Expert-parallel MoE (bramha_b200/moe_ep.py): the dispatch / expert / combine
logic across ranks, checked against the oracle's single-process restatement of
run_mlp_into's MoE branch (cpu_engine.rs:1799-1989).

CPU: two `gloo` ranks on 127.0.0.1, the experts computed by the oracle's GEMVs
(every rank holds half of the experts, tokens stay on their rank).  GPU
(2 devices or more): two NCCL ranks, the experts on the CUDA plane.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle

E, H, I, K, T_RANK = 8, 256, 128, 3, 10


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def make_model(fmt="log4", seed=3, all_rank0=False):
    r = np.random.Generator(np.random.PCG64(seed))
    mk = lambda n, k: oracle.quantize(fmt, r.normal(0, 0.02, n * k).astype(np.float32), n, k)
    gates = [mk(I, H) for _ in range(E)]
    ups = [mk(I, H) for _ in range(E)]
    downs = [mk(H, I) for _ in range(E)]
    x = r.normal(0, 1, (2 * T_RANK, H)).astype(np.float32)
    lg = r.normal(0, 1, (2 * T_RANK, E)).astype(np.float32)
    lg[3] = np.array([0, -200, 50, -200, -200, -200, -200, -200], np.float32)  # weights that underflow: skipped
    lg[T_RANK:, 0] += 8.0  # the second rank's tokens all go first to expert 0 (rank 0)
    if all_rank0:  # every choice on rank 0's experts: rank 1 receives no rows at all
        lg[:, E // 2:] -= 200.0
    return gates, ups, downs, x, lg


def cat(ws):
    return np.concatenate([q.view(np.uint8) for q, _ in ws]), np.concatenate([s for _, s in ws])


def cpu_worker(rank, world, port, out_dir, all_rank0=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from bramha_b200.moe_ep import ExpertParallelMoE
        gates, ups, downs, x, lg = make_model(all_rank0=all_rank0)
        e_local = E // world
        xs, ls = x[rank * T_RANK:(rank + 1) * T_RANK], lg[rank * T_RANK:(rank + 1) * T_RANK]
        ref, ref_ids, ref_w = oracle.moe_mlp("log4", xs, ls, K, cat(gates), cat(ups), cat(downs))

        def route_fn(logits):
            _, ids, w = oracle.moe_mlp("log4", xs, logits.numpy(), K, cat(gates), cat(ups), cat(downs))
            return torch.from_numpy(ids), torch.from_numpy(w)

        def experts_fn(xr, ids):
            y = np.empty(xr.shape, np.float32)
            for r, (row, le) in enumerate(zip(xr.numpy(), ids.numpy())):
                e = rank * e_local + int(le)
                g = oracle.matvec_mul_into("log4", row, gates[e][0], gates[e][1], I)
                u = oracle.matvec_mul_into("log4", row, ups[e][0], ups[e][1], I)
                m = (g / (np.float32(1) + np.exp(-g)) * u).astype(np.float32)
                y[r] = oracle.matvec_mul_into("log4", m, downs[e][0], downs[e][1], H)
            return torch.from_numpy(y)

        moe = ExpertParallelMoE(E, K, route_fn, experts_fn)
        out = moe.forward(torch.from_numpy(xs), torch.from_numpy(ls)).numpy()
        np.save(os.path.join(out_dir, f"out{rank}.npy"), out)
        np.save(os.path.join(out_dir, f"ref{rank}.npy"), ref)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("all_rank0", [False, True])
def test_expert_parallel_two_ranks_gloo(tmp_path, all_rank0):
    port = free_port()
    mp.start_processes(cpu_worker, args=(2, port, str(tmp_path), all_rank0), nprocs=2, join=True,
                       start_method="spawn")
    for rank in range(2):
        out, ref = np.load(tmp_path / f"out{rank}.npy"), np.load(tmp_path / f"ref{rank}.npy")
        assert np.max(np.abs(out - ref)) <= 1e-5 * np.max(np.abs(ref)), rank


def gpu_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from bramha_b200 import CudaComputePlane, stack_gate_up
        from bramha_b200.moe_ep import ExpertParallelMoE, cuda_moe_fns
        gates, ups, downs, x, lg = make_model()
        e_local = E // world
        mine = range(rank * e_local, (rank + 1) * e_local)
        plane = CudaComputePlane(rank)
        gq, gs = stack_gate_up([gates[e] for e in mine], [ups[e] for e in mine])
        dq, ds = cat([downs[e] for e in mine])
        gu = plane.register("ep:gu", "log4", e_local * 2 * I, H, gq, gs)
        dn = plane.register("ep:dn", "log4", e_local * H, I, dq, ds)
        moe = ExpertParallelMoE(E, K, *cuda_moe_fns(plane, gu, dn, e_local, K))
        dev = torch.device("cuda", rank)
        xs = torch.from_numpy(x[rank * T_RANK:(rank + 1) * T_RANK]).to(dev)
        ls = torch.from_numpy(lg[rank * T_RANK:(rank + 1) * T_RANK]).to(dev)
        out = moe.forward(xs, ls)
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"gout{rank}.npy"), out.cpu().numpy())
        dist.barrier()
        plane.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_expert_parallel_two_gpus_nccl(tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    port = free_port()
    mp.start_processes(gpu_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    gates, ups, downs, x, lg = make_model()
    ref, _, _ = oracle.moe_mlp("log4", x, lg, K, cat(gates), cat(ups), cat(downs))
    out = np.concatenate([np.load(tmp_path / f"gout{r}.npy") for r in range(2)])
    assert np.max(np.abs(out - ref)) <= 1e-3 * np.max(np.abs(ref))
