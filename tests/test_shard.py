"""Column sharding of a linear's output rows across ranks (bramha_b200/sharded.py,
the bramha_cuda_shard_* calls of include/bramha_cuda.h), against the oracle's
`matvec_mul_into` (src/inference/cpu_engine.rs:1307-1444) on the whole weight.

CPU: `gloo` ranks on 127.0.0.1 check the host logic -- the row split
(shard_rows), the packed-row slicing (shard_slab) and the rank-order assembly
(gather_rows): every rank computes its rows with the oracle, the rows are
all-gathered, and the result must equal the oracle's whole GEMV bit for bit
(rows are independent), with uneven N and N < world.

GPU (two devices): two NCCL ranks (NVLS off), each a CudaComputePlane with a
ShardedPlane; the sharded GEMV's epilogue stores each rank's rows into both
ranks' copies of the output over NVLink.  Checked: the Qwen2-7B lm_head at
full size, two chained sharded GEMVs (the second reads the first's output),
uneven N and N < world, the host-buffer call, and a rank that stops issuing
sharded GEMVs: the other rank's bounded wait runs out and reports
BRAMHA_ERR_TIMEOUT (no fault, no hang).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from bramha_b200.sharded import gather_rows, shard_rows, shard_slab

SHAPES = [("log4", 1001, 256), ("w4zp8", 1, 128), ("w8", 300, 130), ("log4", 2, 64)]


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def weight(fmt, n, k, seed):
    r = np.random.Generator(np.random.PCG64(seed))
    q, s = oracle.quantize(fmt, r.normal(0, 0.02, n * k).astype(np.float32), n, k)
    x = r.normal(0, 1, k).astype(np.float32)
    return q, s, x


def test_shard_rows_cover_every_row_once():
    for n in (0, 1, 2, 7, 1001, 152064):
        for world in (2, 3, 4, 8):
            spans = [shard_rows(n, world, r) for r in range(world)]
            assert spans[0][0] == 0
            for (a0, an), (b0, _) in zip(spans, spans[1:]):
                assert a0 + an == b0
            assert sum(c for _, c in spans) == n
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1


def cpu_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        for i, (fmt, n, k) in enumerate(SHAPES):
            q, s, x = weight(fmt, n, k, seed=i)
            qs, ss = shard_slab(fmt, q, s, n, k, world, rank)
            rows = shard_rows(n, world, rank)[1]
            mine = oracle.matvec_mul_into(fmt, x, qs, ss, rows) if rows else np.zeros(0, np.float32)
            parts = [None] * world
            dist.all_gather_object(parts, mine)
            np.save(os.path.join(out_dir, f"y{i}_{rank}.npy"), gather_rows(parts))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_shard_and_gather_host_logic_gloo(tmp_path, world):
    port = free_port()
    mp.start_processes(cpu_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True, start_method="spawn")
    for i, (fmt, n, k) in enumerate(SHAPES):
        q, s, x = weight(fmt, n, k, seed=i)
        ref = oracle.matvec_mul_into(fmt, x, q, s, n)
        for r in range(world):
            y = np.load(tmp_path / f"y{i}_{r}.npy")
            assert y.tobytes() == ref.tobytes(), (fmt, n, k, r)


# ---------------------------------------------------------------------- GPU
def gpu_worker(rank, world, port, out_dir, case):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    plane = None
    try:
        from bramha_b200 import BramhaError, CudaComputePlane, ShardedPlane
        plane = CudaComputePlane(rank)
        sp = ShardedPlane(plane, arena_bytes=64 << 20)
        if case == "parity":
            # the Qwen2-7B lm_head, generated and packed on the device identically on both ranks
            n, k = 152064, 3584
            g = torch.Generator(device=dev).manual_seed(77)
            wf = torch.randn((n, k), generator=g, device=dev) * 0.02
            qd = torch.empty(n * k // 2, dtype=torch.uint8, device=dev)
            sd = torch.empty(n, dtype=torch.float32, device=dev)
            plane.quantize_dev("log4", wf, qd, sd)
            del wf
            w = sp.register_dev("lm7", "log4", n, k, qd, sd)
            x = torch.from_numpy(np.random.Generator(np.random.PCG64(5)).normal(0, 1, (1, k)).astype(np.float32)).to(dev)
            y = sp.empty((1, n))
            plane.gemv_dev(w, x, y)
            # two chained sharded GEMVs: the second reads the first's full output
            q1, s1, _ = weight("log4", 3584, 3584, seed=11)
            q2, s2, _ = weight("w8", 1001, 3584, seed=12)
            w1 = sp.register("c1", "log4", 3584, 3584, q1, s1)
            w2 = sp.register("c2", "w8", 1001, 3584, q2, s2)
            x1 = torch.from_numpy(np.random.Generator(np.random.PCG64(6)).normal(0, 1, (2, 3584)).astype(np.float32)).to(dev)
            y1, y2 = sp.empty((2, 3584)), sp.empty((2, 1001))
            plane.gemv_chain_dev([([w1], x1, [y1]), ([w2], y1, [y2])], batch=2)
            # N < world: one row
            q3, s3, x3 = weight("w4zp8", 1, 256, seed=13)
            w3 = sp.register("c3", "w4zp8", 1, 256, q3, s3)
            y3 = sp.empty((1, 1))
            plane.gemv_dev(w3, torch.from_numpy(x3[None, :]).to(dev), y3)
            sp.sync()
            plane.stream_sync()
            np.save(os.path.join(out_dir, f"lm{rank}.npy"), y.cpu().numpy())
            np.save(os.path.join(out_dir, f"y1_{rank}.npy"), y1.cpu().numpy())
            np.save(os.path.join(out_dir, f"y2_{rank}.npy"), y2.cpu().numpy())
            np.save(os.path.join(out_dir, f"y3_{rank}.npy"), y3.cpu().numpy())
            if rank == 0:
                np.save(os.path.join(out_dir, "lm_q.npy"), qd.cpu().numpy())
                np.save(os.path.join(out_dir, "lm_s.npy"), sd.cpu().numpy())
                np.save(os.path.join(out_dir, "lm_x.npy"), x.cpu().numpy())
                np.save(os.path.join(out_dir, "x1.npy"), x1.cpu().numpy())
            # host buffers: every rank gets the full output
            yh = sp.gemv(w2, x1.cpu().numpy())
            np.save(os.path.join(out_dir, f"yh_{rank}.npy"), yh)
            # a host chain bound once over a sharded weight: each run is a per-call chain
            yb = np.full((2, 1001), np.nan, np.float32)
            hc = plane.prepare_chain([([w2], x1.cpu().numpy(), [yb])], batch=2)
            assert not hc.uses_graph()
            hc.run()
            hc.close()
            np.save(os.path.join(out_dir, f"yb_{rank}.npy"), yb)
        elif case == "stop":
            q1, s1, x1 = weight("log4", 512, 1024, seed=21)
            w1 = sp.register("s1", "log4", 512, 1024, q1, s1)
            xd = torch.from_numpy(x1[None, :]).to(dev)
            y = sp.empty((1, 512))
            plane.gemv_dev(w1, xd, y)
            sp.sync()
            plane.stream_sync()
            status = "ok"
            if rank == 0:  # rank 1 issues no second GEMV: rank 0's wait for it must run out
                plane.set_wait_timeout(50_000_000)
                plane.gemv_dev(w1, xd, y)
                sp.sync()
                try:
                    plane.stream_sync()
                    status = "no error"
                except BramhaError as e:
                    status = "timeout" if e.code == -7 else f"code {e.code}"
            np.save(os.path.join(out_dir, f"stop{rank}.npy"), np.array([status]))
        dist.barrier()
    finally:
        if plane is not None:
            plane.close()
        dist.destroy_process_group()


def two_gpus():
    return torch.cuda.is_available() and torch.cuda.device_count() >= 2


@pytest.mark.gpu
def test_sharded_gemv_two_gpus(tmp_path):
    if not two_gpus():
        pytest.skip("needs two GPUs")
    mp.start_processes(gpu_worker, args=(2, free_port(), str(tmp_path), "parity"), nprocs=2, join=True,
                       start_method="spawn")
    from tests._util import GEMV_TOL, normwise_err
    q, s, x = np.load(tmp_path / "lm_q.npy"), np.load(tmp_path / "lm_s.npy"), np.load(tmp_path / "lm_x.npy")
    ref = oracle.matvec_mul_into("log4", x[0], q, s, 152064)
    x1 = np.load(tmp_path / "x1.npy")
    q1, s1, _ = weight("log4", 3584, 3584, seed=11)
    q2, s2, _ = weight("w8", 1001, 3584, seed=12)
    q3, s3, x3 = weight("w4zp8", 1, 256, seed=13)
    r1 = np.stack([oracle.matvec_mul_into("log4", xb, q1, s1, 3584) for xb in x1])
    for r in range(2):
        assert normwise_err(np.load(tmp_path / f"lm{r}.npy"), ref) <= GEMV_TOL
        y1 = np.load(tmp_path / f"y1_{r}.npy")
        assert normwise_err(y1, r1) <= GEMV_TOL
        # the second GEMV read the first's gathered output: compare with the oracle on that input
        r2 = np.stack([oracle.matvec_mul_into("w8", yb, q2, s2, 1001) for yb in y1])
        assert normwise_err(np.load(tmp_path / f"y2_{r}.npy"), r2) <= GEMV_TOL
        assert normwise_err(np.load(tmp_path / f"y3_{r}.npy"), oracle.matvec_mul_into("w4zp8", x3, q3, s3, 1)) <= GEMV_TOL
        rh = np.stack([oracle.matvec_mul_into("w8", xb, q2, s2, 1001) for xb in x1])
        assert normwise_err(np.load(tmp_path / f"yh_{r}.npy"), rh) <= GEMV_TOL
        assert np.load(tmp_path / f"yb_{r}.npy").tobytes() == np.load(tmp_path / f"yh_{r}.npy").tobytes()
    # both ranks hold identical full outputs
    assert np.load(tmp_path / "lm0.npy").tobytes() == np.load(tmp_path / "lm1.npy").tobytes()


@pytest.mark.gpu
def test_sharded_wait_runs_out_when_a_rank_stops(tmp_path):
    if not two_gpus():
        pytest.skip("needs two GPUs")
    mp.start_processes(gpu_worker, args=(2, free_port(), str(tmp_path), "stop"), nprocs=2, join=True,
                       start_method="spawn")
    assert str(np.load(tmp_path / "stop0.npy")[0]) == "timeout"
    assert str(np.load(tmp_path / "stop1.npy")[0]) == "ok"
