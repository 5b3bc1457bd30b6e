"""GEMV programs (bramha_cuda_gemv_program_*): a chain of dependent GEMVs run
as ONE persistent launch, against the op-by-op chain and the oracle's
`matvec_mul_into` (src/inference/cpu_engine.rs:1307-1444).

Checked: a decoder layer's GEMVs (q|k|v fused, o, gate|up fused, the SwiGLU
down projection) at the Qwen2-0.5B and -7B shapes, batch 1, 3 and 8, every
format; an op that reads the previous op's output (the dependency the
program's per-op counters enforce); repeated runs and a CUDA-graph replay
(the counters return to zero); and a bounded wait that runs out (a test-only
withheld weight copy) reporting BRAMHA_ERR_TIMEOUT, after which the program
runs correctly again.  Tolerance: 1e-3 normwise against the oracle; 1e-5
against the op-by-op launches (same arithmetic, fp32 summation grouped
differently).
"""
import numpy as np
import pytest

from tests._util import GEMV_TOL, make_weight, make_x, normwise_err, oracle_gemv

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

Q05 = dict(H=896, I=4864, QD=896, KV=128)
Q7 = dict(H=3584, I=18944, QD=3584, KV=512)


@pytest.fixture(scope="module")
def plane():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from bramha_b200 import CudaComputePlane
    p = CudaComputePlane(0)
    yield p
    p.close()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def silu_mul_np(g, u):
    return (g * (1.0 / (1.0 + np.exp(-g.astype(np.float64)))) * u).astype(np.float32)


def layer(plane, fmt, batch, seed, shapes, device_weights=False):
    H, I, QD, KV = shapes["H"], shapes["I"], shapes["QD"], shapes["KV"]
    groups = [[("q", QD, H), ("k", KV, H), ("v", KV, H)], [("o", H, QD)], [("gate", I, H), ("up", I, H)],
              [("down", H, I)]]
    ops, refs = [], []
    for gi, group in enumerate(groups):
        ws, ys, wref = [], [], []
        k = group[0][2]
        for name, n, kk in group:
            _, q, s = make_weight(fmt, n, kk, seed=seed + n + kk + gi)
            ws.append(plane.register(f"prog:{fmt}:{seed}:{name}:{n}", fmt, n, kk, q, s))
            ys.append(torch.full((batch, n), float("nan"), device="cuda"))
            wref.append((q, s, n))
        x = make_x(batch, k, seed=seed + 7 * gi)
        up = make_x(batch, k, seed=seed + 7 * gi + 3) if group[0][0] == "down" else None
        ops.append((ws, dev(x), ys) + ((dev(up),) if up is not None else ()))
        refs.append((x, up, wref))
    return ops, refs


def evict(plane, ops):
    for op in ops:
        for w in op[0]:
            plane.evict(w.key)


def snapshot(ops):
    return [[y.clone() for y in op[2]] for op in ops]


@pytest.mark.parametrize("fmt", ["log4", "w4zp8", "w8"])
@pytest.mark.parametrize("batch", [1, 3, 8])
def test_program_matches_chain_and_oracle_qwen05(plane, fmt, batch):
    ops = layer(plane, fmt, batch, 10 + batch, Q05)[0]
    ops2, refs2 = layer(plane, fmt, batch, 60 + batch, Q05)
    allops = ops + ops2
    plane.gemv_chain_dev(allops, batch)
    plane.stream_sync()
    ref_chain = snapshot(allops)
    prog = plane.gemv_program(allops, batch)
    for _ in range(2):  # runs back to back: the per-op counters return to zero
        for op in allops:
            for y in op[2]:
                y.fill_(float("nan"))
        prog.run()
        plane.stream_sync()
        for r, op in zip(ref_chain, allops):
            for a, y in zip(r, op[2]):
                assert normwise_err(y.cpu().numpy(), a.cpu().numpy()) <= 1e-5
    for (x, up, wref), op in zip(refs2, ops2):
        xin = silu_mul_np(x, up) if up is not None else x
        for (q, s, n), y in zip(wref, op[2]):
            assert normwise_err(y.cpu().numpy(), oracle_gemv(fmt, xin, q, s, n)) <= GEMV_TOL
    prog.close()
    evict(plane, allops)


@pytest.mark.parametrize("fmt", ["log4", "w8"])
def test_program_qwen7_layer(plane, fmt):
    """7B shapes: gate|up is 296 tiles (2 per CTA), down is K-split."""
    ops, refs = layer(plane, fmt, 1, 5, Q7)
    prog = plane.gemv_program(ops, 1)
    prog.run()
    plane.stream_sync()
    for (x, up, wref), op in zip(refs, ops):
        xin = silu_mul_np(x, up) if up is not None else x
        for (q, s, n), y in zip(wref, op[2]):
            assert normwise_err(y.cpu().numpy(), oracle_gemv(fmt, xin, q, s, n)) <= GEMV_TOL
    prog.close()
    evict(plane, ops)


@pytest.mark.parametrize("fmt", ["log4", "w4zp8"])
def test_program_op_reads_previous_output(plane, fmt):
    """op 1 reads op 0's output, op 2 reads op 1's: the program must wait for
    every CTA's rows before an op reads its input."""
    n, k = 3584, 3584
    ws, qs = [], []
    for i in range(3):
        _, q, s = make_weight(fmt, n, k, seed=100 + i)
        ws.append(plane.register(f"dep:{fmt}:{i}", fmt, n, k, q, s))
        qs.append((q, s))
    x = dev(make_x(1, k, seed=7))
    y = [torch.full((1, n), float("nan"), device="cuda") for _ in range(3)]
    ops = [([ws[0]], x, [y[0]]), ([ws[1]], y[0], [y[1]]), ([ws[2]], y[1], [y[2]])]
    prog = plane.gemv_program(ops, 1)
    prog.run()
    plane.stream_sync()
    h = x.cpu().numpy()
    for i in range(3):
        ref = oracle_gemv(fmt, h, qs[i][0], qs[i][1], n)
        got = y[i].cpu().numpy()
        assert normwise_err(got, ref) <= GEMV_TOL, i
        h = got  # the next op's input is what this op produced
    prog.close()
    for w in ws:
        plane.evict(w.key)


def test_program_in_cuda_graph(plane):
    ops, refs = layer(plane, "log4", 1, 31, Q05)
    prog = plane.gemv_program(ops, 1)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        prog.run(s)
    torch.cuda.synchronize()
    base = snapshot(ops)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        prog.run(s)
    for _ in range(3):
        for op in ops:
            for y in op[2]:
                y.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        for b, op in zip(base, ops):
            for a, y in zip(b, op[2]):
                assert torch.equal(a, y)
    del g
    plane.stream_sync(s)
    prog.close()
    evict(plane, ops)


def test_program_wait_runs_out_and_recovers(plane):
    from bramha_b200 import BramhaError
    ops, refs = layer(plane, "log4", 1, 41, Q7)
    prog = plane.gemv_program(ops, 1)
    prog.run()
    plane.stream_sync()
    base = snapshot(ops)
    plane.set_wait_timeout(5_000_000)
    plane.test_fault("gemv")
    try:
        prog.run()
        with pytest.raises(BramhaError) as ei:
            plane.stream_sync()
        assert ei.value.code == -7
    finally:
        plane.test_fault("none")
        plane.set_wait_timeout(0)
    prog.run()
    plane.stream_sync()
    for b, op in zip(base, ops):
        for a, y in zip(b, op[2]):
            assert torch.equal(a, y)
    prog.close()
    evict(plane, ops)


def test_program_rejects_mixed_formats_and_shards(plane):
    from bramha_b200 import BramhaError
    _, q, s = make_weight("log4", 128, 256, seed=1)
    _, q2, s2 = make_weight("w8", 128, 256, seed=2)
    w1 = plane.register("pm:a", "log4", 128, 256, q, s)
    w2 = plane.register("pm:b", "w8", 128, 256, q2, s2)
    x = torch.zeros((1, 256), device="cuda")
    y = torch.zeros((1, 128), device="cuda")
    with pytest.raises(BramhaError, match="same one of"):
        plane.gemv_program([([w1], x, [y]), ([w2], x, [y])], 1)
    with pytest.raises(BramhaError, match="batch"):
        plane.gemv_program([([w1], x, [y])], 9)
    plane.evict(w1.key)
    plane.evict(w2.key)
