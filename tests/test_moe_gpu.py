"""MoE expert MLP on the GPU (moe.cu + grouped tcgen05 GEMMs, through the C ABI)
against the oracle's restatement of run_mlp_into's MoE branch
(cpu_engine.rs:1799-1989).

Tolerance: normwise relative error 1e-3 (the expert GEMMs run on the tensor
cores with the activations split into bf16 hi + lo, fp32 accumulation).  The
selected experts must equal the oracle's except where two probabilities are
within 1e-6 of each other (the GPU's expf and the host's may differ in the
last bit).
"""
import numpy as np
import pytest

import oracle
from tests._util import normwise_err, rng

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 1e-3


@pytest.fixture(scope="module")
def plane():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from bramha_b200 import CudaComputePlane
    p = CudaComputePlane(0)
    yield p
    p.close()


def experts(fmt, E, H, I, seed):
    r = rng(seed)
    mk = lambda n, k: oracle.quantize(fmt, r.normal(0, 0.02, n * k).astype(np.float32), n, k)
    gates = [mk(I, H) for _ in range(E)]
    ups = [mk(I, H) for _ in range(E)]
    downs = [mk(H, I) for _ in range(E)]
    cat = lambda ws: (np.concatenate([q.view(np.uint8) for q, _ in ws]), np.concatenate([s for _, s in ws]))
    return gates, ups, downs, cat


def register(plane, tag, fmt, E, H, I, gates, ups, downs):
    from bramha_b200 import stack_gate_up
    gq, gs = stack_gate_up(gates, ups)
    dq = np.concatenate([q.view(np.uint8) for q, _ in downs])
    ds = np.concatenate([s for _, s in downs])
    gu = plane.register(f"{tag}:gate_up", fmt, E * 2 * I, H, gq, gs)
    dn = plane.register(f"{tag}:down", fmt, E * H, I, dq, ds)
    return gu, dn


def check_selection(ids, ref_ids, lg):
    p = np.exp(lg - lg.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    for t in range(ids.shape[0]):
        if not np.array_equal(ids[t], ref_ids[t]):
            diff = np.flatnonzero(ids[t] != ref_ids[t])
            for j in diff:  # only a near-tie may reorder
                assert abs(p[t, ids[t][j]] - p[t, ref_ids[t][j]]) <= 1e-6, (t, ids[t], ref_ids[t])


@pytest.mark.parametrize("fmt", ["log4", "w4zp8", "w8"])
def test_moe_small_vs_oracle(plane, fmt):
    E, H, I, T, k = 8, 256, 128, 20, 3
    gates, ups, downs, cat = experts(fmt, E, H, I, seed=3)
    gu, dn = register(plane, f"moe:{fmt}", fmt, E, H, I, gates, ups, downs)
    r = rng(4)
    x = r.normal(0, 1, (T, H)).astype(np.float32)
    lg = r.normal(0, 1, (T, E)).astype(np.float32)
    out, ids = plane.moe_mlp(gu, dn, E, k, x, lg)
    ref, ref_ids, _ = oracle.moe_mlp(fmt, x, lg, k, cat(gates), cat(ups), cat(downs))
    check_selection(ids, ref_ids, lg)
    assert normwise_err(out, ref) <= TOL
    out2, _ = plane.moe_mlp(gu, dn, E, k, x, lg)
    assert np.array_equal(out, out2)  # deterministic
    plane.evict(gu.key)
    plane.evict(dn.key)


def test_moe_config5_shapes(plane):
    """64 experts, top-8, hidden 3584, expert intermediate 2560, log4; 64 tokens."""
    E, H, I, T, k = 64, 3584, 2560, 64, 8
    gates, ups, downs, cat = experts("log4", E, H, I, seed=5)
    gu, dn = register(plane, "moe5", "log4", E, H, I, gates, ups, downs)
    r = rng(6)
    x = r.normal(0, 1, (T, H)).astype(np.float32)
    lg = r.normal(0, 1, (T, E)).astype(np.float32)
    out, ids = plane.moe_mlp(gu, dn, E, k, x, lg)
    ref, ref_ids, _ = oracle.moe_mlp("log4", x, lg, k, cat(gates), cat(ups), cat(downs),
                                     threads=oracle.max_threads())
    check_selection(ids, ref_ids, lg)
    assert normwise_err(out, ref) <= TOL
    plane.evict(gu.key)
    plane.evict(dn.key)


def test_moe_crowded_expert_and_skipped_weights(plane):
    """150 tokens all routed first to expert 2 (three 64-token tiles), tokens
    whose other probabilities underflow to 0 (skipped, cpu_engine.rs:1832-1834),
    and top_k above the expert count."""
    E, H, I, T = 4, 128, 64, 150
    gates, ups, downs, cat = experts("w4zp8", E, H, I, seed=7)
    gu, dn = register(plane, "moe:crowd", "w4zp8", E, H, I, gates, ups, downs)
    r = rng(8)
    x = r.normal(0, 1, (T, H)).astype(np.float32)
    lg = r.normal(0, 1, (T, E)).astype(np.float32)
    lg[:, 2] += 6.0
    lg[::5] = np.array([0.0, -200.0, 50.0, -200.0], np.float32)  # one expert keeps all the weight
    for k in (2, 7):
        out, ids = plane.moe_mlp(gu, dn, E, k, x, lg)
        ref, ref_ids, _ = oracle.moe_mlp("w4zp8", x, lg, k, cat(gates), cat(ups), cat(downs))
        check_selection(ids, ref_ids, lg)
        assert ids.shape == (T, min(k, E))
        assert normwise_err(out, ref) <= TOL
    plane.evict(gu.key)
    plane.evict(dn.key)


def test_moe_device_call_and_errors(plane):
    from bramha_b200 import BramhaError
    E, H, I, T, k = 8, 256, 128, 12, 2
    gates, ups, downs, cat = experts("log4", E, H, I, seed=9)
    gu, dn = register(plane, "moe:dev", "log4", E, H, I, gates, ups, downs)
    r = rng(10)
    x = r.normal(0, 1, (T, H)).astype(np.float32)
    lg = r.normal(0, 1, (T, E)).astype(np.float32)
    host, ids = plane.moe_mlp(gu, dn, E, k, x, lg)
    dev = torch.device("cuda", 0)
    xd, ld = torch.from_numpy(x).to(dev), torch.from_numpy(lg).to(dev)
    od = torch.empty((T, H), device=dev)
    sd = torch.empty((T, k), dtype=torch.int32, device=dev)
    plane.moe_mlp_dev(gu, dn, E, k, xd, ld, od, sd)
    plane.stream_sync()
    assert np.array_equal(od.cpu().numpy(), host) and np.array_equal(sd.cpu().numpy(), ids)
    with pytest.raises(BramhaError, match="equal blocks"):
        plane.moe_mlp(gu, dn, 7, k, x, lg[:, :7])
    with pytest.raises(BramhaError, match="exceeds"):
        plane.moe_mlp(gu, dn, E, k, np.zeros((9000, H), np.float32), np.zeros((9000, E), np.float32))
    plane.evict(gu.key)
    plane.evict(dn.key)


def test_moe_route_and_experts_entry_points(plane):
    """The two halves used for expert parallelism on one GPU: the routing alone
    gives the layer's expert choice and the oracle's probabilities, and the
    experts run on the routed rows, combined in the sorted order, reproduce the
    whole layer bit for bit."""
    E, H, I, T, k = 8, 256, 128, 24, 3
    gates, ups, downs, cat = experts("log4", E, H, I, seed=11)
    gu, dn = register(plane, "moe:halves", "log4", E, H, I, gates, ups, downs)
    r = rng(12)
    x = r.normal(0, 1, (T, H)).astype(np.float32)
    lg = r.normal(0, 1, (T, E)).astype(np.float32)
    lg[5] = np.array([0, -200, 50, -200, -200, -200, -200, -200], np.float32)  # weights that underflow
    dev = torch.device("cuda", 0)
    xd, ld = torch.from_numpy(x).to(dev), torch.from_numpy(lg).to(dev)
    full = torch.empty((T, H), device=dev)
    sel = torch.empty((T, k), dtype=torch.int32, device=dev)
    plane.moe_mlp_dev(gu, dn, E, k, xd, ld, full, sel)
    ids = torch.empty((T, k), dtype=torch.int32, device=dev)
    w = torch.empty((T, k), device=dev)
    plane.moe_route_dev(ld, k, ids, w)
    plane.stream_sync()
    assert torch.equal(ids, sel)
    _, ref_ids, ref_w = oracle.moe_mlp("log4", x, lg, k, cat(gates), cat(ups), cat(downs))
    check_selection(ids.cpu().numpy(), ref_ids, lg)
    assert np.allclose(w.cpu().numpy(), ref_w, rtol=1e-6, atol=1e-12)
    rows = xd.repeat_interleave(k, dim=0).contiguous()
    y = torch.empty_like(rows)
    plane.moe_experts_dev(gu, dn, E, rows, ids.reshape(-1).contiguous(), y)
    plane.stream_sync()
    y = y.view(T, k, H)
    out = torch.zeros((T, H), device=dev)
    for j in range(k):
        out = torch.where((w[:, j:j + 1] > 0), out + y[:, j] * w[:, j:j + 1], out)
    assert torch.equal(out, full)
    plane.evict(gu.key)
    plane.evict(dn.key)
