"""GEMV chains (bramha_cuda_gemv_chain_dev / bramha_cuda_gemv_chain): the
decode loop's back-to-back `matvec_mul_into` calls (src/inference/
cpu_engine.rs:2873-2976) as one call whose launches request the next launch's
weights into L2 while they run.  Prefetching changes no result: a chain must
equal its ops run one by one bit for bit, and the oracle within 1e-3.
"""
import numpy as np
import pytest

from tests._util import GEMV_TOL, make_weight, make_x, normwise_err, oracle_gemv

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


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


def layer_ops(plane, fmt, batch, seed, H=896, I=4864, QD=896, KV=128):
    """One decoder layer's GEMVs (q|k|v, o, gate|up, SwiGLU down) with
    independent inputs, plus what the oracle needs."""
    shapes = [[("q", QD, H), ("k", KV, H), ("v", KV, H)], [("o", H, QD)], [("gate", I, H), ("up", I, H)],
              [("down", H, I)]]
    ops, refs = [], []
    for gi, group in enumerate(shapes):
        ws, ys, wref = [], [], []
        k = group[0][2]
        for name, n, kk in group:
            _, q, s = make_weight(fmt, n, kk, seed=seed + n + kk + gi)
            ws.append(plane.register(f"chain:{fmt}:{seed}:{name}", fmt, n, kk, q, s))
            ys.append(torch.full((batch, n), float("nan"), device="cuda"))
            wref.append((q, s, n))
        x = make_x(batch, k, seed=seed + 7 * gi)
        up = make_x(batch, k, seed=seed + 7 * gi + 3) if group[0][0] == "down" else None
        ops.append((ws, dev(x), ys) + ((dev(up),) if up is not None else ()))
        refs.append((x, up, wref))
    return ops, refs


def silu_mul_np(g, u):
    return (g * (1.0 / (1.0 + np.exp(-g.astype(np.float64)))) * u).astype(np.float32)


@pytest.mark.parametrize("fmt", ["log4", "w4zp8", "w8"])
@pytest.mark.parametrize("batch", [1, 3])
def test_chain_equals_ops_one_by_one(plane, fmt, batch):
    ops, refs = layer_ops(plane, fmt, batch, seed=10 + batch)
    ops2 = ops + layer_ops(plane, fmt, batch, seed=50 + batch)[0]  # two layers: 8 launches
    plane.gemv_chain_dev(ops2, batch)
    plane.stream_sync()
    got = [[y.clone() for y in op[2]] for op in ops2]
    for op in ops2:  # the same ops, one call each
        for y in op[2]:
            y.fill_(float("nan"))
        if len(op) > 3:
            plane.gemv_swiglu_dev(op[0][0], op[1], op[3], op[2][0])
        else:
            plane.gemv_multi_dev(op[0], op[1], op[2])
    plane.stream_sync()
    for g, op in zip(got, ops2):
        for a, b in zip(g, op[2]):
            assert torch.equal(a, b)
    # the first layer against the oracle
    for (x, up, wref), g in zip(refs, got):
        xin = silu_mul_np(x, up) if up is not None else x
        for (q, s, n), y in zip(wref, g):
            assert normwise_err(y.cpu().numpy(), oracle_gemv(fmt, xin, q, s, n)) <= GEMV_TOL
    for op in ops2:
        for w in op[0]:
            plane.evict(w.key)


@pytest.mark.parametrize("prefetch", [(0, 0), (128 << 10, 24 << 20), (512 << 10, 96 << 20)],
                         ids=["off", "default", "deep"])
def test_prefetch_settings_change_no_result(plane, prefetch):
    ops, _ = layer_ops(plane, "log4", 1, seed=90)
    plane.set_prefetch(0, 0)
    plane.gemv_chain_dev(ops)
    plane.stream_sync()
    base = [[y.clone() for y in op[2]] for op in ops]
    plane.set_prefetch(*prefetch)
    plane.gemv_chain_dev(ops)
    plane.stream_sync()
    plane.set_prefetch()
    for b, op in zip(base, ops):
        for a, y in zip(b, op[2]):
            assert torch.equal(a, y)
    for op in ops:
        for w in op[0]:
            plane.evict(w.key)


def test_host_chain_matches_oracle_unaligned_k(plane):
    """Host buffers of any alignment (K = 1001 odd), batch 2, w8 and log4 ops."""
    specs = [("w8", 300, 1001), ("log4", 520, 1002), ("w8", 64, 130)]
    ops, refs = [], []
    for i, (fmt, n, k) in enumerate(specs):
        _, q, s = make_weight(fmt, n, k, seed=i + 1)
        w = plane.register(f"hchain:{i}", fmt, n, k, q, s)
        x = make_x(2, k, seed=i + 20)
        y = np.full((2, n), np.nan, np.float32)
        ops.append(([w], x, [y]))
        refs.append((fmt, x, q, s, n))
    plane.gemv_chain(ops, batch=2)
    for (ws, x, ys), (fmt, _, q, s, n) in zip(ops, refs):
        assert normwise_err(ys[0], oracle_gemv(fmt, x, q, s, n)) <= GEMV_TOL
        plane.evict(ws[0].key)


def test_host_chain_swiglu_and_fused(plane):
    ops_d, refs = layer_ops(plane, "log4", 1, seed=123)
    ops = []
    for (ws, xd, ys, *up), (x, u, _) in zip(ops_d, refs):
        yh = [np.full(tuple(y.shape), np.nan, np.float32) for y in ys]
        ops.append((ws, x, yh) + ((u,) if u is not None else ()))
    plane.gemv_chain(ops)
    for (ws, x, ys, *up), (_, u, wref) in zip(ops, refs):
        xin = silu_mul_np(x, u) if u is not None else x
        for (q, s, n), y in zip(wref, ys):
            assert normwise_err(y, oracle_gemv("log4", xin, q, s, n)) <= GEMV_TOL
    for op in ops:
        for w in op[0]:
            plane.evict(w.key)


def test_chain_errors(plane):
    from bramha_b200 import BramhaError
    _, q, s = make_weight("log4", 64, 128, seed=1)
    w = plane.register("chainerr:a", "log4", 64, 128, q, s)
    _, q2, s2 = make_weight("w8", 64, 256, seed=2)
    w2 = plane.register("chainerr:b", "w8", 64, 256, q2, s2)
    x = torch.zeros((1, 128), device="cuda")
    y = torch.zeros((1, 64), device="cuda")
    with pytest.raises(BramhaError, match="share format and K"):
        plane.gemv_chain_dev([([w, w2], x, [y, y])])
    xm = torch.zeros(129, device="cuda")[1:]  # 4 bytes past a 16-byte boundary
    with pytest.raises(BramhaError, match="16-byte aligned"):
        plane.gemv_chain_dev([([w], xm, [y])])
    plane.gemv_chain_dev([])  # empty chain: nothing to do
    plane.evict(w.key)
    plane.evict(w2.key)


@pytest.mark.parametrize("pinned", [False, True])
def test_host_chain_many_blocks_equals_device_chain(plane, pinned):
    """A host-buffer chain of 8 layers (32 launches in nine copy blocks of 1, 2,
    4, 8, 2, 8, 4, 2 and 1 ops, each block's inputs copied in while earlier
    blocks run and its outputs copied back while later ones run) equals the
    same chain on device tensors bit for bit, on pageable numpy or pinned torch
    buffers: through bramha_cuda_gemv_chain, and through a chain bound once
    (bramha_cuda_host_chain_*, replayed from a CUDA graph when the buffers are
    pinned) run twice, the second time on new contents of the same buffers."""
    from bramha_b200 import BramhaError
    layers = [layer_ops(plane, "log4", 2, seed=400 + 31 * i) for i in range(8)]
    ops_d = [op for ops, _ in layers for op in ops]

    def host(a):
        a = a.cpu()
        if pinned:
            return a.pin_memory()
        return a.numpy().copy()

    def host_ops():
        return [(ws, host(x), [host(torch.full_like(y, float("nan"))) for y in ys]) + tuple(host(u) for u in up)
                for ws, x, ys, *up in ops_d]

    def same(ops_h):
        for (_, _, ysd, *_), (_, _, ysh, *_) in zip(ops_d, ops_h):
            for yd, yh in zip(ysd, ysh):
                assert torch.equal(yd.cpu(), yh if pinned else torch.from_numpy(yh))

    plane.gemv_chain_dev(ops_d, 2)
    plane.stream_sync()  # the chains share the context's K-split workspace: one at a time
    once = host_ops()
    plane.gemv_chain(once, batch=2)
    same(once)
    ops_h = host_ops()
    chain = plane.prepare_chain(ops_h, batch=2)
    assert chain.uses_graph() == pinned
    for rep in range(2):
        if rep:  # new inputs in the same host buffers, and on the device side
            for (ws, xh, *_), (_, xd, *__) in zip(ops_h, ops_d):
                fresh = torch.from_numpy(make_x(2, xd.shape[1], seed=900 + xd.shape[1]))
                xd.copy_(fresh.cuda())
                xh[...] = fresh if pinned else fresh.numpy()
            plane.gemv_chain_dev(ops_d, 2)
            plane.stream_sync()
        chain.run()
        same(ops_h)
    # and against the oracle for one op (layer 0's gate|up)
    (ws, x, ys, *up), (xr, ur, wref) = ops_h[2], layers[0][1][2]
    xn = x.numpy() if pinned else x
    for (q, s, n), y in zip(wref, ys):
        assert normwise_err(y.numpy() if pinned else y, oracle_gemv("log4", np.asarray(xn), q, s, n)) <= GEMV_TOL
    # a bound chain whose weight was evicted refuses to run
    gone = ops_d[-1][0][0].key
    plane.evict(gone)
    with pytest.raises(BramhaError):
        chain.run()
    chain.close()
    for ops, _ in layers:
        for op in ops:
            for w in op[0]:
                if w.key != gone:
                    plane.evict(w.key)
