"""GPU decode step (BASELINE config 2 structure) against the oracle's restatement
of the reference's single-token decode (cpu_engine.rs:2819-3064), through the C
ABI (bramha_cuda_op_* and the tensor-core GEMVs).

Parity is teacher-forced per step (both sides consume the same tokens), on a
2-layer model with the Qwen2-0.5B layer shapes (hidden 896, 14 query / 2 KV
heads of 64, intermediate 4864) and a 4096-token vocabulary.

Tolerance: logits within normwise relative error 1e-3 (fp32 accumulate; the
GEMVs carry the activations as 8-bit terms, ~1e-5 each, and the reductions run
in a different order).  Greedy tokens must agree wherever the oracle's top two
logits are further apart than that tolerance allows.
"""
import numpy as np
import pytest

import oracle
from oracle.decode import Layer, Linear, Model, Qwen2Config
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


def oracle_model(fmt, layers=2, vocab=4096, seed=31):
    cfg = Qwen2Config(layers=layers, vocab=vocab)
    r = rng(seed)

    def lin(n, k):
        w = r.normal(0, 0.02, n * k).astype(np.float32)
        q, s = oracle.quantize(fmt, w, n, k)
        return Linear(fmt, n, k, q, s)

    qd, kvd, H, I = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim, cfg.hidden, cfg.intermediate
    L = [Layer(r.normal(1, 0.1, H).astype(np.float32), lin(qd, H), lin(kvd, H), lin(kvd, H),
               r.normal(0, 0.1, qd).astype(np.float32), r.normal(0, 0.1, kvd).astype(np.float32),
               r.normal(0, 0.1, kvd).astype(np.float32), lin(H, qd), r.normal(1, 0.1, H).astype(np.float32),
               lin(I, H), lin(I, H), lin(H, I)) for _ in range(layers)]
    m = Model(cfg, r.normal(0, 1, (vocab, H)).astype(np.float32), L, r.normal(1, 0.1, H).astype(np.float32),
              lin(vocab, H))
    m.reset()
    return m


def gpu_model(plane, m, tag, max_ctx=64, fuse_norm=True):
    from bramha_b200 import DecodeConfig, DecodeLayer, DecodeModel
    c = m.cfg
    dev = torch.device("cuda", 0)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    reg = lambda name, lin: plane.register(f"{tag}:{name}", lin.fmt, lin.n, lin.k, lin.q, lin.s)
    layers = [DecodeLayer(t(L.ln1), reg(f"{i}.q", L.q), reg(f"{i}.k", L.k), reg(f"{i}.v", L.v), t(L.bq), t(L.bk),
                          t(L.bv), reg(f"{i}.o", L.o), t(L.ln2), reg(f"{i}.g", L.gate), reg(f"{i}.u", L.up),
                          reg(f"{i}.d", L.down)) for i, L in enumerate(m.layers)]
    cfg = DecodeConfig(layers=c.layers, hidden=c.hidden, heads=c.heads, kv_heads=c.kv_heads, head_dim=c.head_dim,
                       intermediate=c.intermediate, vocab=c.vocab, eps=c.eps, rope_theta=c.rope_theta)
    return DecodeModel(plane, cfg, layers, t(m.embed), t(m.norm), reg("lm", m.lm_head), max_ctx=max_ctx,
                       fuse_norm=fuse_norm)


@pytest.mark.parametrize("fmt", ["log4", "w4zp8", "w8"])
def test_decode_step_teacher_forced_and_greedy_vs_oracle(plane, fmt):
    m = oracle_model(fmt)
    dm = gpu_model(plane, m, f"dec:{fmt}")
    prompt = [int(v) for v in rng(7).integers(0, m.cfg.vocab, 10)]
    # teacher-forced prompt, eagerly launched
    dm.reset()
    for pos, tok in enumerate(prompt[:-1]):
        dm.set_token(tok)
        dm.step(greedy=False)
        dm.sync()
        ref = m.forward(tok, pos)
        assert normwise_err(dm.logits.cpu().numpy(), ref) <= TOL, pos
    assert dm.position() == len(prompt) - 1
    # greedy continuation: the oracle follows the GPU's tokens
    dm.set_token(prompt[-1])
    tok, generated = prompt[-1], []
    for s in range(6):
        dm.step(greedy=True)
        dm.sync()
        ref = m.forward(tok, len(prompt) - 1 + s)
        want = oracle.penalty_argmax(ref.copy(), generated)
        got = dm.last_token()
        if got != want:  # only a near-tie may differ
            pen = ref.copy()
            oracle.penalty_argmax(pen, generated)
            assert abs(pen[got] - pen[want]) <= 2 * TOL * np.max(np.abs(ref)), (s, got, want)
        generated.append(got)
        tok = got
    assert dm.generated_tokens() == generated
    assert dm.position() == len(prompt) - 1 + 6
    for L in dm.layers:
        for w in (L.q, L.k, L.v, L.o, L.gate, L.up, L.down):
            plane.evict(w.key)
    plane.evict(dm.lm_head.key)


def test_decode_graph_replay_matches_eager(plane):
    m = oracle_model("log4", layers=1, vocab=2048, seed=5)
    dm = gpu_model(plane, m, "decg")
    toks = [3, 1999, 42, 7, 7]

    def run(use_graph):
        dm.reset()
        outs = []
        for tok in toks:
            dm.set_token(tok)
            dm.step(greedy=False)
            dm.sync()
            outs.append(dm.logits.clone())
        dm.set_token(toks[-1])
        for _ in range(4):
            dm.step(greedy=True)
        dm.sync()
        return [o.cpu().numpy() for o in outs], dm.generated_tokens()

    eager = run(False)
    dm.capture()
    graph = run(True)
    for a, b in zip(eager[0], graph[0]):
        assert np.array_equal(a, b)
    assert eager[1] == graph[1]
    dm.release()


def test_rope_attention_fused_equals_two_kernels(plane):
    """bramha_cuda_op_rope_attention == op_qkv_rope then op_attention, bit for bit
    (outputs and the appended cache row), at a position with cached rows."""
    from bramha_b200 import lib
    from bramha_b200._lib import check
    from bramha_b200.plane import _stream
    st = _stream(None)  # torch's current stream: plane.stream_sync() waits for it
    nq, nkv, hd, ctx_len, pos = 14, 2, 64, 64, 37
    r = rng(12)
    dev = torch.device("cuda", 0)
    mk = lambda *shape: torch.from_numpy(r.normal(0, 1, shape).astype(np.float32)).to(dev)
    q, k, v = mk(nq * hd), mk(nkv * hd), mk(nkv * hd)
    bq, bk, bv = mk(nq * hd), mk(nkv * hd), mk(nkv * hd)
    kc0, vc0 = mk(ctx_len, nkv * hd), mk(ctx_len, nkv * hd)
    p = torch.tensor([pos], dtype=torch.int32, device=dev)
    L, c = lib(), plane.ctx
    # two kernels
    q1, kc1, vc1, o1 = q.clone(), kc0.clone(), vc0.clone(), torch.empty(nq * hd, device=dev)
    kc2, vc2, o2 = kc0.clone(), vc0.clone(), torch.empty(nq * hd, device=dev)
    torch.cuda.synchronize()  # the ops below run on the context's own stream
    check(L.bramha_cuda_op_qkv_rope(c, q1.data_ptr(), k.data_ptr(), v.data_ptr(), bq.data_ptr(), bk.data_ptr(),
                                    bv.data_ptr(), nq, nkv, hd, 1e6, p.data_ptr(), ctx_len, kc1.data_ptr(),
                                    vc1.data_ptr(), st))
    check(L.bramha_cuda_op_attention(c, q1.data_ptr(), kc1.data_ptr(), vc1.data_ptr(), p.data_ptr(), nq, nkv, hd,
                                     ctx_len, o1.data_ptr(), st))
    # fused
    check(L.bramha_cuda_op_rope_attention(c, q.data_ptr(), k.data_ptr(), v.data_ptr(), bq.data_ptr(), bk.data_ptr(),
                                          bv.data_ptr(), nq, nkv, hd, 1e6, p.data_ptr(), ctx_len, kc2.data_ptr(),
                                          vc2.data_ptr(), o2.data_ptr(), st))
    plane.stream_sync()
    assert torch.equal(o1, o2)
    assert torch.equal(kc1, kc2) and torch.equal(vc1, vc2)
    # against the oracle's restatement
    qn = (q + bq).cpu().numpy().copy()
    kn = (k + bk).cpu().numpy().copy()
    oracle.rope_(qn, pos, nq, hd, 1e6)
    oracle.rope_(kn, pos, nkv, hd, 1e6)
    kcache = kc0.cpu().numpy()[:pos + 1].copy()
    vcache = vc0.cpu().numpy()[:pos + 1].copy()
    kcache[pos], vcache[pos] = kn, (v + bv).cpu().numpy()
    ref = oracle.attention(qn, kcache, vcache, pos + 1, nq, nkv, hd)
    assert normwise_err(o2.cpu().numpy(), ref) <= 1e-5


@pytest.mark.parametrize("nq,nkv,hd,max_ctx,pos", [
    (14, 2, 64, 640, 0),        # one row: 31 of the 32 splits empty
    (14, 2, 64, 640, 511),      # the config-2 shape
    (14, 2, 64, 640, 639),      # the cache's last row
    (28, 4, 128, 4096, 3000),   # 64 splits of 47 rows: two staged chunks each
    (8, 2, 96, 51200, 20000),   # the largest cache: 64 splits of 313 rows
    (4, 1, 6, 100, 57),         # head_dim % 4 != 0: scalar staging
    (6, 3, 33, 50, 49),         # odd head_dim (the unfused attention only)
])
def test_attention_splits_vs_oracle(plane, nq, nkv, hd, max_ctx, pos):
    """bramha_cuda_op_attention within 1e-5 (normwise) of the oracle's single
    pass over rows 0 .. pos (flash_attention_single_into,
    cpu_engine.rs:1450-1509) and bit-identical run to run, across split counts,
    empty splits, multi-chunk ranges and head sizes; for an even head_dim,
    bramha_cuda_op_rope_attention equals op_qkv_rope then op_attention bit for
    bit, the appended cache row included."""
    from bramha_b200 import lib
    from bramha_b200._lib import check
    from bramha_b200.plane import _stream
    st = _stream(None)  # torch's current stream: plane.stream_sync() waits for it
    r = rng(pos + hd)
    dev = torch.device("cuda", 0)
    mk = lambda *shape: torch.from_numpy(r.normal(0, 1, shape).astype(np.float32)).to(dev)
    L, c = lib(), plane.ctx
    q = mk(nq * hd)
    kc, vc = mk(max_ctx, nkv * hd), mk(max_ctx, nkv * hd)
    p = torch.tensor([pos], dtype=torch.int32, device=dev)
    torch.cuda.synchronize()  # the ops below run on the context's own stream
    outs = []
    for _ in range(2):
        o = torch.empty(nq * hd, device=dev)
        check(L.bramha_cuda_op_attention(c, q.data_ptr(), kc.data_ptr(), vc.data_ptr(), p.data_ptr(), nq, nkv, hd,
                                         max_ctx, o.data_ptr(), st))
        outs.append(o)
    plane.stream_sync()
    assert torch.equal(outs[0], outs[1])
    ref = oracle.attention(q.cpu().numpy(), kc[:pos + 1].cpu().numpy(), vc[:pos + 1].cpu().numpy(), pos + 1, nq, nkv,
                           hd)
    assert normwise_err(outs[0].cpu().numpy(), ref) <= 1e-5
    if hd % 2:
        return
    k, v = mk(nkv * hd), mk(nkv * hd)
    bq, bk, bv = mk(nq * hd), mk(nkv * hd), mk(nkv * hd)
    q1, kc1, vc1, o1 = q.clone(), kc.clone(), vc.clone(), torch.empty(nq * hd, device=dev)
    kc2, vc2, o2 = kc.clone(), vc.clone(), torch.empty(nq * hd, device=dev)
    torch.cuda.synchronize()
    check(L.bramha_cuda_op_qkv_rope(c, q1.data_ptr(), k.data_ptr(), v.data_ptr(), bq.data_ptr(), bk.data_ptr(),
                                    bv.data_ptr(), nq, nkv, hd, 1e6, p.data_ptr(), max_ctx, kc1.data_ptr(),
                                    vc1.data_ptr(), st))
    check(L.bramha_cuda_op_attention(c, q1.data_ptr(), kc1.data_ptr(), vc1.data_ptr(), p.data_ptr(), nq, nkv, hd,
                                     max_ctx, o1.data_ptr(), st))
    check(L.bramha_cuda_op_rope_attention(c, q.data_ptr(), k.data_ptr(), v.data_ptr(), bq.data_ptr(), bk.data_ptr(),
                                          bv.data_ptr(), nq, nkv, hd, 1e6, p.data_ptr(), max_ctx, kc2.data_ptr(),
                                          vc2.data_ptr(), o2.data_ptr(), st))
    plane.stream_sync()
    assert torch.equal(o1, o2)
    assert torch.equal(kc1, kc2) and torch.equal(vc1, vc2)


@pytest.mark.parametrize("fmt", ["log4", "w4zp8", "w8"])
def test_gemv_swiglu_equals_silu_then_gemv(plane, fmt):
    """bramha_cuda_gemv_swiglu_dev == bramha_cuda_op_silu_mul then the GEMV, bit
    for bit (the same rounding of silu(g) * up), at the 0.5B down shape and at a
    7B-sized one, batch 1 and 3."""
    from bramha_b200 import lib
    from bramha_b200._lib import check
    from tests._util import make_weight
    dev = torch.device("cuda", 0)
    for n, k in [(896, 4864), (3584, 18944)]:
        _, q, s = make_weight(fmt, n, k, seed=n)
        w = plane.register(f"swiglu:{fmt}:{n}", fmt, n, k, q, s)
        for batch in (1, 3):
            r = rng(batch)
            g = torch.from_numpy(r.normal(0, 2, (batch, k)).astype(np.float32)).to(dev)
            u = torch.from_numpy(r.normal(0, 1, (batch, k)).astype(np.float32)).to(dev)
            m = torch.empty_like(g)
            from bramha_b200.plane import _stream
            check(lib().bramha_cuda_op_silu_mul(plane.ctx, g.data_ptr(), u.data_ptr(), batch * k, m.data_ptr(),
                                                _stream(None)))
            y1 = torch.empty((batch, n), device=dev)
            y2 = torch.empty((batch, n), device=dev)
            plane.stream_sync()
            plane.gemv_dev(w, m, y1)
            plane.gemv_swiglu_dev(w, g, u, y2)
            plane.stream_sync()
            assert torch.equal(y1, y2), (n, batch)
        plane.evict(w.key)


@pytest.mark.parametrize("fmt,fuse", [("log4", True), ("w4zp8", True), ("w8", True), ("log4", "mlp")])
def test_decode_fused_norms_equal_separate_kernels(plane, fmt, fuse):
    """The step with residual adds + RMSNorms formed by the GEMV that reads them
    (bramha_cuda_gemv_rmsnorm_dev, double-buffered residual) equals the step with
    the RMSNorm kernel and the plain GEMV, bit for bit: logits and greedy tokens."""
    m = oracle_model(fmt, layers=3, vocab=2048, seed=13)
    fused = gpu_model(plane, m, f"fnf:{fmt}:{fuse}", fuse_norm=fuse)
    plain = gpu_model(plane, m, f"fnp:{fmt}:{fuse}", fuse_norm=False)
    # log4 / w4zp8: the norms inside the GEMVs; w8 gate|up (8.7 MB) keeps its norm kernel
    per_layer = (1 if fmt == "w8" else 2) if fuse is True else 1
    assert fused.kernel_launches_per_step() == plain.kernel_launches_per_step() - per_layer * m.cfg.layers
    toks = [5, 700, 1999, 12]
    outs = []
    for dm in (fused, plain):
        dm.reset()
        logits = []
        for tok in toks:
            dm.set_token(tok)
            dm.step(greedy=False)
            dm.sync()
            logits.append(dm.logits.clone())
        dm.set_token(toks[-1])
        for _ in range(3):
            dm.step(greedy=True)
        dm.sync()
        outs.append((logits, dm.generated_tokens(), dm.residual.clone()))
    for a, b in zip(outs[0][0], outs[1][0]):
        assert torch.equal(a, b)
    assert outs[0][1] == outs[1][1]
    assert torch.equal(outs[0][2], outs[1][2])  # the residual stream ends in the same buffer
    for dm in (fused, plain):
        for L in dm.layers:
            for w in (L.q, L.k, L.v, L.o, L.gate, L.up, L.down):
                plane.evict(w.key)
        plane.evict(dm.lm_head.key)


@pytest.mark.parametrize("fmt,n_list,k", [("log4", [896, 128, 128], 896), ("w8", [896, 128, 128], 896),
                                          ("log4", [4864, 4864], 896), ("w8", [4864, 4864], 896),
                                          ("w4zp8", [3584], 3584)],
                         ids=["log4_qkv_one_launch", "w8_qkv_one_launch", "log4_gate_up_one_launch",
                              "w8_gate_up_two_kernels", "w4zp8_7b_two_kernels"])
def test_gemv_rmsnorm_dev_equals_rmsnorm_then_gemv(plane, fmt, n_list, k):
    """bramha_cuda_gemv_rmsnorm_dev == bramha_cuda_op_rmsnorm (residual add in
    place) then bramha_cuda_gemv_multi_dev, bit for bit, with and without the
    residual and with and without x_out; the 7B-sized case takes the path that
    runs the RMSNorm kernel first."""
    from bramha_b200 import lib
    from bramha_b200._lib import check
    from bramha_b200.plane import _stream
    from tests._util import make_weight
    dev = torch.device("cuda", 0)
    ws = []
    for i, n in enumerate(n_list):
        _, q, s = make_weight(fmt, n, k, seed=100 + i)
        ws.append(plane.register(f"rmsg:{fmt}:{i}:{n}:{k}", fmt, n, k, q, s))
    r = rng(k)
    x = torch.from_numpy(r.normal(0, 3, k).astype(np.float32)).to(dev)
    delta = torch.from_numpy(r.normal(0, 1, k).astype(np.float32)).to(dev)
    nw = torch.from_numpy(r.normal(1, 0.1, k).astype(np.float32)).to(dev)
    for d in (delta, None):
        for want_out in (True, False):
            xr = x.clone()
            h = torch.empty(k, device=dev)
            check(lib().bramha_cuda_op_rmsnorm(plane.ctx, xr.data_ptr(), None if d is None else d.data_ptr(),
                                               nw.data_ptr(), k, 1e-6, h.data_ptr(), _stream(None)))
            y1 = [torch.empty(n, device=dev) for n in n_list]
            plane.gemv_multi_dev(ws, h, y1)
            y2 = [torch.full((n,), float("nan"), device=dev) for n in n_list]
            xo = torch.full((k,), float("nan"), device=dev) if want_out else None
            plane.gemv_rmsnorm_dev(ws, x, d, nw, 1e-6, xo, y2)
            plane.stream_sync()
            for a, b in zip(y1, y2):
                assert torch.equal(a, b), (d is None, want_out)
            if want_out:
                assert torch.equal(xo, xr)
    # the inputs are untouched; x_out may not alias them
    from bramha_b200 import BramhaError
    with pytest.raises(BramhaError):
        plane.gemv_rmsnorm_dev(ws, x, delta, nw, 1e-6, x, [torch.empty(n, device=dev) for n in n_list])
    for w in ws:
        plane.evict(w.key)
