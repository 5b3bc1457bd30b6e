"""CPU checks of the oracle's decode-step restatement (cpu_engine.rs:1292-1302,
1450-1530, 1682-1698, 2023-2026, 2985-3031) against independent numpy
formulations, and of its model step on a tiny random model."""
import numpy as np
import pytest

import oracle
from oracle.decode import Layer, Linear, Model, Qwen2Config
from tests._util import rng


def test_rms_norm_matches_formula():
    x = rng(1).normal(0, 3, 896).astype(np.float32)
    w = rng(2).normal(1, 0.1, 896).astype(np.float32)
    y = oracle.rms_norm(x, w, 1e-6)
    ref = x / np.sqrt(np.mean(x.astype(np.float64) ** 2) + 1e-6) * w
    assert np.max(np.abs(y - ref)) <= 1e-5 * np.max(np.abs(ref))


def test_rope_is_a_rotation_and_identity_at_zero():
    v = rng(3).normal(0, 1, 14 * 64).astype(np.float32)
    r0 = oracle.rope_(v.copy(), 0, 14, 64, 1e6)
    assert np.array_equal(r0, v)
    r = oracle.rope_(v.copy(), 37, 14, 64, 1e6)
    # each (i, i + 32) pair keeps its length
    a, b = v.reshape(14, 2, 32), r.reshape(14, 2, 32)
    assert np.allclose(np.hypot(a[:, 0], a[:, 1]), np.hypot(b[:, 0], b[:, 1]), rtol=1e-5)
    # the first pair rotates by pos * theta_0 = 37 rad
    c, s = np.cos(37.0), np.sin(37.0)
    assert np.allclose(b[:, 0, 0], a[:, 0, 0] * c - a[:, 1, 0] * s, atol=1e-5)


def test_attention_matches_softmax():
    nq, nkv, hd, t = 14, 2, 64, 33
    q = rng(4).normal(0, 1, nq * hd).astype(np.float32)
    kc = rng(5).normal(0, 1, (t, nkv * hd)).astype(np.float32)
    vc = rng(6).normal(0, 1, (t, nkv * hd)).astype(np.float32)
    out = oracle.attention(q, kc, vc, t, nq, nkv, hd)
    ref = []
    for h in range(nq):
        kh = h // (nq // nkv)
        s = kc[:, kh * hd:(kh + 1) * hd] @ q[h * hd:(h + 1) * hd] / np.sqrt(hd)
        p = np.exp(s - s.max())
        ref.append((p / p.sum()) @ vc[:, kh * hd:(kh + 1) * hd])
    assert np.max(np.abs(out - np.concatenate(ref))) <= 1e-5


def test_silu_mul_and_penalty_argmax():
    g = np.array([-3, -0.5, 0, 0.5, 3], np.float32)
    u = np.array([1, 2, 3, 4, 5], np.float32)
    assert np.allclose(oracle.silu_mul(g, u), g / (1 + np.exp(-g)) * u, rtol=1e-6)
    lg = np.array([2.0, -1.0, 2.0, 1.9], np.float32)
    # id 0 twice (2 / 1.15^2), id 1 once (more negative): the first maximum is id 2
    assert oracle.penalty_argmax(lg, [0, 1, 0]) == 2
    assert np.isclose(lg[0], 2.0 / 1.15 / 1.15) and np.isclose(lg[1], -1.15)
    lg2 = np.array([1.0, 1.0, 0.5], np.float32)
    assert oracle.penalty_argmax(lg2, []) == 0  # ties: first index


def tiny_model(fmt="log4", layers=2, vocab=300, seed=11):
    cfg = Qwen2Config(layers=layers, hidden=128, heads=4, kv_heads=2, head_dim=32, intermediate=256, vocab=vocab)
    r = rng(seed)

    def lin(n, k):
        w = r.normal(0, 0.05, n * k).astype(np.float32)
        q, s = oracle.quantize(fmt, w, n, k)
        return Linear(fmt, n, k, q, s)

    qd, kvd = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    L = [Layer(r.normal(1, 0.1, cfg.hidden).astype(np.float32), lin(qd, cfg.hidden), lin(kvd, cfg.hidden),
               lin(kvd, cfg.hidden), r.normal(0, 0.1, qd).astype(np.float32),
               r.normal(0, 0.1, kvd).astype(np.float32), r.normal(0, 0.1, kvd).astype(np.float32),
               lin(cfg.hidden, qd), r.normal(1, 0.1, cfg.hidden).astype(np.float32),
               lin(cfg.intermediate, cfg.hidden), lin(cfg.intermediate, cfg.hidden),
               lin(cfg.hidden, cfg.intermediate)) for _ in range(layers)]
    m = Model(cfg, r.normal(0, 1, (vocab, cfg.hidden)).astype(np.float32), L,
              r.normal(1, 0.1, cfg.hidden).astype(np.float32), lin(vocab, cfg.hidden))
    m.reset()
    return m


def test_oracle_model_step_is_causal_and_deterministic():
    m = tiny_model()
    toks = [5, 17, 299, 3]
    a = [m.forward(t, p) for p, t in enumerate(toks)]
    m.reset()
    b = [m.forward(t, p) for p, t in enumerate(toks)]
    assert all(np.array_equal(x, y) for x, y in zip(a, b))
    assert all(np.isfinite(x).all() and x.shape == (300,) for x in a)
    # the first token's logits do not depend on what follows
    m.reset()
    c0 = m.forward(toks[0], 0)
    assert np.array_equal(c0, a[0])
    # token ids wrap modulo the vocabulary (cpu_engine.rs:2821)
    m.reset()
    assert np.array_equal(m.forward(toks[0] + 300, 0), a[0])
