"""The oracle's restatement of the MoE branch of run_mlp_into
(cpu_engine.rs:1799-1989) checked against an independent numpy formulation:
softmax of the router logits, a stable descending order (ties to the lower
expert index), the first top_k without renormalisation, experts with a
weight <= 0 skipped, SwiGLU experts through the oracle's matvec_mul_into and
out = sum of weight * expert output in the sorted order."""
import numpy as np
import pytest

import oracle
from tests._util import rng


def stacked(fmt, e, n, k, r):
    qs = [oracle.quantize(fmt, r.normal(0, 0.02, n * k).astype(np.float32), n, k) for _ in range(e)]
    return np.concatenate([q.view(np.uint8) for q, _ in qs]), np.concatenate([s for _, s in qs])


def numpy_moe(fmt, h, lg, k, g, u, d, I):
    T, H = h.shape
    p = np.exp(lg - lg.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    order = np.argsort(-p, 1, kind="stable")[:, :k]
    gb, db = g[0].size // (g[1].size // I), d[0].size // (d[1].size // H)
    out = np.zeros((T, H))
    for t in range(T):
        for e in order[t]:
            if p[t, e] <= 0:
                continue
            G = oracle.matvec_mul_into(fmt, h[t], g[0][e * gb:(e + 1) * gb], g[1][e * I:(e + 1) * I], I)
            U = oracle.matvec_mul_into(fmt, h[t], u[0][e * gb:(e + 1) * gb], u[1][e * I:(e + 1) * I], I)
            M = (G / (1 + np.exp(-G)) * U).astype(np.float32)
            D = oracle.matvec_mul_into(fmt, M, d[0][e * db:(e + 1) * db], d[1][e * H:(e + 1) * H], H)
            out[t] += D * p[t, e]
    return out, order


@pytest.mark.parametrize("fmt", ["log4", "w4zp8", "w8"])
def test_moe_matches_numpy(fmt):
    r = rng(21)
    T, H, I, E, k = 6, 64, 32, 8, 3
    h = r.normal(0, 1, (T, H)).astype(np.float32)
    lg = r.normal(0, 1, (T, E)).astype(np.float32)
    g, u, d = stacked(fmt, E, I, H, r), stacked(fmt, E, I, H, r), stacked(fmt, E, H, I, r)
    if fmt == "w8":
        g, u, d = ((q.view(np.int8), s) for q, s in (g, u, d))
    out, ids, w = oracle.moe_mlp(fmt, h, lg, k, g, u, d)
    ref, order = numpy_moe(fmt, h, lg, k, (g[0].view(np.uint8), g[1]), (u[0].view(np.uint8), u[1]),
                           (d[0].view(np.uint8), d[1]), I)
    assert np.array_equal(ids, order)
    assert np.max(np.abs(out - ref)) <= 1e-5 * np.max(np.abs(ref))
    assert np.array_equal(out, oracle.moe_mlp(fmt, h, lg, k, g, u, d, threads=4)[0])


def test_moe_ties_and_top_k_beyond_experts():
    r = rng(22)
    T, H, I, E = 2, 32, 16, 4
    h = r.normal(0, 1, (T, H)).astype(np.float32)
    lg = np.array([[1.0, 2.0, 2.0, 0.0], [0.0, 0.0, 0.0, 0.0]], np.float32)
    g, u, d = stacked("log4", E, I, H, r), stacked("log4", E, I, H, r), stacked("log4", E, H, I, r)
    _, ids, w = oracle.moe_mlp("log4", h, lg, 2, g, u, d)
    assert ids.tolist() == [[1, 2], [0, 1]]  # equal probabilities keep index order
    assert np.allclose(w[1], 0.25)
    out, ids, _ = oracle.moe_mlp("log4", h, lg, 9, g, u, d)  # top_k > E: every expert
    assert ids.shape == (T, E)


def test_stack_gate_up_layout():
    """Each expert's gate rows, then its up rows (the stacked layout of the MoE call)."""
    from bramha_b200 import stack_gate_up
    r = rng(23)
    E, I, H = 3, 4, 8
    gates = [(r.integers(0, 256, I * H // 2).astype(np.uint8), r.random(I).astype(np.float32)) for _ in range(E)]
    ups = [(r.integers(0, 256, I * H // 2).astype(np.uint8), r.random(I).astype(np.float32)) for _ in range(E)]
    q, s = stack_gate_up(gates, ups)
    rows = q.reshape(E * 2 * I, H // 2)
    for e in range(E):
        assert np.array_equal(rows[2 * I * e:2 * I * e + I].reshape(-1), gates[e][0])
        assert np.array_equal(rows[2 * I * e + I:2 * I * (e + 1)].reshape(-1), ups[e][0])
        assert np.array_equal(s[2 * I * e:2 * I * (e + 1)], np.concatenate([gates[e][1], ups[e][1]]))
