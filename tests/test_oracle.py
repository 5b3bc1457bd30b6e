"""The CPU oracle against the reference's own known-answer test and the golden
fixtures (independent numpy restatement + hand-derived log4 values).

Restates `test_quantization_correctness` (src/inference/cpu_engine.rs:3501-3682).
"""
import json
import os

import numpy as np
import pytest

import oracle

HERE = os.path.dirname(os.path.abspath(__file__))


def test_packers_match_golden_bit_exact(golden):
    n, k, _ = golden["shape"]
    w = golden["w"]
    q4, s4 = oracle.quantize_to_int4(w, n, k)
    q8, s8 = oracle.quantize_to_int8(w, n, k)
    ql, sl = oracle.quantize_to_log4(w, n, k)
    assert np.array_equal(q4, golden["q4"]) and s4.tobytes() == golden["s4"].tobytes()
    assert np.array_equal(q8, golden["q8"]) and s8.tobytes() == golden["s8"].tobytes()
    assert np.array_equal(ql, golden["ql"]) and sl.tobytes() == golden["sl"].tobytes()


def test_gemv_gemm_match_golden_bit_exact(golden):
    n, k, block = (int(v) for v in golden["shape"])
    h, hb = golden["h"], golden["h_block"]
    y4 = oracle.matvec_mul_into("w4zp8", h, golden["q4"], golden["s4"], n, threads=1)
    y8 = oracle.matvec_mul_into("w8", h, golden["q8"], golden["s8"], n, threads=1)
    assert y4.tobytes() == golden["y4_into"].tobytes()
    assert y8.tobytes() == golden["y8_into"].tobytes()
    g4 = oracle.gemm_cpu("w4zp8", hb, golden["q4"], golden["s4"], block, k, n)
    g8 = oracle.gemm_cpu("w8", hb, golden["q8"], golden["s8"], block, k, n)
    assert g4.tobytes() == golden["g4"].tobytes()
    assert g8.tobytes() == golden["g8"].tobytes()


def test_reference_kat_test_quantization_correctness(golden):
    """cpu_engine.rs:3515-3647, restated assertion by assertion."""
    n, k, block = (int(v) for v in golden["shape"])
    w, h, hb = golden["w"], golden["h"], golden["h_block"]
    for fmt, q_fn, dq_fn in (
        ("w8", oracle.quantize_to_int8, oracle.dequantize_int8),
        ("w4zp8", oracle.quantize_to_int4, oracle.dequantize_int4),
    ):
        q, s = q_fn(w, n, k)
        deq = dq_fn(q, s, k)
        # (1) round-trip error <= scale/2 + 1e-5
        err = np.abs(w.reshape(n, k) - deq.reshape(n, k))
        assert np.all(err <= s[:, None] * 0.5 + 1e-5)
        # (2) quantized matvec_mul == dequantized matvec_mul within 1e-4
        res_float = oracle.matvec_mul("f32", h, deq, None, n)
        res_q = oracle.matvec_mul(fmt, h, q, s, n)
        assert np.max(np.abs(res_float - res_q)) < 1e-4
        # (3) quantized gemm_cpu == dequantized gemm_cpu within 1e-4
        gf = oracle.gemm_cpu("f32", hb, deq, None, block, k, n)
        gq = oracle.gemm_cpu(fmt, hb, q, s, block, k, n)
        assert np.max(np.abs(gf - gq)) < 1e-4


def test_log4_decoder_known_answers():
    kat = json.load(open(os.path.join(HERE, "golden", "log4_kat.json")))
    dec = kat["decode"]
    got = oracle.dequantize_log4(np.array(dec["bytes"], np.uint8), dec["scale"])
    assert got.tolist() == dec["values"]
    # high nibble first, value (2^c - 1) * scale, never negative
    assert got[1] == 0.0 and got[3] == 0.5 and np.all(got >= 0)


def test_log4_encoder_known_answers():
    kat = json.load(open(os.path.join(HERE, "golden", "log4_kat.json")))["encode"]
    row = np.array(kat["row"], np.float32)
    q, s = oracle.quantize_to_log4(row, 1, row.size)
    assert q.tolist() == kat["codes"] and float(s[0]) == kat["scale"]


def test_log4_roundtrip_is_nearest_code():
    rng = np.random.default_rng(7)
    n, k = 16, 96
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    q, s = oracle.quantize_to_log4(w, n, k)
    deq = oracle.dequantize_log4_rows(q, s, k).reshape(n, k)
    for j in range(n):
        d = np.array([(2.0 ** c - 1) * s[j] for c in range(16)], np.float32)
        best = np.min(np.abs(np.abs(w[j])[:, None] - d[None, :]), axis=1)
        assert np.allclose(np.abs(np.abs(w[j]) - deq[j]), best, rtol=0, atol=1e-12)
    # the largest magnitude of each row is reproduced by code 15
    assert np.allclose(deq.max(axis=1), np.abs(w).max(axis=1), rtol=1e-6)


def test_log4_gemv_oracle_matches_dequantized_float():
    rng = np.random.default_rng(3)
    n, k = 40, 256
    w = rng.normal(0, 0.02, n * k).astype(np.float32)
    x = rng.normal(0, 1, k).astype(np.float32)
    q, s = oracle.quantize_to_log4(w, n, k)
    deq = oracle.dequantize_log4_rows(q, s, k)
    y = oracle.matvec_mul_into("log4", x, q, s, n, threads=1)
    yf = oracle.matvec_mul_into("f32", x, deq, None, n, threads=1)
    assert y.tobytes() == yf.tobytes()
    yfused = oracle.matvec_fused_log4(x, q, s, n, threads=1)
    assert np.max(np.abs(yfused - y)) <= 1e-5 * np.max(np.abs(y))


def test_threading_does_not_change_results():
    rng = np.random.default_rng(11)
    n, k = 1030, 200
    w = rng.normal(0, 0.02, n * k).astype(np.float32)
    x = rng.normal(0, 1, k).astype(np.float32)
    q, s = oracle.quantize_to_int4(w, n, k)
    a = oracle.matvec_mul_into("w4zp8", x, q, s, n, threads=1)
    b = oracle.matvec_mul_into("w4zp8", x, q, s, n, threads=4)
    assert a.tobytes() == b.tobytes()


def test_int4_odd_k_rejected_like_reference_assert():
    with pytest.raises(ValueError):
        oracle.quantize_to_int4(np.zeros(6, np.float32), 2, 3)


def test_rust_cast_edge_cases():
    # all-zero row -> scale 1.0; values exactly on .5 round away from zero
    w = np.array([0, 0, 0, 0, 7, 3.5, -3.5, 0.5], np.float32)
    q, s = oracle.quantize_to_int4(w, 2, 4)
    assert s.tolist() == [1.0, 1.0]
    assert q.tolist() == [0x88, 0x88, (15 << 4) | 12, (4 << 4) | 9]
