"""Generate the golden fixtures in this folder.

The reference (akshaybhlrp/bramha) is Rust and cannot be built or run here, so
these vectors come from an INDEPENDENT restatement of its arithmetic written
with numpy float32 scalars and plain Python loops (not from the C oracle they
are used to check).  Each function cites the reference lines it restates.

Fixtures:
  kat_quant.npz   -- the fixture of the reference's known-answer test
                     `test_quantization_correctness` (src/inference/cpu_engine.rs:3501-3682):
                     w[i] = cos(0.17 i) * 0.5 (64 x 128), h[i] = sin(0.31 i),
                     h_block[i] = sin(0.23 i) (block 4), plus packed codes, scales,
                     and GEMV / GEMM outputs of the reference loops.
  log4_kat.json   -- hand-derivable decodes of spanda-engine/src/lib.rs:332-342
                     and encoder cases for the log4 quantizer this project defines.

Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import math
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
f32 = np.float32


def rust_round(v: np.float32) -> np.float32:
    """f32::round (half away from zero), evaluated exactly in float64."""
    d = float(v)
    if math.isnan(d):
        return f32(d)
    r = math.floor(abs(d) + 0.5)
    return f32(math.copysign(r, d))


def rust_clamp(v, lo, hi):
    v = f32(v)
    if v < lo:
        v = f32(lo)
    if v > hi:
        v = f32(hi)
    return v


def row_max_abs(row):
    m = f32(0.0)
    for x in row:
        a = f32(abs(x))
        if a > m:
            m = a
    return m


def quantize_to_int8(w, n, k):
    """src/models/quantization.rs:7-38"""
    q = np.zeros(n * k, np.int8)
    s = np.zeros(n, np.float32)
    for j in range(n):
        row = w[j * k:(j + 1) * k]
        m = row_max_abs(row)
        sc = f32(1.0) if m == 0 else f32(m / f32(127.0))
        s[j] = sc
        for i in range(k):
            q[j * k + i] = int(rust_clamp(rust_round(f32(row[i] / sc)), -127.0, 127.0))
    return q, s


def quantize_to_int4(w, n, k):
    """src/models/quantization.rs:41-83 (even column in the high nibble)."""
    half = k // 2
    q = np.zeros(n * half, np.uint8)
    s = np.zeros(n, np.float32)
    for j in range(n):
        row = w[j * k:(j + 1) * k]
        m = row_max_abs(row)
        sc = f32(1.0) if m == 0 else f32(m / f32(7.0))
        s[j] = sc
        for i in range(half):
            q1 = int(f32(rust_clamp(rust_round(f32(row[2 * i] / sc)), -7.0, 7.0) + f32(8.0)))
            q2 = int(f32(rust_clamp(rust_round(f32(row[2 * i + 1] / sc)), -7.0, 7.0) + f32(8.0)))
            q[j * half + i] = ((q1 << 4) | (q2 & 0x0F)) & 0xFF
    return q, s


def log4_value(c: int, scale: np.float32) -> np.float32:
    """spanda-engine/src/lib.rs:335-339: signum(c) * (2^c - 1) * scale, c >= 0."""
    return f32(f32(f32(1.0) * f32(f32(2.0 ** c) - f32(1.0))) * f32(scale))


def quantize_to_log4(w, n, k):
    """Encoder defined by this project: s = max|w|/32767, nearest code, ties low."""
    half = k // 2
    q = np.zeros(n * half, np.uint8)
    s = np.zeros(n, np.float32)
    for j in range(n):
        row = w[j * k:(j + 1) * k]
        m = row_max_abs(row)
        sc = f32(1.0) if m == 0 else f32(m / f32(32767.0))
        s[j] = sc
        d = [log4_value(c, sc) for c in range(16)]
        for i in range(half):
            codes = []
            for t in range(2):
                a = f32(abs(row[2 * i + t]))
                best, best_err = 0, f32(abs(f32(a - d[0])))
                for c in range(1, 16):
                    e = f32(abs(f32(a - d[c])))
                    if e < best_err:
                        best, best_err = c, e
                codes.append(best)
            q[j * half + i] = (codes[0] << 4) | codes[1]
    return q, s


def matvec_into_u4(h, q, s, n, k):
    """matvec_mul_into, QuantizedU4 branch: src/inference/cpu_engine.rs:1363-1411."""
    lut1 = [f32(((i >> 4) & 15) - 8.0) for i in range(256)]
    lut2 = [f32((i & 15) - 8.0) for i in range(256)]
    half = k // 2
    out = np.zeros(n, np.float32)
    for j in range(n):
        rb = q[j * half:(j + 1) * half]
        acc = [f32(0.0)] * 4
        chunks = half // 8
        for c in range(chunks):
            for t in range(8):
                b = int(rb[c * 8 + t])
                hb = c * 16 + 2 * t
                term = f32(f32(h[hb] * lut1[b]) + f32(h[hb + 1] * lut2[b]))
                acc[t % 4] = f32(acc[t % 4] + term)
        tot = f32(f32(f32(acc[0] + acc[1]) + acc[2]) + acc[3])
        for i in range(chunks * 8, half):
            b = int(rb[i])
            tot = f32(tot + f32(f32(h[2 * i] * lut1[b]) + f32(h[2 * i + 1] * lut2[b])))
        out[j] = f32(tot * s[j])
    return out


def matvec_into_i8(h, q, s, n, k):
    """matvec_mul_into, QuantizedI8 branch: src/inference/cpu_engine.rs:1337-1361."""
    out = np.zeros(n, np.float32)
    for j in range(n):
        w = q[j * k:(j + 1) * k]
        acc = [f32(0.0)] * 4
        chunks, rem = k // 4, k % 4
        for i in range(chunks):
            for t in range(4):
                acc[t] = f32(acc[t] + f32(h[4 * i + t] * f32(int(w[4 * i + t]))))
        for i in range(chunks * 4, chunks * 4 + rem):
            acc[0] = f32(acc[0] + f32(h[i] * f32(int(w[i]))))
        out[j] = f32(f32(f32(f32(acc[0] + acc[1]) + acc[2]) + acc[3]) * s[j])
    return out


def gemm_u4(hb, q, s, m, n, k):
    """gemm_cpu, QuantizedU4 sequential branch: src/inference/cpu_engine.rs:607-664."""
    out = np.zeros(m * n, np.float32)
    for b in range(m):
        row = matvec_into_u4(hb[b * k:(b + 1) * k], q, s, n, k)
        out[b * n:(b + 1) * n] = row
    return out


def gemm_i8(hb, q, s, m, n, k):
    """gemm_cpu, QuantizedI8 sequential branch (single accumulator): cpu_engine.rs:592-606."""
    out = np.zeros(m * n, np.float32)
    for j in range(n):
        w = q[j * k:(j + 1) * k]
        for b in range(m):
            acc = f32(0.0)
            for i in range(k):
                acc = f32(acc + f32(hb[b * k + i] * f32(int(w[i]))))
            out[b * n + j] = f32(acc * s[j])
    return out


def main():
    n, k, block = 64, 128, 4
    # The reference computes (i as f32 * 0.17).cos() * 0.5 in f32; evaluate the
    # product in f32 and the cosine of that f32 value in double, then round.
    w = np.array([f32(math.cos(float(f32(f32(i) * f32(0.17))))) for i in range(n * k)], np.float32)
    w = (w * f32(0.5)).astype(np.float32)
    h = np.array([f32(math.sin(float(f32(f32(i) * f32(0.31))))) for i in range(k)], np.float32)
    hb = np.array([f32(math.sin(float(f32(f32(i) * f32(0.23))))) for i in range(block * k)], np.float32)

    q4, s4 = quantize_to_int4(w, n, k)
    q8, s8 = quantize_to_int8(w, n, k)
    ql, sl = quantize_to_log4(w, n, k)
    np.savez_compressed(
        os.path.join(HERE, "kat_quant.npz"),
        w=w, h=h, h_block=hb,
        q4=q4, s4=s4, q8=q8, s8=s8, ql=ql, sl=sl,
        y4_into=matvec_into_u4(h, q4, s4, n, k),
        y8_into=matvec_into_i8(h, q8, s8, n, k),
        g4=gemm_u4(hb, q4, s4, block, n, k),
        g8=gemm_i8(hb, q8, s8, block, n, k),
        shape=np.array([n, k, block], np.int64),
    )

    # Hand-derivable log4 decodes: value = (2^c - 1) * scale, high nibble first.
    data = [0x00, 0x01, 0x10, 0xF0, 0x0F, 0xAB, 0xFF, 0x7E]
    scale = 0.5
    dec = []
    for b in data:
        for c in (b >> 4, b & 15):
            dec.append(float(log4_value(c, f32(scale))))
    # Encoder cases for one 8-wide row (K = 8) with a chosen maximum of 32767 * s.
    row = np.array([0.0, 1.0, -1.0, 0.5, 1.4, 1.6, 3.0, 32767.0], np.float32) * f32(2.0 ** -10)
    eq, es = quantize_to_log4(row, 1, 8)
    payload = {
        "decode": {"bytes": data, "scale": scale, "values": dec},
        "encode": {"row": [float(x) for x in row], "codes": [int(x) for x in eq], "scale": float(es[0])},
    }
    with open(os.path.join(HERE, "log4_kat.json"), "w") as f:
        json.dump(payload, f, indent=1)
    print("wrote kat_quant.npz, log4_kat.json")


if __name__ == "__main__":
    main()
