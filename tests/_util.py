"""Shared helpers for the parity tests: seeded inputs and the error metric."""
import numpy as np

import oracle

# BASELINE shapes (out_features N, in_features K).
QWEN05 = {"q": (896, 896), "k": (128, 896), "v": (128, 896), "o": (896, 896), "gate": (4864, 896),
          "up": (4864, 896), "down": (896, 4864), "lm_head": (151936, 896)}
QWEN7 = {"q": (3584, 3584), "k": (512, 3584), "v": (512, 3584), "o": (3584, 3584), "gate": (18944, 3584),
         "up": (18944, 3584), "down": (3584, 18944), "lm_head": (152064, 3584)}

# GEMV tolerance: max normwise relative error (fp32 accumulate), as stated for this path.
GEMV_TOL = 1e-3
# bf16-tile GEMM tolerance.
GEMM_BF16_TOL = 1e-2


def rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def make_weight(fmt, n, k, seed=0, std=0.02):
    w = rng(seed).normal(0.0, std, n * k).astype(np.float32)
    q, s = oracle.quantize(fmt, w, n, k)
    return w, q, s


def make_x(batch, k, seed=1):
    return rng(seed).normal(0.0, 1.0, (batch, k)).astype(np.float32)


def normwise_err(y, y_ref):
    y = np.asarray(y, np.float64).reshape(-1)
    r = np.asarray(y_ref, np.float64).reshape(-1)
    den = np.max(np.abs(r))
    if den == 0:
        return float(np.max(np.abs(y)))
    return float(np.max(np.abs(y - r)) / den)


def oracle_gemv(fmt, x, q, s, n, threads=0):
    x = np.atleast_2d(x)
    return np.stack([oracle.matvec_mul_into(fmt, xb, q, s, n, threads=threads) for xb in x])
