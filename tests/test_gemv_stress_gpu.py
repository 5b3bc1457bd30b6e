"""GPU parity of the decode GEMV at the Qwen2-7B shapes and batches of BASELINE
config 4 (batch 1, 8, 64), and under activations that stress the kernels'
scaled 8-bit activation terms, against the CPU oracle (restatement of
`matvec_mul_into`, src/inference/cpu_engine.rs:1307-1444; batched rows as
`gemm_cpu`, :565-912, computes them).

The tensor-core GEMV turns each activation row into 8-bit terms scaled by a
power of two chosen from max|x| over the CTA's K range; batches above 8 run on
the tcgen05 GEMM with the rows split into bf16 hi + lo.  Tolerance: max
normwise relative error <= 1e-3 (fp32 accumulate), as for every GEMV test.
"""
import numpy as np
import pytest

import oracle
from tests._util import GEMV_TOL, QWEN7, make_weight, make_x, normwise_err, oracle_gemv, rng

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


@pytest.fixture(params=["tensor_core", "cuda_core"])
def kernel(request, plane):
    plane.set_gemv_kernel(request.param)
    yield request.param
    plane.set_gemv_kernel("auto")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_gemv(plane, w, x):
    y = torch.empty((x.shape[0], w.N), dtype=torch.float32, device="cuda")
    plane.gemv_dev(w, dev(x), y)
    plane.stream_sync()
    return y.cpu().numpy()


def device_weight(plane, key, fmt, n, k, seed):
    """A ~N(0, 0.02) weight generated and packed on the device; returns the
    registered weight and its packed bytes / scales on the host."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    wf = torch.randn((n, k), generator=g, device="cuda", dtype=torch.float32) * 0.02
    nb = n * k if fmt == "w8" else n * (k // 2)
    qd = torch.empty(nb, dtype=torch.uint8, device="cuda")
    sd = torch.empty(n, dtype=torch.float32, device="cuda")
    plane.quantize_dev(fmt, wf, qd, sd)
    del wf
    w = plane.register_dev(key, fmt, n, k, qd, sd)
    q, s = qd.cpu().numpy(), sd.cpu().numpy()
    if fmt == "w8":
        q = q.view(np.int8)
    return w, q, s


def row_slab(fmt, q, s, k, r0, r1):
    """Packed rows [r0, r1) of a row-major packed weight."""
    rb = k if fmt == "w8" else k // 2
    return q[r0 * rb:r1 * rb], s[r0:r1]


# ------------------------------------------------------------ Qwen2-7B shapes
@pytest.mark.parametrize("fmt", ["log4", "w4zp8", "w8"])
def test_gate_up_fused_batch1(plane, kernel, fmt):
    """The bench's dominant launch: gate|up (2 x 18944 x 3584) fused in one launch."""
    n, k = QWEN7["gate"]
    wg, qg, sg = device_weight(plane, f"s7:gate:{fmt}", fmt, n, k, 101)
    wu, qu, su = device_weight(plane, f"s7:up:{fmt}", fmt, n, k, 102)
    x = make_x(1, k, seed=103)
    yg = torch.empty((1, n), device="cuda")
    yu = torch.empty((1, n), device="cuda")
    plane.gemv_multi_dev([wg, wu], dev(x), [yg, yu])
    plane.stream_sync()
    assert normwise_err(yg.cpu().numpy(), oracle_gemv(fmt, x, qg, sg, n)) <= GEMV_TOL
    assert normwise_err(yu.cpu().numpy(), oracle_gemv(fmt, x, qu, su, n)) <= GEMV_TOL
    plane.evict(wg.key)
    plane.evict(wu.key)


@pytest.mark.parametrize("batch", [8, 64])
@pytest.mark.parametrize("fmt,name", [("log4", "q"), ("log4", "gate"), ("log4", "down"), ("w4zp8", "q"),
                                      ("w4zp8", "down"), ("w8", "q"), ("w8", "gate")])
def test_qwen7_batched(plane, fmt, name, batch):
    """Config 4 at batch 8 (tensor-core GEMV, 8 rows per launch) and 64 (tcgen05
    GEMM, K-split for the 28-block q / down): every row against the oracle."""
    n, k = QWEN7[name]
    w, q, s = device_weight(plane, f"b7:{fmt}:{name}:{batch}", fmt, n, k, 7 + batch)
    x = make_x(batch, k, seed=200 + batch)
    y = run_gemv(plane, w, x)
    y_ref = oracle_gemv(fmt, x, q, s, n)
    assert normwise_err(y, y_ref) <= GEMV_TOL
    for b in (0, batch // 2, batch - 1):  # no cross-talk between rows
        assert normwise_err(y[b], y_ref[b]) <= GEMV_TOL
    plane.evict(w.key)


@pytest.mark.parametrize("batch", [8, 64])
def test_qwen7_lm_head_batched(plane, batch):
    """lm_head (152064 x 3584, log4) at batch 8 and 64: a slab of rows against
    the oracle, and linearity over the batch rows for the whole output."""
    n, k = QWEN7["lm_head"]
    w, q, s = device_weight(plane, f"lm7b:{batch}", "log4", n, k, 31)
    x = make_x(batch, k, seed=32)
    y = run_gemv(plane, w, x)
    r0, r1 = 70000, 72048
    qs, ss = row_slab("log4", q, s, k, r0, r1)
    for b in (0, batch - 1):
        assert normwise_err(y[b, r0:r1], oracle_gemv("log4", x[b:b + 1], qs, ss, r1 - r0)) <= GEMV_TOL
    # linearity: W (x0 + 2 x1) == W x0 + 2 W x1 over all 152064 outputs
    xc = np.repeat((x[0] + 2.0 * x[1])[None, :], batch, axis=0).astype(np.float32)
    yc = run_gemv(plane, w, xc)
    assert normwise_err(yc[0], y[0] + 2.0 * y[1]) <= GEMV_TOL
    plane.evict(w.key)


@pytest.mark.parametrize("fmt", ["log4", "w8"])
@pytest.mark.parametrize("batch", [9, 16, 33])
def test_batched_ragged(plane, fmt, batch):
    """Batches above 8 on ragged shapes (tail rows, tail columns, K-split ranges)."""
    for n, k in ((300, 1000), (2000, 4864), (33, 130)):
        _, q, s = make_weight(fmt, n, k, seed=n + batch)
        x = make_x(batch, k, seed=k + batch)
        w = plane.register(f"br:{fmt}:{n}x{k}:{batch}", fmt, n, k, q, s)
        y = plane.gemv(w, x)  # host path (unaligned K staged)
        assert normwise_err(y, oracle_gemv(fmt, x, q, s, n)) <= GEMV_TOL
        plane.evict(w.key)


def test_swiglu_batched_matches_separate(plane):
    """gemv_swiglu_dev at batch 16 (GEMM route) equals silu_mul + GEMV."""
    n, k, b = 896, 4864, 16
    _, q, s = make_weight("log4", n, k, seed=5)
    w = plane.register("swb:down", "log4", n, k, q, s)
    g, u = dev(make_x(b, k, seed=6)), dev(make_x(b, k, seed=7))
    y1 = torch.empty((b, n), device="cuda")
    plane.gemv_swiglu_dev(w, g, u, y1)
    act = g * torch.sigmoid(g) * u  # only for the tolerance check below
    from bramha_b200 import lib
    from bramha_b200.plane import _stream
    act2 = torch.empty_like(g)
    assert lib().bramha_cuda_op_silu_mul(plane.ctx, g.data_ptr(), u.data_ptr(), g.numel(), act2.data_ptr(),
                                         _stream(None)) == 0
    y2 = torch.empty((b, n), device="cuda")
    plane.gemv_dev(w, act2, y2)
    plane.stream_sync()
    assert torch.equal(y1, y2)
    ref = oracle_gemv("log4", act.cpu().numpy(), q, s, n)
    assert normwise_err(y1.cpu().numpy(), ref) <= GEMV_TOL
    plane.evict(w.key)


# ----------------------------------------------------- activation stress cases
def stress_x(kind, batch, k, seed):
    x = make_x(batch, k, seed=seed)
    r = rng(seed + 1)
    if kind == "outlier_1e3":
        x[:, r.integers(0, k)] = 1e3
    elif kind == "outlier_1e4":
        x[:, r.integers(0, k)] = -1e4
    elif kind == "half_zero":
        x[:, r.permutation(k)[:k // 2]] = 0.0
    elif kind == "tiny":  # max|x| = 2^-20
        x = (x / np.max(np.abs(x), axis=1, keepdims=True) * np.float32(2.0 ** -20)).astype(np.float32)
    elif kind == "tiny_tail":  # the second half of K is 2^-20-scaled
        h = k // 2
        x[:, h:] = x[:, h:] / np.max(np.abs(x[:, h:]), axis=1, keepdims=True) * np.float32(2.0 ** -20)
    elif kind == "mixed_scales":  # magnitudes spread over 2^-12 .. 2^12
        x = (x * np.exp2(r.integers(-12, 13, (batch, k)))).astype(np.float32)
    return np.ascontiguousarray(x, np.float32)


KINDS = ["outlier_1e3", "outlier_1e4", "half_zero", "tiny", "tiny_tail", "mixed_scales"]


@pytest.mark.parametrize("fmt", ["log4", "w4zp8", "w8"])
@pytest.mark.parametrize("kind", KINDS)
def test_stress_batch1_both_kernels(plane, kernel, fmt, kind):
    n, k = 1000, 1536
    _, q, s = make_weight(fmt, n, k, seed=61)
    x = stress_x(kind, 1, k, seed=62)
    w = plane.register(f"stress:{fmt}", fmt, n, k, q, s)
    y = run_gemv(plane, w, x)
    assert normwise_err(y, oracle_gemv(fmt, x, q, s, n)) <= GEMV_TOL
    plane.evict(w.key)


@pytest.mark.parametrize("fmt", ["log4", "w4zp8", "w8"])
@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("batch", [1, 4, 16])
def test_stress_qwen7_q(plane, fmt, kind, batch):
    """7B q (3584 x 3584): K-split ranges of the tensor-core GEMV (batch 1, 4)
    and the GEMM route (batch 16) under the same stress activations."""
    n, k = QWEN7["q"]
    w, q, s = device_weight(plane, f"stress7:{fmt}", fmt, n, k, 63)
    x = stress_x(kind, batch, k, seed=64 + batch)
    y = run_gemv(plane, w, x)
    assert normwise_err(y, oracle_gemv(fmt, x, q, s, n)) <= GEMV_TOL
    plane.evict(w.key)
