"""GPU parity of the tcgen05 prefill dequant-GEMM (gemm_cpu, cpu_engine.rs:565-912)
through the C ABI.

References: the CPU oracle's gemm_cpu restatement at sizes it finishes quickly,
and a plain PyTorch fp32 matmul (TF32 off) of the oracle-dequantized weights at
BASELINE config-3 sizes.

Tolerances (max normwise relative error):
  * bf16 activations, one tcgen05 pass: <= 1e-2 (bf16 tiles; the weights are
    exact in bf16, so the error is fp32 accumulation only and is far smaller);
  * f32 activations (hi + lo bf16 split, two passes) and the host call: <= 1e-3.
"""
import numpy as np
import pytest

import oracle
from tests._util import GEMM_BF16_TOL, GEMV_TOL, QWEN05, make_weight, normwise_err, rng

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def plane():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from bramha_b200 import CudaComputePlane
    torch.backends.cuda.matmul.allow_tf32 = False
    p = CudaComputePlane(0)
    yield p
    p.close()


def bf16_x(m, k, seed):
    x = torch.from_numpy(rng(seed).normal(0, 1, (m, k)).astype(np.float32)).to(torch.bfloat16)
    return x


def torch_ref(fmt, q, s, n, k, x_f32_dev):
    w = torch.from_numpy(oracle.dequantize(fmt, q, s, k).reshape(n, k)).cuda()
    return (x_f32_dev @ w.T).cpu().numpy()


def run_gemm_dev(plane, w, x_dev):
    y = torch.empty((x_dev.shape[0], w.N), dtype=torch.float32, device="cuda")
    plane.gemm_dev(w, x_dev, y)
    plane.stream_sync()
    return y.cpu().numpy()


@pytest.mark.parametrize("fmt", ["log4", "w8", "w4zp8"])
@pytest.mark.parametrize("m", [1, 7, 32, 33, 64, 100, 128, 255, 256, 300])
def test_gemm_bf16_tile_widths_vs_oracle(plane, fmt, m):
    n, k = 200, 192
    _, q, s = make_weight(fmt, n, k, seed=m)
    xb = bf16_x(m, k, seed=m + 1)
    w = plane.register(f"g:{fmt}:{m}", fmt, n, k, q, s)
    y = run_gemm_dev(plane, w, xb.cuda())
    ref = oracle.gemm_cpu(fmt, xb.float().numpy(), q, s, m, k, n).reshape(m, n)
    assert normwise_err(y, ref) <= GEMM_BF16_TOL
    assert normwise_err(y, ref) <= 1e-4  # exact weights: only fp32 accumulation differs
    plane.evict(w.key)


@pytest.mark.parametrize("fmt", ["log4", "w8", "w4zp8"])
@pytest.mark.parametrize("n,k", [(129, 64), (1, 130), (300, 1000), (64, 34), (257, 4864)])
def test_gemm_ragged_shapes(plane, fmt, n, k):
    m = 40
    _, q, s = make_weight(fmt, n, k, seed=n + k)
    xb = bf16_x(m, k, seed=3)
    w = plane.register(f"gr:{fmt}:{n}x{k}", fmt, n, k, q, s)
    y = run_gemm_dev(plane, w, xb.cuda())
    ref = oracle.gemm_cpu(fmt, xb.float().numpy(), q, s, m, k, n).reshape(m, n)
    assert normwise_err(y, ref) <= 1e-4
    plane.evict(w.key)


@pytest.mark.parametrize("fmt", ["log4", "w8"])
@pytest.mark.parametrize("name", ["q", "k", "gate", "down"])
def test_gemm_prefill_config3(plane, fmt, name):
    """Config 3: M = 2048 tokens of bf16 ~N(0,1) on the Qwen2-0.5B linears."""
    n, k = QWEN05[name]
    m = 2048
    _, q, s = make_weight(fmt, n, k, seed=5)
    xb = bf16_x(m, k, seed=6).cuda()
    w = plane.register(f"p3:{fmt}:{name}", fmt, n, k, q, s)
    y = run_gemm_dev(plane, w, xb)
    ref = torch_ref(fmt, q, s, n, k, xb.float())
    err = normwise_err(y, ref)
    assert err <= GEMM_BF16_TOL
    assert err <= 1e-4
    plane.evict(w.key)


@pytest.mark.parametrize("fmt", ["log4", "w4zp8", "w8"])
def test_gemm_f32_split_matches_fp32(plane, fmt):
    """f32 activations: hi/lo bf16 split reproduces fp32 within 1e-3."""
    n, k, m = 384, 896, 96
    _, q, s = make_weight(fmt, n, k, seed=8)
    x = rng(9).normal(0, 1, (m, k)).astype(np.float32)
    w = plane.register(f"gs:{fmt}", fmt, n, k, q, s)
    y = run_gemm_dev(plane, w, torch.from_numpy(x).cuda())
    ref = oracle.gemm_cpu(fmt, x, q, s, m, k, n).reshape(m, n)
    assert normwise_err(y, ref) <= GEMV_TOL
    assert normwise_err(y, ref) <= 1e-4
    plane.evict(w.key)


@pytest.mark.parametrize("fmt", ["log4", "w8", "w4zp8"])
@pytest.mark.parametrize("xdt", ["bf16", "f32"])
def test_gemm_sm_pair_ragged(plane, fmt, xdt):
    """The SM-pair kernel (tcgen05.mma.cta_group::2, taken for >= 4 rounds of
    256 x 256 tiles) on ragged rows (N % 256 = 100, the last tile's second
    128-row block absent), tokens (M % 256 = 219) and K (900 = 14 steps + 4),
    with bf16 activations and with the f32 hi|lo split (two K halves)."""
    n, k, m = 9828, 900, 2011
    _, q, s = make_weight(fmt, n, k, seed=21)
    if xdt == "bf16":
        x = bf16_x(m, k, seed=22).cuda()
        xf = x.float()
    else:
        x = torch.from_numpy(rng(23).normal(0, 1, (m, k)).astype(np.float32)).cuda()
        xf = x
    w = plane.register(f"pair:{fmt}:{xdt}", fmt, n, k, q, s)
    y = run_gemm_dev(plane, w, x)
    ref = torch_ref(fmt, q, s, n, k, xf)
    err = normwise_err(y, ref)
    assert err <= (GEMM_BF16_TOL if xdt == "bf16" else GEMV_TOL)
    assert err <= 1e-4
    plane.evict(w.key)


def test_gemm_lm_head_full_size_properties(plane):
    """Qwen2-0.5B lm_head (151936 x 896), M = 256, log4: a row slice against
    the oracle, and linearity in the activations (full output)."""
    n, k = QWEN05["lm_head"]
    m = 256
    g = torch.Generator(device="cuda").manual_seed(17)
    wf = torch.randn((n, k), generator=g, device="cuda") * 0.02
    qd = torch.empty(n * (k // 2), dtype=torch.uint8, device="cuda")
    sd = torch.empty(n, dtype=torch.float32, device="cuda")
    plane.quantize_dev("log4", wf, qd, sd)
    del wf
    w = plane.register_dev("lm05:log4", "log4", n, k, qd, sd)
    xa = bf16_x(m, k, seed=1).cuda()
    xb = bf16_x(m, k, seed=2).cuda()
    ya = run_gemm_dev(plane, w, xa)
    yb = run_gemm_dev(plane, w, xb)
    yab = run_gemm_dev(plane, w, (xa.float() + xb.float()).to(torch.bfloat16))
    # xa + xb is not exact in bf16; compare against the bf16-rounded sum's own reference direction
    rows = slice(70000, 70512)
    q = qd.view(n, k // 2)[rows].cpu().numpy().reshape(-1)
    s = sd[rows].cpu().numpy()
    ref = oracle.gemm_cpu("log4", xa.float().cpu().numpy(), q, s, m, k, 512).reshape(m, 512)
    assert normwise_err(ya[:, rows], ref) <= 1e-4
    assert normwise_err(yab, ya + yb) <= 1e-2
    plane.evict(w.key)
