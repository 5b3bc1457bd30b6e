"""GPU parity of the decode GEMV and the packers, through the C ABI, against the
CPU oracle (restatement of src/inference/cpu_engine.rs:1307-1444 and
src/models/quantization.rs).

Tolerances: GEMV max normwise relative error <= 1e-3 (fp32 accumulate);
packers bit-exact (codes and scales byte-compared).
"""
import numpy as np
import pytest

import oracle
from tests._util import GEMV_TOL, QWEN05, QWEN7, make_weight, make_x, normwise_err, oracle_gemv, rng

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


def run_gemv(plane, w, x):
    xd = dev(x)
    y = torch.empty((x.shape[0], w.N), dtype=torch.float32, device="cuda")
    plane.gemv_dev(w, xd, y)
    torch.cuda.synchronize()
    return y.cpu().numpy()


# ------------------------------------------------------------------ reference KAT
def test_reference_kat_gpu_matches_cpu(plane, golden):
    """Step (4) of test_quantization_correctness (cpu_engine.rs:3649-3681):
    GPU int8/int4 GEMV == CPU matvec_mul within 1e-4, same fixture."""
    n, k, _ = (int(v) for v in golden["shape"])
    h = golden["h"]
    res_q8 = oracle.matvec_mul("w8", h, golden["q8"], golden["s8"], n)
    res_q4 = oracle.matvec_mul("w4zp8", h, golden["q4"], golden["s4"], n)
    gpu8 = plane.matvec_mul_int8(h, golden["q8"], golden["s8"], n, None, None)
    gpu4 = plane.matvec_mul_int4(h, golden["q4"], golden["s4"], n, None, None)
    assert np.max(np.abs(gpu8 - res_q8)) < 1e-4
    assert np.max(np.abs(gpu4 - res_q4)) < 1e-4


# ---------------------------------------------------------------------- packers
@pytest.mark.parametrize("fmt", ["w8", "w4zp8", "log4"])
@pytest.mark.parametrize("n,k", [(64, 128), (7, 30), (129, 896), (3, 4864)])
def test_packers_bit_exact(plane, fmt, n, k):
    w = rng(5).normal(0, 0.02, (n, k)).astype(np.float32)
    w[0, :] = 0.0                     # all-zero row -> scale 1.0
    if n > 2:
        w[1, :4] = [0.5, -0.5, 1.5, -2.5]  # exact halves: round half away from zero
        w[2, 0] = 7.0                      # row max 7 -> int4 scale exactly 1.0
        # just below / at halves: Rust's round never rounds 0.49999997 up
        w[2, 1:6] = [np.float32(0.49999997), -np.float32(0.49999997), np.nextafter(np.float32(1.5), 0), 2.5, -3.5]
    q_ref, s_ref = oracle.quantize(fmt, w.reshape(-1), n, k)
    wd = dev(w)
    qd = torch.zeros(q_ref.size, dtype=torch.uint8, device="cuda")
    sd = torch.zeros(n, dtype=torch.float32, device="cuda")
    plane.quantize_dev(fmt, wd, qd, sd)
    torch.cuda.synchronize()
    assert qd.cpu().numpy().tobytes() == q_ref.view(np.uint8).tobytes()
    assert sd.cpu().numpy().tobytes() == s_ref.tobytes()


# ------------------------------------------------------------------- GEMV parity
@pytest.fixture(params=["tensor_core", "cuda_core"])
def kernel(request, plane):
    """Batch-1 GEMVs of the quantized formats on each of the two kernels."""
    plane.set_gemv_kernel(request.param)
    yield request.param
    plane.set_gemv_kernel("auto")


@pytest.mark.parametrize("fmt", ["w4zp8", "log4", "w8", "f32"])
@pytest.mark.parametrize("name", list(QWEN05))
def test_gemv_qwen05_linears(plane, kernel, fmt, name):
    n, k = QWEN05[name]
    _, q, s = make_weight(fmt, n, k, seed=sum(map(ord, name)))
    x = make_x(1, k, seed=11)
    w = plane.register(f"qwen05:{name}:{fmt}", fmt, n, k, q, s)
    y = run_gemv(plane, w, x)
    y_ref = oracle_gemv(fmt, x, q, s, n)
    assert normwise_err(y, y_ref) <= GEMV_TOL
    plane.evict(w.key)


@pytest.mark.parametrize("fmt", ["log4", "w4zp8", "w8"])
@pytest.mark.parametrize("name", ["q", "k", "o", "down"])
def test_gemv_qwen7_linears(plane, kernel, fmt, name):
    n, k = QWEN7[name]
    _, q, s = make_weight(fmt, n, k, seed=7)
    x = make_x(1, k, seed=12)
    w = plane.register(f"qwen7:{name}:{fmt}", fmt, n, k, q, s)
    y = run_gemv(plane, w, x)
    assert normwise_err(y, oracle_gemv(fmt, x, q, s, n)) <= GEMV_TOL
    plane.evict(w.key)


@pytest.mark.parametrize("fmt", ["log4", "w4zp8", "w8"])
@pytest.mark.parametrize("n,k", [(1, 2), (7, 16), (129, 24), (33, 130), (5, 1000), (300, 34), (2, 18946),
                                 (20000, 4864)])
def test_gemv_ragged_batch1(plane, kernel, fmt, n, k):
    """Ragged rows, columns and blocks at batch 1 on both kernels; (20000, 4864)
    gives the CUDA-core kernel K ranges longer than its register chunk."""
    _, q, s = make_weight(fmt, n, k, seed=n * 17 + k)
    x = make_x(1, k, seed=n + 3 * k)
    w = plane.register(f"ragged1:{fmt}:{n}x{k}", fmt, n, k, q, s)
    y = plane.gemv(w, x)
    assert normwise_err(y, oracle_gemv(fmt, x, q, s, n)) <= GEMV_TOL
    plane.evict(w.key)


@pytest.mark.parametrize("fmt", ["log4", "w4zp8", "w8", "f32"])
@pytest.mark.parametrize("batch", [1, 2, 3, 4, 5, 8, 11])
def test_gemv_batches(plane, fmt, batch):
    n, k = 1000, 1536
    _, q, s = make_weight(fmt, n, k, seed=batch)
    x = make_x(batch, k, seed=100 + batch)
    w = plane.register(f"batch:{fmt}:{batch}", fmt, n, k, q, s)
    y = run_gemv(plane, w, x)
    assert normwise_err(y, oracle_gemv(fmt, x, q, s, n)) <= GEMV_TOL
    # every batch row on its own (no cross-talk between rows)
    for b in range(batch):
        assert normwise_err(y[b], oracle_gemv(fmt, x[b:b + 1], q, s, n)) <= GEMV_TOL
    plane.evict(w.key)


@pytest.mark.parametrize("fmt", ["log4", "w4zp8", "w8", "f32"])
@pytest.mark.parametrize("n,k", [(1, 2), (7, 16), (129, 24), (33, 130), (5, 1000), (300, 34), (2, 18946)])
def test_gemv_ragged_shapes(plane, fmt, n, k):
    _, q, s = make_weight(fmt, n, k, seed=n * 31 + k)
    x = make_x(2, k, seed=n + k)
    w = plane.register(f"ragged:{fmt}:{n}x{k}", fmt, n, k, q, s)
    y = plane.gemv(w, x)  # host path: unaligned K handled by the staging copy
    assert normwise_err(y, oracle_gemv(fmt, x, q, s, n)) <= GEMV_TOL
    plane.evict(w.key)


def test_odd_k_ignores_last_column_like_reference(plane):
    """matvec_mul_into's U4 branch reads K/2 bytes per row (cpu_engine.rs:1364):
    with odd K the last activation is ignored."""
    n, k = 9, 33
    q = rng(3).integers(0, 256, n * (k // 2), dtype=np.uint8)
    s = rng(4).uniform(0.01, 0.1, n).astype(np.float32)
    x = make_x(1, k, seed=5)
    for fmt in ("w4zp8", "log4"):
        y = plane.matvec_mul_int4(x[0], q, s, n) if fmt == "w4zp8" else plane.matvec_mul_log4(x[0], q, s, n)
        assert normwise_err(y, oracle_gemv(fmt, x, q, s, n)) <= GEMV_TOL


def test_fused_multi_weight_launch_matches_separate(plane, kernel):
    k = 896
    x = make_x(1, k, seed=21)
    ws, refs = [], []
    for i, name in enumerate(["q", "k", "v"]):
        n = QWEN05[name][0]
        _, q, s = make_weight("log4", n, k, seed=40 + i)
        ws.append(plane.register(f"fused:{name}", "log4", n, k, q, s))
        refs.append(oracle_gemv("log4", x, q, s, n))
    xd = dev(x)
    ys = [torch.empty((1, w.N), dtype=torch.float32, device="cuda") for w in ws]
    plane.gemv_multi_dev(ws, xd, ys)
    torch.cuda.synchronize()
    for y, r in zip(ys, refs):
        assert normwise_err(y.cpu().numpy(), r) <= GEMV_TOL
    for w in ws:
        plane.evict(w.key)


# --------------------------------------------------------- reference conventions
def test_errors_and_empty_shapes_like_reference(plane):
    from bramha_b200 import BramhaError
    h = np.ones(8, np.float32)
    with pytest.raises(BramhaError, match="Quantized INT4 weight size mismatch"):
        plane.matvec_mul_int4(h, np.zeros(7, np.uint8), np.ones(2, np.float32), 2)
    with pytest.raises(BramhaError, match="Quantized INT8 weight size mismatch"):
        plane.matvec_mul_int8(h, np.zeros(15, np.int8), np.ones(2, np.float32), 2)
    with pytest.raises(BramhaError, match="Weight size mismatch"):
        plane.matvec_mul(h, np.zeros(15, np.float32), 2)
    # N == 0 or K == 0 -> zeros (wgpu_backend.rs:1092-1095)
    assert plane.matvec_mul_int4(np.zeros(0, np.float32), np.zeros(0, np.uint8), np.ones(3, np.float32), 3).tolist() == [0, 0, 0]
    assert plane.matvec_mul_int4(h, np.zeros(0, np.uint8), np.zeros(0, np.float32), 0).size == 0


def test_keyed_cache_and_lru_eviction(plane):
    n, k = 256, 512
    x = make_x(1, k, seed=1)[0]
    _, q1, s1 = make_weight("w4zp8", n, k, seed=1)
    _, q2, s2 = make_weight("w4zp8", n, k, seed=2)
    y1 = plane.matvec_mul_int4(x, q1, s1, n, "m", "l1")
    # same key: cached -- even if different bytes are passed, the cached weight is used
    y1b = plane.matvec_mul_int4(x, q2, s2, n, "m", "l1")
    assert np.array_equal(y1, y1b)
    w1 = plane.lookup("m:l1")
    per = w1.device_bytes
    plane.set_memory_cap(per + per // 2)
    plane.matvec_mul_int4(x, q2, s2, n, "m", "l2")  # forces eviction of m:l1 (least recently used)
    from bramha_b200 import BramhaError
    with pytest.raises(BramhaError):
        plane.lookup("m:l1")
    with pytest.raises(BramhaError, match="evicted"):
        plane.gemv(w1, x)
    assert plane.memory_used() <= per + per // 2
    plane.set_memory_cap(0)
    plane.clear_persistent_buffers()
    assert plane.memory_used() == 0


def test_gemm_host_matches_gemm_cpu(plane):
    n, k, m = 320, 896, 64
    for fmt in ("w4zp8", "w8", "log4"):
        _, q, s = make_weight(fmt, n, k, seed=9)
        hb = make_x(m, k, seed=10)
        w = plane.register(f"gemm:{fmt}", fmt, n, k, q, s)
        out = plane.gemm(w, hb, m)
        ref = oracle.gemm_cpu(fmt, hb, q, s, m, k, n)
        assert normwise_err(out, ref) <= GEMV_TOL
        plane.evict(w.key)


# --------------------------------------------- full-size, size-independent checks
@pytest.mark.parametrize("fmt", ["log4", "w4zp8"])
def test_lm_head_full_size_linearity_and_oracle(plane, fmt):
    """Qwen2-7B lm_head (152064 x 3584), weights generated and packed on the
    device; parity with the oracle on the same packed bytes, plus linearity."""
    n, k = QWEN7["lm_head"]
    g = torch.Generator(device="cuda").manual_seed(1234)
    wf = torch.randn((n, k), generator=g, device="cuda", dtype=torch.float32) * 0.02
    qd = torch.empty(n * (k // 2), dtype=torch.uint8, device="cuda")
    sd = torch.empty(n, dtype=torch.float32, device="cuda")
    plane.quantize_dev(fmt, wf, qd, sd)
    # packer bit-exact on a slab of rows
    rows = slice(1000, 1064)
    q_ref, s_ref = oracle.quantize(fmt, wf[rows].cpu().numpy().reshape(-1), 64, k)
    assert qd.view(n, k // 2)[rows].cpu().numpy().tobytes() == q_ref.tobytes()
    del wf
    w = plane.register_dev(f"lm_head7:{fmt}", fmt, n, k, qd, sd)
    x = make_x(2, k, seed=77)
    y = run_gemv(plane, w, x)
    q, s = qd.cpu().numpy(), sd.cpu().numpy()
    assert normwise_err(y[0], oracle_gemv(fmt, x[:1], q, s, n)) <= GEMV_TOL
    # linearity: W(a x0 + b x1) == a W x0 + b W x1
    xc = (0.75 * x[0] - 1.5 * x[1])[None, :].astype(np.float32)
    yc = run_gemv(plane, w, xc)
    assert normwise_err(yc[0], 0.75 * y[0] - 1.5 * y[1]) <= GEMV_TOL
    plane.evict(w.key)
