"""2:4 structured-sparse GEMV on the GPU (sparse24.cu through the C ABI) against
the oracle's restatement of the reference (sparse.rs:19-138,
cpu_engine.rs:1532-1640).

The kernel computes in fp32 with fp32 accumulation and a different summation
order than the reference's sequential loop, so outputs agree within a
normwise relative error of 1e-5; the selection itself (which two of four
are kept, ties to the lower column) must be exact, and a single wrong pick
moves a row by ~1e-2 of the norm, far outside the tolerance.  The known-answer
cases are small integers and must match bit for bit.
"""
import numpy as np
import pytest

import oracle
from tests._util import make_weight, normwise_err, rng

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 1e-5


@pytest.fixture(scope="module")
def plane():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from bramha_b200 import CudaComputePlane
    p = CudaComputePlane(0)
    yield p
    p.close()


def weights(fmt, n, k, seed):
    if fmt == "f32":
        return rng(seed).normal(0, 0.05, n * k).astype(np.float32), None
    _, q, s = make_weight(fmt, n, k, seed=seed)
    return q, s


def test_reference_known_answers(plane):
    from tests.test_sparse24_oracle import KAT_MASKS, KAT_VALUES, KAT_W
    x = np.ones(8, np.float32)
    assert plane.sparse_matvec_mul_2_4(x, KAT_W, 8).tolist() == [8.0, -8.0]
    assert plane.sparse_matvec_2_4_compressed(x, KAT_MASKS, KAT_VALUES, 2, 8).tolist() == [8.0, -8.0]


@pytest.mark.parametrize("fmt,n,k", [
    ("f32", 896, 896), ("f32", 200, 1001), ("f32", 64, 18944),
    ("w8", 896, 4864), ("w8", 130, 1003), ("w8", 4864, 896),
    ("w4zp8", 4864, 896), ("w4zp8", 896, 4864), ("w4zp8", 130, 1002), ("w4zp8", 3, 2)])
def test_pruned_gemv_vs_oracle(plane, fmt, n, k):
    q, s = weights(fmt, n, k, seed=n + k)
    x = rng(k).normal(0, 1, k).astype(np.float32)
    w = plane.register_sparse24(f"sp:{fmt}:{n}:{k}", fmt, n, k, q, s)
    assert w.fmt == "sp24_" + fmt and plane.lookup(w.key).fmt == "sp24_" + fmt
    y = plane.gemv(w, x)
    ref = oracle.sparse_matvec_2_4(fmt, x, q, s, n)
    assert normwise_err(y, ref) <= TOL
    assert np.array_equal(y, plane.gemv(w, x))  # deterministic, K-split included
    plane.evict(w.key)


def test_qwen7b_mlp_shapes_w4zp8(plane):
    """gate (18944 x 3584) and down (3584 x 18944) of Qwen2-7B, int4 codes."""
    for n, k in [(18944, 3584), (3584, 18944)]:
        q, s = weights("w4zp8", n, k, seed=7)
        x = rng(3).normal(0, 1, k).astype(np.float32)
        w = plane.register_sparse24(f"sp7b:{n}", "w4zp8", n, k, q, s)
        y = plane.gemv(w, x)
        ref = oracle.sparse_matvec_2_4("w4zp8", x, q, s, n, threads=oracle.max_threads())
        assert normwise_err(y, ref) <= TOL
        plane.evict(w.key)


def test_ties_and_nan(plane):
    # int4 codes from {6, 10}: every magnitude is 2, so each group keeps columns 0 and 1
    n, k = 256, 512
    q = np.where(rng(1).random((n, k // 2)) < 0.5, 0x6A, 0xA6).astype(np.uint8)
    s = rng(2).uniform(0.5, 1.5, n).astype(np.float32)
    x = rng(3).normal(0, 1, k).astype(np.float32)
    y = plane.sparse_matvec_mul_2_4_tensor(x, "w4zp8", q, s, n)
    ref = oracle.sparse_matvec_2_4("w4zp8", x, q, s, n)
    assert normwise_err(y, ref) <= TOL
    # a NaN weight is kept (it never moves in the sort) and poisons its row only
    w = rng(4).normal(0, 1, (8, 64)).astype(np.float32)
    w[3, 8] = np.nan
    x = rng(5).normal(0, 1, 64).astype(np.float32)
    y = plane.sparse_matvec_mul_2_4(x, w, 64)
    ref = oracle.sparse_matvec_2_4("f32", x, w, None, 8)
    assert np.isnan(y[3]) and np.isnan(ref[3])
    ok = np.arange(8) != 3
    assert normwise_err(y[ok], ref[ok]) <= TOL


def test_compressed_from_converter_vs_oracle(plane):
    n, k = 896, 4864
    w = rng(8).normal(0, 0.05, n * k).astype(np.float32)
    masks, values = oracle.compress_2_4(w)
    x = rng(9).normal(0, 1, k).astype(np.float32)
    sw = plane.register_sparse24_compressed("spc:down", n, k, masks, values)
    y = plane.gemv(sw, x)
    assert normwise_err(y, oracle.sparse_matvec_2_4_compressed(x, masks, values, n, k)) <= TOL
    # the same weight pruned on the device from the dense f32 matrix
    pw = plane.register_sparse24("spc:down:dense", "f32", n, k, w)
    assert normwise_err(plane.gemv(pw, x), y) <= TOL
    plane.evict(sw.key)
    plane.evict(pw.key)


def test_compressed_irregular_masks(plane):
    """Masks with fewer than two bits, bits above the low four, values that run
    out (sparse.rs:116-122) and columns past the last whole group."""
    n, k = 50, 130  # 32 groups + 2 ignored columns
    r = rng(10)
    pick2 = np.array([3, 5, 6, 9, 10, 12], np.uint16)
    masks = pick2[r.integers(0, 6, n * 32)]
    masks[::7] = 0
    masks[1::7] = np.array([1, 2, 4, 8], np.uint16)[r.integers(0, 4, masks[1::7].size)]
    masks[2::5] |= np.uint16(0xABC0)
    values = r.normal(0, 1, n * 32 * 2 - 150).astype(np.float32)
    x = r.normal(0, 1, k).astype(np.float32)
    y = plane.sparse_matvec_2_4_compressed(x, masks, values, n, k)
    ref = oracle.sparse_matvec_2_4_compressed(x, masks, values, n, k)
    assert normwise_err(y, ref) <= TOL and np.all(y[-2:] == 0)
    from bramha_b200 import BramhaError
    bad = masks.copy()
    bad[5] = 0b0111  # three of four: not 2:4
    with pytest.raises(BramhaError, match="more than two of four"):
        plane.sparse_matvec_2_4_compressed(x, bad, values, n, k)
    with pytest.raises(BramhaError):
        plane.sparse_matvec_2_4_compressed(x, masks[:10], values, n, k)


def test_keyed_calls_batch_and_multi(plane):
    n, k = 384, 768
    q, s = weights("w8", n, k, seed=11)
    x = rng(12).normal(0, 1, (3, k)).astype(np.float32)
    y0 = plane.sparse_matvec_mul_2_4_tensor(x[0], "w8", q, s, n, "m", "l0")
    assert plane.lookup("m:l0").fmt == "sp24_w8"  # cached under model:layer
    assert np.array_equal(y0, plane.sparse_matvec_mul_2_4_tensor(x[0], "w8", q, s, n, "m", "l0"))
    w = plane.lookup("m:l0")
    yb = plane.gemv(w, x)  # batch of three rows
    for b in range(3):
        assert normwise_err(yb[b], oracle.sparse_matvec_2_4("w8", x[b], q, s, n)) <= TOL
    assert np.array_equal(yb[0], y0)
    # two sparse weights sharing x in one multi call, device pointers
    q2, s2 = weights("w8", 200, k, seed=13)
    w2 = plane.register_sparse24("m:l1", "w8", 200, k, q2, s2)
    dev = torch.device("cuda", 0)
    xd = torch.from_numpy(x[1]).to(dev)
    ya, yb2 = torch.empty(n, device=dev), torch.empty(200, device=dev)
    plane.gemv_multi_dev([w, w2], xd, [ya, yb2])
    plane.stream_sync()
    assert np.array_equal(ya.cpu().numpy(), yb[1])
    assert normwise_err(yb2.cpu().numpy(), oracle.sparse_matvec_2_4("w8", x[1], q2, s2, 200)) <= TOL
    # device-side registration prunes the same way
    w3 = plane.register_sparse24_dev("m:l1:dev", "w8", 200, k, torch.from_numpy(q2.view(np.uint8)).to(dev),
                                     torch.from_numpy(s2).to(dev))
    assert np.array_equal(plane.gemv(w3, x[1]), yb2.cpu().numpy())
    for key in ("m:l0", "m:l1", "m:l1:dev"):
        plane.evict(key)


def test_argument_errors(plane):
    from bramha_b200 import BramhaError
    q, s = weights("w4zp8", 4, 8, seed=1)
    with pytest.raises(BramhaError, match="even in_features"):
        plane.register_sparse24("e:odd", "w4zp8", 4, 7, q[:12], s)
    with pytest.raises(BramhaError):
        plane.register_sparse24("e:log4", "log4", 4, 8, q, s)
    with pytest.raises(BramhaError, match="size mismatch"):
        plane.register_sparse24("e:size", "w4zp8", 4, 8, q[:15], s)
    w = plane.register_sparse24("e:ok", "w4zp8", 4, 8, q, s)
    with pytest.raises(BramhaError, match="different shape or format"):
        plane.register("e:ok", "w4zp8", 4, 8, q, s)
    plane.evict(w.key)
    assert plane.sparse_matvec_mul_2_4_tensor(np.zeros(0, np.float32), "w8", np.zeros(0, np.int8),
                                              np.ones(5, np.float32), 5).tolist() == [0.0] * 5
