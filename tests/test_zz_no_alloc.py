"""The allocation-free prefill GEMM entry point, bramha_cuda_gemm_noalloc_dev.

Callers that must not let the library allocate device memory during a call
(for example an engine that has reserved all of HBM for its own pools) use this
entry point; it works out of a fixed scratch array compiled into the library.
These tests call it through the C ABI and check its output against the
ordinary entry point, bramha_cuda_gemm_dev -- bit for bit, since both run the
same kernel on the same bf16 inputs, which is within the bf16-tile tolerance
the GEMM tests use -- on two calls in a row, the second with fewer tokens, so
stale scratch from the first call would show up.  One case takes the SM-pair
kernel, one case is checked against the CPU oracle, and the device's memory
pool is watched to show that the calls allocate nothing while gemm_dev does.
The file is named to be collected last, and it must pass alone in a fresh
process as well as after the others.
"""
import ctypes

import numpy as np
import pytest

import oracle
from tests._util import GEMM_BF16_TOL, make_weight, normwise_err, rng

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


def _bf16(m, k, seed):
    return torch.from_numpy(rng(seed).normal(0, 1, (m, k)).astype(np.float32)).to(torch.bfloat16).cuda()


def _noalloc(plane, w, x, y):
    from bramha_b200 import lib
    from bramha_b200.plane import _stream
    return lib().bramha_cuda_gemm_noalloc_dev(plane.ctx, w.handle, x.data_ptr(), x.shape[0], y.data_ptr(),
                                              _stream(None))


def plane_error():
    from bramha_b200 import last_error
    return last_error()


@pytest.mark.parametrize("fmt,n,k", [("log4", 640, 896), ("w8", 640, 896), ("w4zp8", 640, 896),
                                     ("log4", 38400, 896)],
                         ids=["log4", "w8", "w4zp8", "log4_sm_pair"])
def test_noalloc_matches_gemm_dev_on_two_calls(plane, fmt, n, k):
    _, q, s = make_weight(fmt, n, k, seed=31)
    w = plane.register(f"noalloc:{fmt}:{n}", fmt, n, k, q, s)
    # 38400 rows x 300 tokens is 300 pair tiles: the SM-pair kernel (use_pair needs 4 per SM pair)
    for m, seed in ((300, 1), (77, 2)):
        x = _bf16(m, k, seed)
        y_ref = torch.empty((m, n), dtype=torch.float32, device="cuda")
        plane.gemm_dev(w, x, y_ref)
        y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        rc = _noalloc(plane, w, x, y)
        assert rc == 0, plane_error()
        plane.stream_sync()
        assert normwise_err(y.cpu().numpy(), y_ref.cpu().numpy()) <= GEMM_BF16_TOL
        assert torch.equal(y, y_ref)  # same kernel, same inputs: identical
    plane.evict(w.key)


def test_noalloc_matches_oracle(plane):
    """gemm_cpu (src/inference/cpu_engine.rs:565-912) on the same bf16 activations."""
    fmt, n, k, m = "log4", 320, 896, 48
    _, q, s = make_weight(fmt, n, k, seed=41)
    w = plane.register("noalloc:oracle", fmt, n, k, q, s)
    x = _bf16(m, k, 42)
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    assert _noalloc(plane, w, x, y) == 0, plane_error()
    plane.stream_sync()
    ref = oracle.gemm_cpu(fmt, x.float().cpu().numpy(), q, s, m, k, n)
    assert normwise_err(y.cpu().numpy().reshape(-1), ref) <= GEMM_BF16_TOL
    plane.evict(w.key)


def test_noalloc_empty_k_gives_zeros(plane):
    n, m = 64, 5
    w = plane.register("noalloc:k0", "log4", n, 0, np.zeros(0, np.uint8), np.ones(n, np.float32))
    x = torch.zeros((m, 8), dtype=torch.bfloat16, device="cuda")
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    assert _noalloc(plane, w, x, y) == 0, plane_error()
    plane.stream_sync()
    assert torch.count_nonzero(y).item() == 0
    plane.evict(w.key)


class _DefaultPool:
    """The device's default memory pool (the one cudaMallocAsync draws from),
    read through the driver API."""
    RESERVED_CURRENT, RESERVED_HIGH, USED_CURRENT, USED_HIGH = 5, 6, 7, 8

    def __init__(self, ordinal=0):
        self.cu = ctypes.CDLL("libcuda.so.1")
        d = ctypes.c_int()
        assert self.cu.cuDeviceGet(ctypes.byref(d), ordinal) == 0
        self.pool = ctypes.c_void_p()
        assert self.cu.cuDeviceGetDefaultMemPool(ctypes.byref(self.pool), d) == 0

    def get(self, attr):
        v = ctypes.c_uint64()
        assert self.cu.cuMemPoolGetAttribute(self.pool, attr, ctypes.byref(v)) == 0
        return v.value

    def reset_high(self):
        z = ctypes.c_uint64(0)
        for attr in (self.RESERVED_HIGH, self.USED_HIGH):
            assert self.cu.cuMemPoolSetAttribute(self.pool, attr, ctypes.byref(z)) == 0


def test_noalloc_allocates_nothing_while_gemm_dev_does(plane):
    fmt, n, k, m = "log4", 640, 896, 300
    _, q, s = make_weight(fmt, n, k, seed=51)
    w = plane.register("noalloc:pool", fmt, n, k, q, s)
    x = _bf16(m, k, 52)
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    assert _noalloc(plane, w, x, y) == 0, plane_error()  # first call: looks up the array's address
    plane.stream_sync()
    pool = _DefaultPool(torch.cuda.current_device())
    used, reserved = pool.get(pool.USED_CURRENT), pool.get(pool.RESERVED_CURRENT)
    pool.reset_high()
    for _ in range(2):
        assert _noalloc(plane, w, x, y) == 0, plane_error()
    plane.stream_sync()
    assert pool.get(pool.USED_HIGH) <= used
    assert pool.get(pool.RESERVED_CURRENT) == reserved
    # the ordinary entry point takes its per-token sums from the same pool
    pool.reset_high()
    plane.gemm_dev(w, x, y)
    plane.stream_sync()
    assert pool.get(pool.USED_HIGH) > used
    plane.evict(w.key)


def test_noalloc_rejects_more_tokens_than_its_scratch(plane):
    from bramha_b200 import last_error
    n, k = 128, 64
    _, q, s = make_weight("log4", n, k, seed=3)
    w = plane.register("noalloc:big", "log4", n, k, q, s)
    m = 16385
    x = torch.zeros((m, k), dtype=torch.bfloat16, device="cuda")
    y = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    rc = _noalloc(plane, w, x, y)
    assert rc == -5  # BRAMHA_ERR_UNSUPPORTED, nothing launched
    assert "16384" in last_error()
    plane.evict(w.key)
