"""Failure detection on the GPU without faulting it.

Every mbarrier wait of the tensor-core GEMV and GEMM is bounded (a %globaltimer
deadline that the context sets); a kernel whose wait runs out records
BRAMHA_ERR_TIMEOUT in the context's error word, drains the copies and MMAs it
issued, frees its TMEM and returns.  Here a test-only switch makes CTA 0 of
the next launches withhold one weight copy -- a barrier that nothing
completes -- with a 5 ms bound, and the tests check that

* the host-buffer calls (bramha_cuda_gemv, _matvec, _gemm) return
  BRAMHA_ERR_TIMEOUT (the reference's per-call `Err(String)`,
  src/compute/wgpu_backend.rs:1096-1104),
* the device-pointer calls followed by bramha_cuda_stream_sync do too,
* the next normal call on the same context succeeds and matches the oracle.

No GPU fault, trap or hang is caused: the withheld copy is simply never
issued, and every wait that depends on it gives up after 5 ms.
"""
import numpy as np
import pytest

import oracle
from tests._util import GEMM_BF16_TOL, GEMV_TOL, make_weight, make_x, normwise_err, oracle_gemv

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TIMEOUT = -7  # BRAMHA_ERR_TIMEOUT


@pytest.fixture(scope="module")
def plane():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from bramha_b200 import CudaComputePlane
    p = CudaComputePlane(0)
    p.set_wait_timeout(5_000_000)  # 5 ms
    yield p
    p.test_fault("none")
    p.set_wait_timeout(0)
    p.close()


def expect_timeout(fn):
    from bramha_b200 import BramhaError
    with pytest.raises(BramhaError) as ei:
        fn()
    assert ei.value.code == TIMEOUT, str(ei.value)
    assert "bounded wait" in ei.value.message


@pytest.mark.parametrize("fmt", ["log4", "w4zp8", "w8"])
def test_gemv_wait_runs_out_and_context_recovers(plane, fmt):
    n, k = 8192, 8192  # every CTA streams more slot pairs than its prologue requests
    _, q, s = make_weight(fmt, n, k, seed=3)
    w = plane.register(f"fault:gemv:{fmt}", fmt, n, k, q, s)
    x = make_x(1, k, seed=4)
    plane.set_gemv_kernel("tensor_core")
    plane.test_fault("gemv")
    try:
        expect_timeout(lambda: plane.gemv(w, x))                     # host buffers
        expect_timeout(lambda: plane.matvec_mul_log4(x[0], q, s, n) if fmt == "log4" else
                       plane.matvec_mul_int8(x[0], q, s, n) if fmt == "w8" else
                       plane.matvec_mul_int4(x[0], q, s, n))         # the reference-shaped call
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty((1, n), device="cuda")
        plane.gemv_dev(w, xd, yd)                                    # stream-ordered: no error yet
        expect_timeout(plane.stream_sync)
    finally:
        plane.test_fault("none")
        plane.set_gemv_kernel("auto")
    y = plane.gemv(w, x)  # the same context works again
    assert normwise_err(y, oracle_gemv(fmt, x, q, s, n)) <= GEMV_TOL
    plane.evict(w.key)


@pytest.mark.parametrize("n,m", [(640, 300), (38400, 512)], ids=["single_cta", "sm_pair"])
def test_gemm_wait_runs_out_and_context_recovers(plane, n, m):
    fmt, k = "log4", 256
    _, q, s = make_weight(fmt, n, k, seed=5)
    w = plane.register(f"fault:gemm:{n}", fmt, n, k, q, s)
    hb = make_x(m, k, seed=6)
    xb = torch.from_numpy(hb).cuda().to(torch.bfloat16)
    plane.test_fault("gemm")
    try:
        expect_timeout(lambda: plane.gemm(w, hb, m))                 # host buffers
        y = torch.empty((m, n), device="cuda")
        plane.gemm_dev(w, xb, y)
        expect_timeout(plane.stream_sync)
    finally:
        plane.test_fault("none")
    out = plane.gemm(w, hb, m)
    assert normwise_err(out, oracle.gemm_cpu(fmt, hb, q, s, m, k, n)) <= GEMV_TOL
    y = torch.empty((m, n), device="cuda")
    plane.gemm_dev(w, xb, y)
    plane.stream_sync()
    ref = oracle.gemm_cpu(fmt, xb.float().cpu().numpy(), q, s, m, k, n)
    assert normwise_err(y.cpu().numpy().reshape(-1), ref) <= GEMM_BF16_TOL
    plane.evict(w.key)


def test_timeout_setting_and_fault_kinds_validated(plane):
    from bramha_b200 import BramhaError, lib
    assert lib().bramha_cuda_test_fault(plane.ctx, 7) == -1
    assert lib().bramha_cuda_set_prefetch(plane.ctx, -1, 0) == -1
    with pytest.raises(KeyError):
        plane.test_fault("bogus")
    with pytest.raises(BramhaError):
        from bramha_b200._lib import check
        check(lib().bramha_cuda_test_fault(plane.ctx, 9))
