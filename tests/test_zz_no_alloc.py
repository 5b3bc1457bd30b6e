"""The allocation-free prefill GEMM entry point, bramha_cuda_gemm_noalloc_dev.

Callers that must not let the library allocate device memory during a call
(for example an engine that has reserved all of HBM for its own pools) use this
entry point; it works out of a fixed scratch array compiled into the library.
These tests call it through the C ABI and check its output against the
ordinary entry point, bramha_cuda_gemm_dev, within the bf16-tile tolerance the
GEMM tests use, on two calls in a row -- the second with fewer tokens, so stale
scratch from the first call would show up.  The file is named to be collected
last, and it must pass alone in a fresh process as well as after the others.
"""
import ctypes

import numpy as np
import pytest

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


@pytest.mark.parametrize("fmt", ["log4", "w8", "w4zp8"])
def test_noalloc_matches_gemm_dev_on_two_calls(plane, fmt):
    n, k = 640, 896
    _, q, s = make_weight(fmt, n, k, seed=31)
    w = plane.register(f"noalloc:{fmt}", fmt, n, k, q, s)
    for m, seed in ((300, 1), (77, 2)):
        x = _bf16(m, k, seed)
        y_ref = torch.empty((m, n), dtype=torch.float32, device="cuda")
        plane.gemm_dev(w, x, y_ref)
        y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        rc = _noalloc(plane, w, x, y)
        assert rc == 0, plane_error()
        plane.stream_sync()
        assert normwise_err(y.cpu().numpy(), y_ref.cpu().numpy()) <= GEMM_BF16_TOL
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


def plane_error():
    from bramha_b200 import last_error
    return last_error()
