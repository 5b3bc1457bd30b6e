"""The oracle's 2:4 restatements (spanda-engine/src/sparse.rs:19-138,
cpu_engine.rs:1532-1640, bin/convert.rs:55-92) pinned to the reference's own
known-answer tests (sparse.rs:141-200) and checked against an independent numpy
formulation of the selection (stable argsort on descending magnitude)."""
import numpy as np
import pytest

import oracle
from tests._util import make_weight, rng

# sparse.rs:145-160 / 178-200: one 2 x 8 matrix, x = ones.
KAT_W = np.array([0.1, 10.0, -5.0, 0.2, 1.0, -0.1, 0.5, 2.0,
                  0.0, 0.0, 1.0, 2.0, -5.0, -6.0, 1.0, 0.1], np.float32)
KAT_MASKS = np.array([6, 9, 12, 3], np.uint16)
KAT_VALUES = np.array([10.0, -5.0, 1.0, 2.0, 1.0, 2.0, -5.0, -6.0], np.float32)


def test_reference_known_answers():
    x = np.ones(8, np.float32)
    assert oracle.sparse_matvec_2_4("f32", x, KAT_W, None, 2).tolist() == [8.0, -8.0]
    assert oracle.sparse_matvec_2_4_compressed(x, KAT_MASKS, KAT_VALUES, 2, 8).tolist() == [8.0, -8.0]
    masks, values = oracle.compress_2_4(KAT_W)  # the compression the KAT spells out by hand
    assert masks.tolist() == KAT_MASKS.tolist() and values.tolist() == KAT_VALUES.tolist()


def _codes(fmt, q, n, k):
    if fmt == "f32":
        return q.reshape(n, k).astype(np.float64)
    if fmt == "w8":
        return q.view(np.int8).reshape(n, k).astype(np.float64)
    b = q.reshape(n, k // 2)
    out = np.empty((n, k), np.float64)
    out[:, 0::2] = (b >> 4) - 8.0
    out[:, 1::2] = (b & 0xF) - 8.0
    return out


def numpy_sparse(fmt, x, q, s, n, k):
    w = _codes(fmt, q, n, k)
    g = k // 4
    blocks = w[:, :4 * g].reshape(n, g, 4)
    order = np.argsort(-np.abs(blocks), axis=2, kind="stable")[:, :, :2]
    keep = np.zeros_like(blocks, dtype=bool)
    np.put_along_axis(keep, order, True, axis=2)
    y = (np.where(keep, blocks, 0.0).reshape(n, 4 * g) @ x[:4 * g].astype(np.float64)
         + w[:, 4 * g:] @ x[4 * g:].astype(np.float64))
    return y if fmt == "f32" else y * s


@pytest.mark.parametrize("fmt,n,k", [("f32", 96, 1001), ("w8", 70, 515), ("w4zp8", 64, 898), ("w4zp8", 33, 4)])
def test_selection_matches_stable_argsort(fmt, n, k):
    if fmt == "f32":
        q, s = rng(2).normal(0, 1, n * k).astype(np.float32), None
    else:
        _, q, s = make_weight(fmt, n, k, seed=3)
    x = rng(4).normal(0, 1, k).astype(np.float32)
    y = oracle.sparse_matvec_2_4(fmt, x, q, s, n)
    ref = numpy_sparse(fmt, x, q, s, n, k)
    assert np.max(np.abs(y - ref)) <= 1e-5 * np.max(np.abs(ref))
    assert np.array_equal(y, oracle.sparse_matvec_2_4(fmt, x, q, s, n, threads=4))


def test_ties_keep_lower_columns_and_nan_does_not_move():
    # magnitudes [3, 3, 3, 1]: columns 0 and 1; [1, 2, 2, 2]: 1 and 2
    w = np.array([3, -3, 3, 1, 1, 2, -2, 2], np.float32)
    masks, values = oracle.compress_2_4(w)
    assert masks.tolist() == [0b0011, 0b0110] and values.tolist() == [3, -3, 2, -2]
    # a NaN at column 0 is never passed: [NaN, 1, 2, 3] keeps 0 and 3
    masks, _ = oracle.compress_2_4(np.array([np.nan, 1, 2, 3], np.float32))
    assert masks.tolist() == [0b1001]


def test_compressed_equals_on_the_fly_and_guards():
    n, k = 40, 256
    w = rng(5).normal(0, 1, n * k).astype(np.float32)
    x = rng(6).normal(0, 1, k).astype(np.float32)
    masks, values = oracle.compress_2_4(w)
    a = oracle.sparse_matvec_2_4_compressed(x, masks, values, n, k)
    b = oracle.sparse_matvec_2_4("f32", x, w, None, n)
    assert np.max(np.abs(a - b)) <= 1e-5 * np.max(np.abs(b))
    # values running out: the reference's `val_idx < len` guard drops the rest
    # (row 0 needs values 0..127, row 1 128..255: with 200, row 1 stops early)
    short = oracle.sparse_matvec_2_4_compressed(x, masks, values[:200], n, k)
    assert short[0] == a[0] and np.array_equal(short[2:], np.zeros(n - 2, np.float32))
    cols = np.flatnonzero(np.unpackbits(masks[64:128].view(np.uint8), bitorder="little").reshape(64, 16)[:, :4])
    assert np.isclose(short[1], float(values[128:200] @ x[cols[:72]]), rtol=1e-5)
    # mask bits above the low four are ignored
    hi = oracle.sparse_matvec_2_4_compressed(x, masks | np.uint16(0xFFF0), values, n, k)
    assert np.array_equal(hi, a)
