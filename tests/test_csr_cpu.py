"""The CSR input path on the host (no GPU): DMatrix::from_csr's checks,
cuts from each feature's stored entries in row order, and the CSR index of
global bins.

The reference sketches a CSR feature by pushing its stored entries in row
order (src/data/quantile.rs:199) and a dense feature by pushing its
non-missing values in row order (push_unit_column, which src/data/
sketch.rs:541 documents as equal to repeated push), with the same present
count; so the cuts of a CSR matrix equal the oracle's cuts of the dense
matrix holding NaN in every absent cell, bit for bit. That is the pin."""

import numpy as np
import pytest

import hessboost_b200 as H
import oracle_lib as O
from hessboost_b200 import synth


def _random_csr(n, f, density, seed, shuffle=True, empty_rows=(), absent_cols=()):
    rng = np.random.default_rng(seed)
    mask = rng.random((n, f)) < density
    for r in empty_rows:
        mask[r] = False
    for c in absent_cols:
        mask[:, c] = False
    indptr = np.zeros(n + 1, np.uint64)
    indptr[1:] = np.cumsum(mask.sum(axis=1))
    rows, cols = np.nonzero(mask)
    values = (rng.standard_normal(rows.size) * 3).round(1).astype(np.float32)  # repeats
    indices = cols.astype(np.uint32)
    if shuffle:  # column order within a row is free in from_csr
        for r in range(n):
            a, b = int(indptr[r]), int(indptr[r + 1])
            p = rng.permutation(b - a) + a
            indices[a:b], values[a:b] = indices[p].copy(), values[p].copy()
    return indptr, indices, values


CASES = [
    ("sparse", dict(n=3000, f=40, density=0.05, seed=1), 256),
    ("few_bins", dict(n=2000, f=9, density=0.3, seed=2), 16),
    ("gaps", dict(n=1500, f=12, density=0.2, seed=3, empty_rows=(0, 7, 1499), absent_cols=(4, 11)), 64),
    ("full", dict(n=500, f=5, density=1.1, seed=4), 256),
]


@pytest.mark.parametrize("name,kw,max_bin", CASES, ids=[c[0] for c in CASES])
def test_csr_cuts_and_bins_match_dense_oracle(name, kw, max_bin):
    indptr, indices, values = _random_csr(**kw)
    f = kw["f"]
    x = synth.csr_to_dense(indptr, indices, values, f)
    off, cuts = H.cuts_csr(indptr, indices, values, f, max_bin)
    off_o, cuts_o = O.cuts_dense(x, max_bin)
    np.testing.assert_array_equal(off, off_o)
    np.testing.assert_array_equal(cuts.view(np.uint32), cuts_o.view(np.uint32))
    m = H.BinnedMatrix.from_csr(indptr, indices, values, f, max_bin)
    assert m.is_csr and m.n_rows == kw["n"] and m.n_cols == f
    np.testing.assert_array_equal(m.row_ptr, indptr)
    bins_o, miss_o, dense_o = O.bin_dense(x, off_o, cuts_o)
    assert m.dense == dense_o
    for r in range(kw["n"]):
        got = m.row_bins[int(indptr[r]) : int(indptr[r + 1])]
        present = np.nonzero(~np.isnan(x[r]))[0]
        want = off_o[present] + bins_o[present, r]
        np.testing.assert_array_equal(got, want.astype(np.uint32))


def test_csr_shard_slices_rows():
    indptr, indices, values = _random_csr(1000, 8, 0.3, 5)
    m = H.BinnedMatrix.from_csr(indptr, indices, values, 8)
    a, b = m.shard(0, 400), m.shard(400, 1000)
    assert a.n_rows == 400 and b.n_rows == 600
    np.testing.assert_array_equal(np.concatenate([a.row_bins, b.row_bins]), m.row_bins)
    np.testing.assert_array_equal(b.row_ptr, m.row_ptr[400:] - m.row_ptr[400])


@pytest.mark.parametrize("bad", ["duplicate", "column", "nan", "inf", "indptr", "start"])
def test_from_csr_checks(bad):
    indptr = np.array([0, 2, 3, 5], np.uint64)
    indices = np.array([0, 2, 1, 0, 3], np.uint32)
    values = np.array([1, 2, 3, 4, 5], np.float32)
    if bad == "duplicate":
        indices[1] = 0
    elif bad == "column":
        indices[4] = 4
    elif bad == "nan":
        values[2] = np.nan
    elif bad == "inf":
        values[0] = np.inf
    elif bad == "indptr":
        indptr[2] = 1
    elif bad == "start":
        indptr = indptr + np.uint64(1)
    with pytest.raises(H.HbError) as ex:
        H.cuts_csr(indptr, indices, values, 4)
    assert ex.value.status == H.HB_INVALID_ARGUMENT


def test_synthetic_c4_shape():
    indptr, indices, values, y = synth.sparse_c4(20_000, 300, density=0.05, seed=3)
    nnz = np.diff(indptr.astype(np.int64))
    assert abs(nnz.mean() - 15) < 0.5
    for r in range(0, 20_000, 997):  # ascending, distinct columns
        c = indices[int(indptr[r]) : int(indptr[r + 1])]
        assert np.all(np.diff(c.astype(np.int64)) > 0) and (c.size == 0 or c[-1] < 300)
    assert np.all(values > 0) and set(np.unique(y)) <= {0.0, 1.0}


@pytest.mark.parametrize("name,kw,max_bin", CASES, ids=[c[0] for c in CASES])
def test_oracle_csr_cuts_match_dense(name, kw, max_bin):
    indptr, indices, values = _random_csr(**kw)
    x = synth.csr_to_dense(indptr, indices, values, kw["f"])
    off, cuts = O.cuts_csr(indptr, indices, values, kw["f"], max_bin)
    off_o, cuts_o = O.cuts_dense(x, max_bin)
    np.testing.assert_array_equal(off, off_o)
    np.testing.assert_array_equal(cuts.view(np.uint32), cuts_o.view(np.uint32))


@pytest.mark.parametrize("fixed", [True, False], ids=["fixed_point", "f64"])
@pytest.mark.parametrize("policy", [0, 1], ids=["depthwise", "lossguide"])
def test_oracle_csr_training_equals_dense(fixed, policy):
    """The oracle's CSR index (stored cells only) trains the trees of its
    dense index on the same cells: bit for bit in fixed point; in f64 the
    reference's row-order chains give the same sums too on this set."""
    indptr, indices, values = _random_csr(2500, 15, 0.3, 9)
    x = synth.csr_to_dense(indptr, indices, values, 15)
    rng = np.random.default_rng(2)
    y = (np.nan_to_num(x[:, 0]) + np.nan_to_num(x[:, 3]) * 0.5 + rng.standard_normal(2500) * 0.1).astype(np.float32)
    kw = dict(max_depth=5, grow_policy=policy, max_leaves=20 if policy else 0, fixed_point=fixed)
    a = O.train_csr(indptr, indices, values, 15, y, 3, **kw)
    b = O.train(x, y, 3, **kw)
    np.testing.assert_array_equal(a[1], b[1])
    for k in ("left", "right", "split_feature", "default_left", "split_bin"):
        np.testing.assert_array_equal(a[0][k], b[0][k], err_msg=k)
    if fixed:
        for k in ("leaf_value", "sum_hess", "split_gain", "split_cond"):
            np.testing.assert_array_equal(a[0][k].view(np.uint32), b[0][k].view(np.uint32), err_msg=k)
        np.testing.assert_array_equal(a[3].view(np.uint32), b[3].view(np.uint32))
    else:
        np.testing.assert_allclose(a[0]["leaf_value"], b[0]["leaf_value"], rtol=1e-5, atol=1e-7)
