"""The device quantile sketch and binning (hb_sketch_dense / hb_sketch_csr /
hb_engine_upload_dense / hb_engine_upload_csr) against the CPU oracle's
restatement of the reference's WQSketch (src/data/sketch.rs, pinned to the
reference's saved-model fixtures) and against the host binning.

Cut values must agree bit for bit, bins and missing bitmaps byte for byte,
and a model trained from the device-built index must equal the one trained
from the host-built index. The inputs cover what makes the sketch's
streaming order matter: many queue flushes and ladder levels, long runs of
equal values (folded queue entries), -0/+0, infinities, empty and constant
features, and an entry count that is an exact multiple of the queue."""

import math

import numpy as np
import pytest

import hessboost_b200 as H
import oracle_lib as O
from hessboost_b200 import synth

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _limit(max_bin, n):
    """sketch.rs:65/83 summary_budget, for choosing edge-case sizes."""
    if n == 0:
        return 1
    eps = 1.0 / min(max_bin, max(n, 1))
    internal = eps / 2.0
    lv = 1
    while True:
        lim = min(math.ceil(lv / internal) + 1, n)
        if (1 << lv) * lim >= n:
            return lim
        lv += 1


def _check_dense(x, max_bin):
    off, cuts, cols, miss, dense = H.sketch_dense(x, max_bin, device=0)
    ooff, ocuts = O.cuts_dense(x, max_bin)
    np.testing.assert_array_equal(off, ooff)
    np.testing.assert_array_equal(_bits(cuts), _bits(ocuts))
    hoff, hcuts = H.cuts_dense(x, max_bin)
    np.testing.assert_array_equal(_bits(cuts), _bits(hcuts))
    hcols, hmiss, hdense = H.bin_dense(x, off, cuts)
    np.testing.assert_array_equal(cols, hcols)
    assert dense == hdense
    if not dense:
        np.testing.assert_array_equal(miss, np.asarray(hmiss).reshape(miss.shape))
    return off, cuts


def test_sketch_c2_shape_many_flushes():
    # 600,003 rows: ~70 queue flushes per feature, a ladder 7 levels deep
    x, _ = synth.logistic_c2(600_003, 28, seed=3)
    _check_dense(x, 256)


@pytest.mark.parametrize("max_bin", [2, 16, 64, 255, 256])
def test_sketch_max_bins(max_bin):
    rng = np.random.default_rng(max_bin)
    x = rng.standard_normal((50_000, 5)).astype(np.float32)
    x[rng.random(x.shape) < 0.1] = np.nan
    _check_dense(x, max_bin)


def test_sketch_repeats_and_runs():
    rng = np.random.default_rng(7)
    n = 120_000
    x = np.empty((n, 6), np.float32)
    x[:, 0] = rng.integers(0, 50, n)                           # few distinct values
    x[:, 1] = np.repeat(np.arange(n // 400), 400)[:n]          # long runs: folded queue entries
    x[:, 2] = np.sort(rng.standard_normal(n))                  # ascending stream
    x[:, 3] = 3.5                                              # constant
    x[:, 4] = np.nan                                           # never present
    x[:, 5] = rng.choice(np.array([-0.0, 0.0, 1.0, -1.0, np.inf, -np.inf], np.float32), n)
    x[rng.random(n) < 0.05, 2] = np.nan
    _check_dense(x, 256)
    _check_dense(x, 16)


def test_sketch_many_features():
    # 70 features (three feature groups of the index), mixed missing rates
    rng = np.random.default_rng(21)
    x = rng.standard_normal((40_000, 70)).astype(np.float32)
    x[:, ::3] = np.round(x[:, ::3] * 4)            # repeated values
    x[rng.random(x.shape) < np.linspace(0.0, 0.5, 70)] = np.nan
    _check_dense(x, 256)


def test_sketch_tiny_and_ragged():
    rng = np.random.default_rng(11)
    for n in (1, 2, 3, 7, 64, 65, 257):
        x = rng.standard_normal((n, 3)).astype(np.float32)
        if n > 2:
            x[::3, 1] = np.nan
        _check_dense(x, 256)
        _check_dense(x, 4)


def test_sketch_exact_multiple_of_the_queue():
    # distinct values only, so entries = present values; pick n with
    # n % (2 * limit(n)) == 0: the last flush happens in summary()
    max_bin = 16
    n = next(k for k in range(400, 20_000) if k % (2 * _limit(max_bin, k)) == 0)
    rng = np.random.default_rng(5)
    x = rng.permutation(np.arange(n, dtype=np.float32)).reshape(n, 1)
    _check_dense(x, max_bin)


def test_sketch_refuses_2_24_present_values():
    n = 1 << 24
    x = np.zeros((n, 1), np.float32)
    x[:, 0] = np.arange(n, dtype=np.float32) % 1000
    with pytest.raises(H.HbError) as e:
        H.sketch_dense(x, 256, device=0, bins=False)
    assert e.value.status == H.HB_REFUSED


def _check_csr(indptr, indices, values, n_cols, max_bin):
    off, cuts, rb, dense = H.sketch_csr(indptr, indices, values, n_cols, max_bin, device=0)
    ooff, ocuts = O.cuts_csr(indptr, indices, values, n_cols, max_bin)
    np.testing.assert_array_equal(off, ooff)
    np.testing.assert_array_equal(_bits(cuts), _bits(ocuts))
    hptr, hbins, hdense = H.bin_csr(indptr, indices, values, n_cols, off, cuts)
    np.testing.assert_array_equal(rb, hbins)
    assert dense == hdense


def test_sketch_csr_c4_like():
    indptr, indices, values, _ = synth.sparse_c4(60_000, 400, density=0.05, seed=2)
    _check_csr(indptr, indices, values, 400, 64)


def test_sketch_csr_full_rows_and_empty_features():
    rng = np.random.default_rng(9)
    n, f = 5_000, 8
    x = rng.standard_normal((n, f)).astype(np.float32)
    indptr = np.arange(0, n * f + 1, f, dtype=np.uint64)
    indices = np.tile(np.arange(f, dtype=np.uint32), n)
    _check_csr(indptr, indices, x.reshape(-1), f, 256)
    # features 3 and 7 never stored
    keep = (indices != 3) & (indices != 7)
    counts = keep.reshape(n, f).sum(1)
    ip2 = np.concatenate([[0], np.cumsum(counts)]).astype(np.uint64)
    _check_csr(ip2, indices[keep], x.reshape(-1)[keep], f, 256)


def test_sketch_csr_rejects():
    indptr = np.array([0, 2, 3], np.uint64)
    with pytest.raises(H.HbError) as e:  # columns out of order in row 0
        H.sketch_csr(indptr, np.array([1, 0, 0], np.uint32), np.ones(3, np.float32), 2, 16, device=0)
    assert e.value.status == H.HB_REFUSED
    with pytest.raises(H.HbError) as e:  # column beyond n_cols
        H.sketch_csr(indptr, np.array([0, 5, 0], np.uint32), np.ones(3, np.float32), 2, 16, device=0)
    assert e.value.status == H.HB_INVALID_ARGUMENT
    with pytest.raises(H.HbError) as e:  # a stored NaN
        H.sketch_csr(indptr, np.array([0, 1, 0], np.uint32), np.array([1, np.nan, 2], np.float32), 2, 16,
                     device=0)
    assert e.value.status == H.HB_INVALID_ARGUMENT


def _assert_same(a_nodes, a_ptr, b_nodes, b_ptr):
    np.testing.assert_array_equal(np.asarray(a_ptr, np.uint64), np.asarray(b_ptr, np.uint64))
    for k in ("left", "right", "split_feature", "default_left", "split_bin"):
        np.testing.assert_array_equal(a_nodes[k], b_nodes[k], err_msg=k)
    for k in ("split_cond", "leaf_value", "sum_hess", "split_gain"):
        np.testing.assert_array_equal(_bits(a_nodes[k]), _bits(b_nodes[k]), err_msg=k)


def test_engine_upload_dense_trains_like_host_index():
    x, y = synth.logistic_c2(200_000, 28, seed=4)
    params = H.TrainingParams(objective="binary:logistic", max_depth=6, eta=0.1)
    host = H.train(params, y=y, rounds=3, device=0, matrix=H.BinnedMatrix.from_dense(x, 256))
    eng = H.Engine(0)
    try:
        idx = eng.upload_dense(x, 256)
        np.testing.assert_array_equal(_bits(idx.cut_values), _bits(H.cuts_dense(x, 256)[1]))
        nodes, ptr = eng.train(params, y, 3, H.base_margin(params, y))
    finally:
        eng.close()
    _assert_same(nodes, ptr, host.nodes, host.tree_ptr)


def test_engine_upload_dense_many_features_trains_like_host_index():
    rng = np.random.default_rng(8)
    x = rng.standard_normal((60_000, 70)).astype(np.float32)
    x[rng.random(x.shape) < 0.05] = np.nan
    y = (np.nan_to_num(x[:, :5]).sum(1) + 0.1 * rng.standard_normal(60_000)).astype(np.float32)
    params = H.TrainingParams(objective="reg:squarederror", max_depth=5, eta=0.3)
    host = H.train(params, y=y, rounds=3, device=0, matrix=H.BinnedMatrix.from_dense(x, 256))
    dev = H.train(params, x, y, rounds=3, device=0)  # sketches and bins on the device
    _assert_same(dev.nodes, dev.tree_ptr, host.nodes, host.tree_ptr)


def test_engine_upload_csr_trains_like_host_index():
    indptr, indices, values, y = synth.sparse_c4(30_000, 200, density=0.05, seed=6)
    params = H.TrainingParams(objective="binary:logistic", grow_policy="lossguide", max_depth=0, max_leaves=31,
                              max_bin=64)
    m = H.BinnedMatrix.from_csr(indptr, indices, values, 200, 64)
    host = H.train(params, y=y, rounds=2, device=0, matrix=m)
    eng = H.Engine(0)
    try:
        eng.upload_csr(indptr, indices, values, 200, 64)
        nodes, ptr = eng.train(params, y, 2, H.base_margin(params, y))
    finally:
        eng.close()
    _assert_same(nodes, ptr, host.nodes, host.tree_ptr)


def test_engine_reupload_smaller_matrix_matches_fresh_engine():
    # an engine keeps no row count from an earlier index: the fixed-point
    # scale of the second index is its own
    x, y = synth.logistic_c2(120_000, 28, seed=22)
    params = H.TrainingParams(objective="binary:logistic", max_depth=5, eta=0.1)
    fresh = H.train(params, x[:50_000], y[:50_000], rounds=2, device=0)
    eng = H.Engine(0)
    try:
        eng.upload_dense(x, 256)
        eng.upload_dense(x[:50_000], 256)
        nodes, ptr = eng.train(params, y[:50_000], 2, H.base_margin(params, y[:50_000]))
    finally:
        eng.close()
    _assert_same(nodes, ptr, fresh.nodes, fresh.tree_ptr)


def test_engine_upload_dense_refused_on_a_shard():
    x, _ = synth.logistic_c2(10_000, 8, seed=23)
    eng = H.Engine(0)
    try:
        eng.set_shard(0, 20_000)  # these rows are half of a larger matrix
        with pytest.raises(H.HbError) as e:
            eng.upload_dense(x, 256)
        assert e.value.status == H.HB_REFUSED
    finally:
        eng.close()
