"""The reference's own known answers for cuts, binning and histogram sum order
(src/data/quantile.rs tests `few_distinct_values_one_bin_each`,
`monotone_binning`, `constant_feature_has_one_bin`,
`split_threshold_consistency`; src/tree/hist/mod.rs tests
`histograms_do_not_depend_on_the_thread_count`,
`blocked_build_matches_the_block_order_reference`), checked against the CPU
oracle and, for cuts and bins, against the library's host binning
(hb_cuts_dense / hb_bin_dense), which the device sketch equals bit for bit
(tests/test_sketch_gpu.py)."""

import numpy as np
import pytest

import hessboost_b200 as H
import oracle_lib as O

CUTTERS = {"oracle": O.cuts_dense, "host": H.cuts_dense}


def _bin_of(off, cuts, f, v):
    """bin = #{cuts <= v}, clamped to the last bin (quantile.rs:285)."""
    c = cuts[off[f] : off[f + 1]]
    return min(int(np.searchsorted(c, np.float32(v), side="right")), len(c) - 1)


@pytest.mark.parametrize("who", sorted(CUTTERS))
def test_few_distinct_values_one_bin_each(who):
    # three distinct values 0, 1, 2: cuts [1, 2, sentinel]; the minimum is
    # never a cut, so each value has its own bin
    x = np.array([[0.0], [1.0], [2.0], [1.0]], np.float32)
    off, cuts = CUTTERS[who](x, 256)
    assert off[1] - off[0] == 3
    np.testing.assert_array_equal(cuts[:2], np.array([1.0, 2.0], np.float32))
    assert cuts[2] == np.float32(2.0) + (np.float32(2.0) + np.float32(1e-5))  # the sentinel
    assert [_bin_of(off, cuts, 0, v) for v in (0.0, 1.0, 2.0)] == [0, 1, 2]
    cols, _, dense = H.bin_dense(x, off, cuts)
    assert dense
    np.testing.assert_array_equal(cols[0], [0, 1, 2, 1])


@pytest.mark.parametrize("who", sorted(CUTTERS))
def test_monotone_binning(who):
    x = np.arange(1000, dtype=np.float32).reshape(-1, 1)
    off, cuts = CUTTERS[who](x, 16)
    assert off[1] - off[0] <= 16  # at most max_bin - 1 cuts plus the sentinel
    cols, _, _ = H.bin_dense(x, off, cuts)
    assert np.all(np.diff(cols[0].astype(np.int32)) >= 0)
    assert cols[0][0] < cols[0][999]


@pytest.mark.parametrize("who", sorted(CUTTERS))
def test_constant_feature_has_one_bin(who):
    x = np.full((3, 1), 5.0, np.float32)
    off, cuts = CUTTERS[who](x, 256)
    assert off[1] - off[0] == 1  # only the sentinel
    assert _bin_of(off, cuts, 0, 5.0) == 0


@pytest.mark.parametrize("who", sorted(CUTTERS))
def test_split_threshold_consistency(who):
    # value < cut_value(b) exactly when bin_of(value) <= b: the rule that
    # lets a split on bins carry a float threshold
    x = np.arange(10, dtype=np.float32).reshape(-1, 1)
    off, cuts = CUTTERS[who](x, 256)
    cols, _, _ = H.bin_dense(x, off, cuts)
    for b in range(int(off[1] - off[0]) - 1):
        thr = cuts[off[0] + b]
        np.testing.assert_array_equal(x[:, 0] < thr, cols[0].astype(np.int64) <= b)


# ---- histogram sum order (src/tree/hist/mod.rs tests) -----------------------
ROWS_PER_TASK = 4096


def test_histogram_block_order_2_54_case():
    # `histograms_do_not_depend_on_the_thread_count`: 8,192 rows in one bin,
    # g = 2^54 at row 0, -2^54 at row 4096, 1 at row 4097. The row-order
    # chain would give 1; the two 4,096-row blocks give 2^54 and
    # -2^54 + 1 = -2^54 (rounded), so 0.
    n = 2 * ROWS_PER_TASK
    # the reference builds this on a sparse index: an all-missing second
    # feature makes this index sparse too, which selects the blocked order
    x = np.ones((n, 2), np.float32)
    x[:, 1] = np.nan
    off, cuts = O.cuts_dense(x, 256)
    assert off[1] - off[0] == 1
    gp = np.zeros((n, 2), np.float32)
    gp[:, 1] = 1.0
    gp[0, 0] = 2.0**54
    gp[4096, 0] = -(2.0**54)
    gp[4097, 0] = 1.0
    h = O.hist(x, off, cuts, np.arange(n, dtype=np.uint32), gp)
    assert (h[0, 0], h[0, 1]) == (0.0, float(n))
    assert np.all(h[1:] == 0.0)


def test_histogram_blocked_build_matches_block_order_reference():
    # `blocked_build_matches_the_block_order_reference`: f64 sums formed per
    # block of `grain` rows (in row order), the blocks then added in order;
    # the gradients span enough exponents that this differs from one chain
    n = 6 * ROWS_PER_TASK + 123
    i = np.arange(n)
    x = np.stack([(i % 7).astype(np.float32), np.full(n, np.nan, np.float32)], 1)  # sparse, as above
    off, cuts = O.cuts_dense(x, 256)
    scale = np.array([np.float32(2.0) ** (int(k) - 30) for k in (i * 37 % 61)], np.float32)
    g = (((i * 7919) % 1237).astype(np.float32) / np.float32(331.0) * scale - np.float32(1.0)).astype(np.float32)
    gp = np.stack([g, scale], 1).astype(np.float32)
    rows = np.array([r for r in range(n) if r % 11 != 3], np.uint32)
    blocks = len(rows) // ROWS_PER_TASK
    grain = -(-len(rows) // blocks)
    nb = int(off[-1])
    bins = [_bin_of(off, cuts, 0, v) for v in range(7)]
    expect = np.zeros((nb, 2))
    for b0 in range(0, len(rows), grain):
        part = np.zeros((nb, 2))
        for r in rows[b0 : b0 + grain]:
            k = bins[int(x[r, 0])]
            part[k, 0] += float(gp[r, 0])
            part[k, 1] += float(gp[r, 1])
        expect += part
    chain = np.zeros((nb, 2))
    for r in rows:
        k = bins[int(x[r, 0])]
        chain[k, 0] += float(gp[r, 0])
        chain[k, 1] += float(gp[r, 1])
    assert not np.array_equal(expect, chain), "the case must separate the groupings"
    np.testing.assert_array_equal(O.hist(x, off, cuts, rows, gp), expect)
