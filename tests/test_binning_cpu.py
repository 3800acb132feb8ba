"""The reference's own known answers for cuts and binning
(src/data/quantile.rs tests `few_distinct_values_one_bin_each`,
`monotone_binning`, `constant_feature_has_one_bin`,
`split_threshold_consistency`), checked against the CPU oracle and against
the library's host binning (hb_cuts_dense / hb_bin_dense), which the device
sketch equals bit for bit (tests/test_sketch_gpu.py)."""

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
