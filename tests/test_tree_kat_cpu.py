"""The reference's tree-growth and gain known answers, on the CPU oracle
(src/tree/gain.rs tests `threshold_l1_shrinks_toward_zero`,
`weight_and_gain_closed_form`, `max_delta_step_clamps_weight`;
src/tree/builder/hist/mod.rs tests `splits_on_separating_feature`,
`no_split_below_gamma`, `lossguide_respects_max_leaves`,
`fully_present_feature_never_splits_missing_left` without its monotone
constraint, which this path does not carry).

The reference's tests grow one tree from given gradient pairs. Here the
pairs come from squared error at base score 0 and unit weights, so
g = -y and h = 1, and eta 1 leaves each leaf at its raw weight."""

import numpy as np
import pytest

import oracle_lib as O

RAW = dict(base_score=0.0, eta=1.0)


def _grow(x, g, **kw):
    x = np.asarray(x, np.float32).reshape(len(g), -1)
    y = -np.asarray(g, np.float32)
    return O.train(x, y, 1, **RAW, **kw)


@pytest.mark.parametrize("fixed", [False, True], ids=["f64", "fixed_point"])
def test_splits_on_separating_feature(fixed):
    nodes, ptr, base, margins = _grow([0.0, 0.0, 1.0, 1.0], [1.0, 1.0, -1.0, -1.0], max_depth=1,
                                      reg_lambda=0.0, min_child_weight=0.0, gamma=0.0, fixed_point=fixed)
    assert base[0] == 0.0
    assert len(nodes) == 3
    assert margins[0, 0] == np.float32(-1.0) and margins[2, 0] == np.float32(1.0)


@pytest.mark.parametrize("fixed", [False, True], ids=["f64", "fixed_point"])
def test_no_split_below_gamma(fixed):
    nodes, _, _, margins = _grow([0.0, 1.0], [1.0, -1.0], max_depth=3, gamma=1e9, fixed_point=fixed)
    assert len(nodes) == 1 and nodes[0]["left"] == -1
    # the root keeps the whole node's weight, -G/(H + lambda) = 0
    assert margins[0, 0] == margins[1, 0] == 0.0


@pytest.mark.parametrize("fixed", [False, True], ids=["f64", "fixed_point"])
def test_lossguide_respects_max_leaves(fixed):
    n = 64
    g = np.where(np.arange(n) % 2 == 0, 1.0, -1.0)
    nodes, ptr, _, _ = _grow(np.arange(n), g, grow_policy=1, max_leaves=4, max_depth=0,
                             min_child_weight=0.0, gamma=0.0, reg_lambda=0.0, fixed_point=fixed)
    leaves = int(np.sum(nodes["left"] == -1))
    assert 1 < leaves <= 4, leaves


@pytest.mark.parametrize("fixed", [False, True], ids=["f64", "fixed_point"])
def test_fully_present_feature_never_splits_missing_left(fixed):
    # feature 1 holds the one NaN that makes the index sparse and is
    # otherwise constant; feature 0 is fully present, so its backward
    # (missing-left) pass never runs
    x = np.array([[0, 5], [1, 5], [2, 5], [3, np.nan], [4, 5], [5, 5]], np.float32)
    nodes, _, _, _ = _grow(x, [1.0, 1.0, 1.0, -1.0, -1.0, -1.0], max_depth=1, reg_lambda=0.0,
                           min_child_weight=0.0, gamma=0.0, fixed_point=fixed)
    _, _, dense = O.bin_dense(x, *O.cuts_dense(x, 256))
    assert not dense
    assert len(nodes) == 3
    root = nodes[0]
    assert root["split_feature"] == 0
    assert not root["default_left"]
    assert 2.0 < root["split_cond"] <= 3.0


def _root_leaf(g, **kw):
    nodes, _, _, _ = _grow(np.zeros(len(g)), g, max_depth=1, min_child_weight=0.0, **kw)
    assert len(nodes) == 1  # one value: nothing to split on
    return nodes[0]["leaf_value"]


def test_weight_closed_form():
    # G = -4, H = 2, lambda = 1: w = 4/3
    assert _root_leaf([-2.0, -2.0], reg_lambda=1.0) == np.float32(4.0 / 3.0)


def test_l1_threshold_shrinks_toward_zero():
    # T_alpha(G): -5 with alpha 2 -> -3, so w = 3 / (1 + 1); |G| <= alpha -> 0
    assert _root_leaf([-5.0], reg_lambda=1.0, alpha=2.0) == np.float32(1.5)
    assert _root_leaf([5.0], reg_lambda=1.0, alpha=2.0) == np.float32(-1.5)
    assert _root_leaf([1.0], reg_lambda=1.0, alpha=2.0) == 0.0


def test_max_delta_step_clamps_weight():
    # unclamped weight 100, clamped to 1
    assert _root_leaf([-100.0], reg_lambda=0.0, max_delta_step=1.0) == np.float32(1.0)
    assert _root_leaf([100.0], reg_lambda=0.0, max_delta_step=1.0) == np.float32(-1.0)
