"""Monotone constraints in the oracle, pinned to the reference's own tests.

The reference grows one tree from given gradient pairs
(src/tree/builder/hist/mod.rs: `monotone_increasing_is_enforced` :1346,
`missing_only_left_split_under_monotone_constraint` :1463,
`fully_present_feature_never_splits_missing_left` :1516). The oracle trains
from labels, so the pairs are injected through reg:squarederror with base
score 0 and unit weights (g = 0 - y, h = 1) and eta 1 (the margins are the
tree's leaf values). Each case runs in both summation modes.
"""

import numpy as np
import pytest

import oracle_lib as O

MODES = [False, True]


def one_tree(x, g, **kw):
    x = np.asarray(x, np.float32).reshape(len(g), -1)
    y = -np.asarray(g, np.float32)
    kw = dict(dict(objective=0, eta=1.0, base_score=0.0, rounds=1), **kw)
    rounds = kw.pop("rounds")
    nodes, ptr, base, margins = O.train(x, y, rounds, **kw)
    assert base[0] == 0.0
    return nodes, margins[:, 0]


def v_shape():
    """builder/mod.rs:403 `monotone_v_shape_data`: 60 rows, x = i/60,
    pseudo-residual -(|x - 0.5| - 0.25), unit Hessian."""
    x = (np.arange(60) / np.float32(60)).astype(np.float32)
    g = -(np.abs(x - np.float32(0.5)) - np.float32(0.25))
    return x, g.astype(np.float32)


@pytest.mark.parametrize("fixed", MODES)
def test_monotone_increasing_is_enforced(fixed):
    x, g = v_shape()
    kw = dict(max_depth=4, min_child_weight=0.0, gamma=0.0, reg_lambda=1.0, fixed_point=fixed)
    _, pred = one_tree(x, g, monotone=[1], **kw)
    assert np.all(np.diff(pred) >= -1e-5), pred
    # the unconstrained fit of the same data is not monotone
    _, free = one_tree(x, g, **kw)
    assert not np.all(np.diff(free) >= -1e-5)


@pytest.mark.parametrize("fixed", MODES)
def test_monotone_decreasing_mirrors_increasing(fixed):
    x, g = v_shape()
    kw = dict(max_depth=4, min_child_weight=0.0, gamma=0.0, reg_lambda=1.0, fixed_point=fixed)
    _, pred = one_tree(x, g, monotone=[-1], **kw)
    assert np.all(np.diff(pred) <= 1e-5), pred


@pytest.mark.parametrize("fixed", MODES)
def test_missing_only_left_split_under_monotone_constraint(fixed):
    x = [0.0, 1.0, 2.0, 3.0, np.nan, np.nan]
    g = [-1.0] * 4 + [1.0, 1.0]
    nodes, pred = one_tree(x, g, max_depth=1, reg_lambda=0.0, min_child_weight=0.0, gamma=0.0,
                           monotone=[1], fixed_point=fixed)
    assert len(nodes) == 3
    root = nodes[0]
    assert root["default_left"] == 1 and np.isfinite(root["split_cond"])
    assert abs(nodes[root["left"]]["sum_hess"] - 2.0) < 1e-6
    assert abs(nodes[root["right"]]["sum_hess"] - 4.0) < 1e-6
    np.testing.assert_allclose(pred[:4], 1.0, atol=1e-6)
    np.testing.assert_allclose(pred[4:], -1.0, atol=1e-6)


@pytest.mark.parametrize("fixed", MODES)
def test_fully_present_feature_never_splits_missing_left(fixed):
    x = [0.0, 5.0, 1.0, 5.0, 2.0, 5.0, 3.0, np.nan, 4.0, 5.0, 5.0, 5.0]
    g = [1.0, 1.0, 1.0, -1.0, -1.0, -1.0]
    nodes, pred = one_tree(x, g, max_depth=1, reg_lambda=0.0, min_child_weight=0.0, gamma=0.0,
                           monotone=[1, 0], fixed_point=fixed)
    assert len(nodes) == 3
    root = nodes[0]
    assert root["split_feature"] == 0 and root["default_left"] == 0
    assert 2.0 < root["split_cond"] <= 3.0
    np.testing.assert_allclose(pred[:3], -1.0, atol=1e-6)
    np.testing.assert_allclose(pred[3:], 1.0, atol=1e-6)


def test_child_bounds_follow_the_midpoint():
    """constraints.rs:136 `increasing_child_bounds_order` through training: a
    depth-2 increasing fit keeps every leaf of the left subtree at or below
    every leaf of the right one."""
    rng = np.random.default_rng(1)
    x = rng.standard_normal(400).astype(np.float32)
    g = (-np.sin(3 * x) - 0.5 * x).astype(np.float32)
    for fixed in MODES:
        nodes, pred = one_tree(x, g, max_depth=3, min_child_weight=0.0, monotone=[1], fixed_point=fixed)
        order = np.argsort(x, kind="stable")
        assert np.all(np.diff(pred[order]) >= -1e-6)
