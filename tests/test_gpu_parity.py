"""The CUDA path (through the C ABI) against the CPU oracle.

* Gradients: bit-exact against the reference's host arithmetic.
* Training: bit-exact against the oracle's fixed-point mode (the same
  arithmetic by construction: exact int64 sums, the reference's f32 scoring)
  on every config shape at test size; bit-exact against the reference's own
  saved training fixtures; against the reference's f64 mode, identical
  structure except exact-gain ties and leaf values within 1e-5 relative.
* Prediction: bit-exact against the saved prediction fixtures and the oracle.
* RowEngine calls one by one: histograms, totals, partitions and scans.
"""

import numpy as np
import pytest

import hessboost_b200 as H
import oracle_lib as O
import parity as P
from hessboost_b200 import synth

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def assert_forest_equal(nodes, ptr, onodes, optr, what=""):
    assert len(ptr) == len(optr), what
    np.testing.assert_array_equal(np.asarray(ptr, np.uint64), np.asarray(optr, np.uint64), err_msg=what)
    for k in ("left", "right", "split_feature", "default_left", "split_bin"):
        np.testing.assert_array_equal(nodes[k], onodes[k], err_msg=f"{what} {k}")
    for k in ("split_cond", "leaf_value", "sum_hess", "split_gain"):
        np.testing.assert_array_equal(_bits(nodes[k]), _bits(onodes[k]), err_msg=f"{what} {k}")


def gpu_train(x, y, rounds, **kw):
    params = H.TrainingParams(**kw)
    m = H.train(params, x, y, rounds)
    return m


# ------------------------------------------------------------- gradients
@pytest.mark.parametrize("n", [7, 16, 1000, 4099])
def test_gradients_bit_exact(n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal((n, 3)).astype(np.float32)
    y = (rng.random(n) < 0.5).astype(np.float32)
    m = (rng.standard_normal(n) * 4).astype(np.float32)
    if n > 100:
        m[40:48] = 85.0  # a vector group past the fast-exp range (scalar path)
        m[97] = -120.0
    e = H.Engine()
    e.upload(H.BinnedMatrix.from_dense(x))
    for kind in (H.HB_LOSS_LOGISTIC, H.HB_LOSS_SQUARED_ERROR):
        e.load_margins(m)
        assert e.gradients(kind, y)
        got, sg, sh = e.read_gradients()
        want = O.gradients(kind, m, y)
        np.testing.assert_array_equal(_bits(got), _bits(want))
        assert sg == O.fixed_scale(np.abs(want[:, 0]).max(), n)
        assert sh == O.fixed_scale(np.abs(want[:, 1]).max(), n)
    e.close()


# ------------------------------------------------------ training: fixtures
def test_training_fixture_early_stopping_bit_exact():
    g = O.golden()
    ref = [m for m in g["models"] if m["name"] == "early_stopping"][-1]
    m = gpu_train(g["x"], g["y1"][:, 0], 4, max_depth=3, eta=0.3)
    gn, gp = O.golden_nodes(ref)
    gn["split_bin"] = m.nodes["split_bin"]  # the fixture has no bins
    assert np.float32(m.base).view(np.uint32) == np.float32(ref["base_score"][0]).view(np.uint32)
    assert_forest_equal(m.nodes, m.tree_ptr, gn, gp, "early_stopping")


def test_training_fixture_multi_target_bit_exact():
    # Squared error's targets are independent: output t's trees are a
    # single-output run on label column t (round.rs:318 output-major order).
    g = O.golden()
    ref = [m for m in g["models"] if m["name"] == "multi_target"][-1]
    gn, gp = O.golden_nodes(ref)
    runs = [gpu_train(g["x"], g["y2"][:, t], 4, max_depth=3, eta=0.3) for t in range(2)]
    for r in range(4):
        for t in range(2):
            k = 2 * r + t
            want = gn[int(gp[k]) : int(gp[k + 1])].copy()
            run = runs[t]
            got = run.nodes[int(run.tree_ptr[r]) : int(run.tree_ptr[r + 1])]
            want["split_bin"] = got["split_bin"]
            assert_forest_equal(got, [0, len(got)], want, [0, len(want)], f"round {r} target {t}")


# --------------------------------------------- training: oracle fixed point
def _step_dataset(n):
    """training/train/tests.rs:22 `step_dataset`: x = i / n, y = [x >= 0.5]."""
    x = (np.arange(n, dtype=np.float32) / np.float32(n)).reshape(n, 1)
    return x, (x[:, 0] >= 0.5).astype(np.float32)


CASES = {
    # shape of C1 (dense regression), reduced rows
    "c1_regression": dict(gen=lambda: synth.regression_c1(20_000, 28, seed=3), rounds=4,
                          kw=dict(max_depth=6, eta=0.1)),
    # shape of C2 (5% NaN, logistic, depth 8), reduced rows
    "c2_logistic": dict(gen=lambda: synth.logistic_c2(30_011, 28, seed=5), rounds=4,
                        kw=dict(objective="binary:logistic", max_depth=8, eta=0.1)),
    # odd shapes: few rows, ragged count, depth 1, a few features
    "tiny_ragged": dict(gen=lambda: synth.logistic_c2(37, 5, seed=9, missing=0.2), rounds=3,
                        kw=dict(objective="binary:logistic", max_depth=4, eta=0.3)),
    "stump": dict(gen=lambda: synth.regression_c1(5000, 6, seed=2), rounds=2, kw=dict(max_depth=1)),
    "regularised": dict(gen=lambda: synth.regression_c1(8000, 10, seed=4), rounds=3,
                        kw=dict(max_depth=5, reg_lambda=3.0, alpha=0.5, gamma=0.2, min_child_weight=20.0,
                                max_delta_step=0.7)),
    # 13-28 features (three records a row block): leaves above the depth
    # limit from regularisation, and the deepest complete-tree walk (10)
    "regularised_rows3": dict(gen=lambda: synth.logistic_c2(30_011, 20, seed=31), rounds=4,
                              kw=dict(objective="binary:logistic", max_depth=6, reg_lambda=2.0, gamma=0.4,
                                      min_child_weight=30.0, eta=0.3)),
    "depth10_rows3": dict(gen=lambda: synth.logistic_c2(50_021, 16, seed=32), rounds=3,
                          kw=dict(objective="binary:logistic", max_depth=10, eta=0.3)),
    "few_bins": dict(gen=lambda: synth.logistic_c2(6000, 12, seed=8), rounds=3,
                     kw=dict(objective="binary:logistic", max_depth=6, max_bin=16)),
    # enough rows for the 32-bit split-accumulator histogram kernel
    "c2_large": dict(gen=lambda: synth.logistic_c2(600_003, 28, seed=6), rounds=2,
                     kw=dict(objective="binary:logistic", max_depth=8, eta=0.1)),
    # several 32-feature groups: one group per histogram CTA (256 bins), and
    # two groups per CTA (bins <= 128; the last CTA row holds one group)
    "wide_bins256": dict(gen=lambda: synth.logistic_c2(600_003, 70, seed=12), rounds=1,
                         kw=dict(objective="binary:logistic", max_depth=5, eta=0.1)),
    "wide_bins64": dict(gen=lambda: synth.logistic_c2(600_003, 70, seed=13), rounds=1,
                        kw=dict(objective="binary:logistic", max_depth=5, eta=0.1, max_bin=64)),
    # narrow last groups (<= 8 features, accumulated in column copies): 4
    # features (C3's 100 at 128 bins, two groups per CTA) and 1 feature
    "narrow_group4": dict(gen=lambda: synth.logistic_c2(600_003, 100, seed=18), rounds=1,
                          kw=dict(objective="binary:logistic", max_depth=4, eta=0.1, max_bin=128)),
    "narrow_group1": dict(gen=lambda: synth.logistic_c2(600_003, 33, seed=19), rounds=1,
                          kw=dict(objective="binary:logistic", max_depth=4, eta=0.1)),
    # lossguide growth (best loss change first): by max_leaves, by max_depth
    # alone (2^max_depth leaves), both, with regularisation leaving nodes
    # unexpandable, a tiny ragged set, and the 32-bit histogram kernel
    "lossguide_leaves": dict(gen=lambda: synth.logistic_c2(30_011, 28, seed=15), rounds=3,
                             kw=dict(objective="binary:logistic", grow_policy="lossguide", max_depth=0,
                                     max_leaves=31, eta=0.1)),
    "lossguide_depth": dict(gen=lambda: synth.regression_c1(20_000, 12, seed=16), rounds=3,
                            kw=dict(grow_policy="lossguide", max_depth=5, max_leaves=0)),
    "lossguide_both": dict(gen=lambda: synth.regression_c1(9000, 10, seed=17), rounds=3,
                           kw=dict(grow_policy="lossguide", max_depth=4, max_leaves=12, gamma=0.3,
                                   min_child_weight=40.0, reg_lambda=2.0)),
    "lossguide_tiny": dict(gen=lambda: synth.logistic_c2(41, 5, seed=18, missing=0.2), rounds=3,
                           kw=dict(objective="binary:logistic", grow_policy="lossguide", max_depth=0,
                                   max_leaves=8, eta=0.3)),
    # the reference's lossguide end-to-end set (training/train/tests.rs:218)
    "lossguide_step": dict(gen=lambda: _step_dataset(120), rounds=60,
                           kw=dict(grow_policy="lossguide", max_leaves=16, eta=0.3)),
    "lossguide_large": dict(gen=lambda: synth.logistic_c2(600_003, 28, seed=19), rounds=2,
                            kw=dict(objective="binary:logistic", grow_policy="lossguide", max_depth=0,
                                    max_leaves=96, eta=0.1)),
    # monotone constraints (constraints.rs): bounded child weights, direction
    # checks, child bounds at the midpoint, bounded leaves; depthwise with
    # missing values, lossguide, and the CTA scan (256 bins) and warp scan
    # (64 bins)
    "monotone_depthwise": dict(gen=lambda: synth.logistic_c2(40_009, 8, seed=24), rounds=4,
                               kw=dict(objective="binary:logistic", max_depth=6, eta=0.3,
                                       monotone_constraints=(1, -1, 0, 1, 0, 0, -1, 0))),
    "monotone_bins64": dict(gen=lambda: synth.regression_c1(30_011, 6, seed=25), rounds=4,
                            kw=dict(max_depth=5, max_bin=64, min_child_weight=0.0, reg_lambda=0.5,
                                    monotone_constraints=(-1, 1, 1, 0, 0, 1))),
    # indexes the row records cannot hold: 300 features (the dense index
    # converted to the CSR layout on upload) and features of up to 1024 bins
    # (the CSR index, the chunked split scan), depthwise and lossguide
    "wide_300": dict(gen=lambda: synth.logistic_c2(20_011, 300, seed=28), rounds=2,
                     kw=dict(objective="binary:logistic", max_depth=5, eta=0.3)),
    "bins_1024": dict(gen=lambda: synth.regression_c1(30_011, 8, seed=29), rounds=3,
                      kw=dict(max_depth=6, max_bin=1024)),
    "bins_1024_missing_lossguide": dict(gen=lambda: synth.logistic_c2(25_013, 6, seed=30, missing=0.1), rounds=3,
                                        kw=dict(objective="binary:logistic", grow_policy="lossguide", max_depth=0,
                                                max_leaves=20, max_bin=1024, eta=0.3)),
    "monotone_lossguide": dict(gen=lambda: synth.logistic_c2(20_011, 8, seed=26), rounds=3,
                               kw=dict(objective="binary:logistic", grow_policy="lossguide", max_depth=0,
                                       max_leaves=24, eta=0.3, monotone_constraints=(1, 1, -1, 0, 0, 0, 0, -1))),
}


def _orc_kw(kw):
    m = dict(kw)
    if "monotone_constraints" in m:
        m["monotone"] = list(m.pop("monotone_constraints"))
    if "objective" in m:
        m["objective"] = 1 if m["objective"] == "binary:logistic" else 0
    if "grow_policy" in m:
        m["grow_policy"] = 1 if m["grow_policy"] == "lossguide" else 0
    return m


@pytest.mark.parametrize("case", sorted(CASES))
def test_training_matches_oracle_fixed_point(case):
    spec = CASES[case]
    x, y = spec["gen"]()
    m = gpu_train(x, y, spec["rounds"], **spec["kw"])
    on, op, ob, omarg = O.train(x, y, spec["rounds"], fixed_point=True, **_orc_kw(spec["kw"]))
    assert np.float32(m.base).view(np.uint32) == ob.view(np.uint32)[0]
    assert_forest_equal(m.nodes, m.tree_ptr, on, op, case)
    # training margins: base + leaves in round order; prediction of the
    # training rows routes them as the binned partitions did
    pred = m.predict_margin(x)
    np.testing.assert_array_equal(_bits(pred), _bits(omarg[:, 0]))


@pytest.mark.parametrize("case", ["c1_regression", "c2_logistic", "c2_large", "regularised", "few_bins",
                                  "monotone_depthwise"])
def test_training_against_reference_f64_mode(case):
    """North-star criteria against the reference's own summation (the
    oracle's f64 mode), round by round: each round both start from the
    oracle's margins, so a tie in one round leaves every later round
    compared. Identical structure except gain ties (1e-5), leaves within
    1e-5 relative (atol 1e-7), margins within 1e-6 relative (atol 1e-7);
    tolerances in tests/parity.py."""
    spec = CASES[case]
    x, y = spec["gen"]()
    params = H.TrainingParams(**spec["kw"])
    e = H.Engine()
    try:
        e.upload(H.BinnedMatrix.from_dense(x, params.max_bin))
        e.train_begin(y, H.base_margin(params, y))
        t64 = O.Trainer(x, y, fixed_point=False, **_orc_kw(spec["kw"]))
        out = P.forced_f64_rounds(e, params, t64, max(spec["rounds"], 6))
        t64.close()
    finally:
        e.close()
    assert out["pass"], out
    assert out["trees_structure_equal"] + len(out["ties"]) == out["rounds"]


def _first_difference_is_a_tie(on, op, nodes, ptr):
    """Where two forests first differ in structure, the two splits' gains
    agree to 1e-5 relative (an f32 gain tie), else False."""
    t = next(i for i in range(min(len(op), len(ptr)) - 1)
             if not np.array_equal(on[int(op[i]):int(op[i + 1])]["split_bin"],
                                   nodes[int(ptr[i]):int(ptr[i + 1])]["split_bin"]))
    a = on[int(op[t]):int(op[t + 1])]
    b = nodes[int(ptr[t]):int(ptr[t + 1])]
    k = next(i for i in range(min(len(a), len(b))) if a[i]["split_bin"] != b[i]["split_bin"])
    rel = abs(float(a[k]["split_gain"]) - float(b[k]["split_gain"])) / max(abs(float(a[k]["split_gain"])), 1e-30)
    return rel <= 1e-5


@pytest.mark.parametrize("n,f,k,depth,max_bin,rounds", [(20_011, 12, 5, 5, 64, 3),
                                                        (60_000, 100, 10, 6, 128, 2),
                                                        (20_013, 12, 2, 5, 64, 3),
                                                        (30_001, 20, 4, 6, 128, 3)])
def test_softmax_training_matches_oracle(n, f, k, depth, max_bin, rounds):
    """multi:softmax, gradients on the device (C3's shape at the second
    size). The device exp is CUDA's double exp rounded once to f32, the
    oracle's (as the reference's) glibc expf; they can differ in the last
    bit on rare inputs, so the bar is the north-star criteria: identical
    structure except gain ties, leaves within 1e-5 relative, margins within
    1e-6 relative."""
    x, y = synth.multiclass_c3(n, f, k, seed=n)
    p = H.TrainingParams(objective="multi:softmax", num_class=k, max_depth=depth, eta=0.2,
                         max_bin=max_bin)
    m = H.train(p, x, y, rounds)
    assert len(m.tree_ptr) == rounds * k + 1
    on, op, obase, omarg = O.train(x, y, rounds, objective=2, n_outputs=k, max_depth=depth, eta=0.2,
                                   max_bin=max_bin, fixed_point=True)
    np.testing.assert_array_equal(m.bases().view(np.uint32), obase.view(np.uint32))
    if np.array_equal(op, m.tree_ptr) and np.array_equal(on["split_bin"], m.nodes["split_bin"]):
        np.testing.assert_array_equal(on["split_feature"], m.nodes["split_feature"])
        np.testing.assert_array_equal(on["default_left"], m.nodes["default_left"])
        np.testing.assert_allclose(m.nodes["leaf_value"], on["leaf_value"], rtol=1e-5, atol=1e-7)
        pred = m.predict_margin(x)
        np.testing.assert_allclose(pred, omarg, rtol=1e-6, atol=1e-6)
    else:
        assert _first_difference_is_a_tie(on, op, m.nodes, m.tree_ptr)


def test_lossguide_grow_tree_matches_oracle_and_refusals():
    """One lossguide tree through hb_grow_tree (the RowEngine seam) equals the
    oracle's first tree; softmax and unbounded lossguide are refused."""
    x, y = synth.logistic_c2(12_007, 9, seed=23)
    params = H.TrainingParams(objective="binary:logistic", grow_policy="lossguide", max_depth=0,
                              max_leaves=17, eta=0.3)
    mtx = H.BinnedMatrix.from_dense(x)
    base = H.base_margin(params, y)
    e = H.Engine()
    try:
        e.upload(mtx)
        e.load_margins(np.full(mtx.n_rows, base, np.float32))
        assert e.gradients(H.HB_LOSS_LOGISTIC, y)
        got = e.grow_tree(params)
        on, op, _, _ = O.train(x, y, 1, objective=1, grow_policy=1, max_depth=0, max_leaves=17, eta=0.3,
                               fixed_point=True)
        assert_forest_equal(got, [0, len(got)], on, op, "grow_tree")
        assert e.gradients(H.HB_LOSS_LOGISTIC, y)
        for bad in (dict(max_depth=0, max_leaves=0), dict(max_depth=0, max_leaves=2000)):
            p = H.TrainingParams(objective="binary:logistic", grow_policy="lossguide", **bad)
            with pytest.raises(H.HbError):
                e.grow_tree(p)
    finally:
        e.close()


@pytest.mark.parametrize("k", [2, 4])
def test_short_softmax_classes_bit_exact(k):
    """2 and 4 classes take x86_64's short-row vector kernel (whole rows per
    8-lane vector) on every row of a vector with no irregular row: its
    exponential is the reference's own polynomial, so with every margin
    regular the device's gradients, trees and margins equal the oracle's bit
    for bit (a row count that leaves a scalar tail, and one class refused:
    num_class 1)."""
    x, y = synth.multiclass_c3(9_003, 8, k, seed=40 + k)
    p = H.TrainingParams(objective="multi:softmax", num_class=k, max_depth=4, eta=0.3, max_bin=64)
    m = H.train(p, x, y, 3)
    on, op, obase, omarg = O.train(x, y, 3, objective=2, n_outputs=k, max_depth=4, eta=0.3, max_bin=64,
                                   fixed_point=True)
    np.testing.assert_array_equal(m.bases().view(np.uint32), obase.view(np.uint32))
    assert_forest_equal(m.nodes, m.tree_ptr, on, op, f"softmax k={k}")
    np.testing.assert_array_equal(_bits(m.predict_margin(x).reshape(omarg.shape)), _bits(omarg))
    with pytest.raises(H.HbError):
        H.train(H.TrainingParams(objective="multi:softmax", num_class=1, max_depth=3), x, np.zeros_like(y), 1)


def test_training_is_deterministic():
    x, y = synth.logistic_c2(20_000, 28, seed=11)
    a = gpu_train(x, y, 3, objective="binary:logistic", max_depth=8)
    b = gpu_train(x, y, 3, objective="binary:logistic", max_depth=8)
    assert_forest_equal(a.nodes, a.tree_ptr, b.nodes, b.tree_ptr, "rerun")


def test_constant_labels_give_single_leaves():
    x, _ = synth.regression_c1(1000, 6, seed=1)
    y = np.full(1000, 2.5, np.float32)
    m = gpu_train(x, y, 2, max_depth=4)
    assert list(m.tree_ptr) == [0, 1, 2]
    assert np.all(m.nodes["left"] == -1)


# ----------------------------------------------------------- prediction
def test_prediction_fixtures_bit_exact():
    g = O.golden()
    for ref in g["models"]:
        nodes, ptr = O.golden_nodes(ref)
        n, outs, w = O.golden_layout(ref)
        gn = nodes[: int(ptr[n])].copy().view(H.NODE_DTYPE)
        p = H.Predictor(gn, ptr[: n + 1], np.array(ref["base_score"], np.float32), 4, outs, w)
        got = p.predict_margin(g["x"])
        p.close()
        np.testing.assert_array_equal(_bits(got).ravel(), np.array(ref["margins_bits"], np.uint32), err_msg=ref["name"])


def test_prediction_random_forest_matches_oracle():
    nodes, ptr = synth.forest_c5(n_trees=40, depth=8, n_cols=50, seed=3)
    x = synth.rows_c5(20_003, 50, seed=4)
    base = np.array([0.25], np.float32)
    p = H.Predictor(nodes, ptr, base, 50)
    got = p.predict_margin(x)
    p.close()
    want = O.predict(nodes.view(O.NODE_DTYPE), ptr, 1, base, x)
    np.testing.assert_array_equal(_bits(got), _bits(want))


def _chain_tree(depth, n_cols, rng):
    """A tree of one long path (depth `depth`) with leaves hanging off it."""
    n = 2 * depth + 1
    a = np.zeros(n, H.NODE_DTYPE)
    for i in range(depth):
        a[2 * i]["left"], a[2 * i]["right"] = 2 * i + 1, 2 * i + 2
        a[2 * i]["split_feature"] = rng.integers(0, n_cols)
        a[2 * i]["split_cond"] = np.float32(rng.standard_normal())
        a[2 * i]["default_left"] = rng.integers(0, 2)
        a[2 * i + 1]["left"] = a[2 * i + 1]["right"] = -1
        a[2 * i + 1]["leaf_value"] = np.float32(rng.normal(0, 0.1))
    a[2 * depth]["left"] = a[2 * depth]["right"] = -1
    a[2 * depth]["leaf_value"] = np.float32(0.5)
    a["split_bin"] = -1
    return a


@pytest.mark.parametrize("depth", [3, 10, 14])
def test_prediction_deep_and_shallow_trees(depth):
    """Trees up to depth 10 take the complete-tree layout (shallow leaves
    padded), deeper ones the general walk; both equal the oracle."""
    rng = np.random.default_rng(depth)
    trees = [_chain_tree(depth, 12, rng) for _ in range(5)]
    f5, p5 = synth.forest_c5(n_trees=3, depth=4, n_cols=12, seed=depth)
    nodes = np.concatenate(trees + [f5])
    ptr = np.concatenate([[0], np.cumsum([len(t) for t in trees])]).astype(np.uint64)
    ptr = np.concatenate([ptr, ptr[-1] + p5[1:]]).astype(np.uint64)
    x = synth.rows_c5(5_001, 12, seed=depth, missing=0.2)
    base = np.array([-0.5], np.float32)
    w = rng.uniform(0.5, 1.5, len(ptr) - 1).astype(np.float32)
    p = H.Predictor(nodes, ptr, base, 12, tree_weight=w)
    got = p.predict_margin(x)
    p.close()
    want = O.predict(nodes.view(O.NODE_DTYPE), ptr, 1, base, x, tree_weight=w)
    np.testing.assert_array_equal(_bits(got), _bits(want))


def test_prediction_wide_rows():
    """300 features: the complete-tree path with a smaller row tile."""
    nodes, ptr = synth.forest_c5(n_trees=30, depth=8, n_cols=300, seed=8)
    x = synth.rows_c5(3_001, 300, seed=9)
    base = np.array([0.0], np.float32)
    p = H.Predictor(nodes, ptr, base, 300)
    got = p.predict_margin(x)
    p.close()
    want = O.predict(nodes.view(O.NODE_DTYPE), ptr, 1, base, x)
    np.testing.assert_array_equal(_bits(got), _bits(want))


# ------------------------------------------------------ RowEngine calls
def _setup_engine(n=3001, f=7, seed=21, missing=0.1):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, f)).astype(np.float32)
    x[rng.random(x.shape) < missing] = np.nan
    y = (rng.random(n) < 0.4).astype(np.float32)
    mtx = H.BinnedMatrix.from_dense(x)
    e = H.Engine()
    e.upload(mtx)
    margins = (rng.standard_normal(n) * 0.5).astype(np.float32)
    e.load_margins(margins)
    assert e.gradients(H.HB_LOSS_LOGISTIC, y)
    gp, sg, sh = e.read_gradients()
    return e, x, mtx, gp, sg, sh


def _oracle_hist(x, mtx, rows, gp, sg, sh):
    q = O.hist(x, mtx.feature_offset, mtx.cut_values, rows, gp, fixed_point=True, sg=sg, sh=sh)
    return q[:, 0].astype(np.float64) * 2.0 ** -sg, q[:, 1].astype(np.float64) * 2.0 ** -sh


def test_row_engine_histograms_partition_scan():
    e, x, mtx, gp, sg, sh = _setup_engine()
    n = x.shape[0]
    root = e.begin_tree(np.arange(n))
    assert root.len == n and root.contiguous == 1
    g, h = e.root_total(root)
    q = np.rint(gp.astype(np.float64) * [2.0 ** sg, 2.0 ** sh]).astype(np.int64).sum(axis=0)
    assert g == q[0] * 2.0 ** -sg and h == q[1] * 2.0 ** -sh
    hist = e.histograms([root])[0]
    og, oh = _oracle_hist(x, mtx, np.arange(n), gp, sg, sh)
    np.testing.assert_array_equal(hist[:, 0], og)
    np.testing.assert_array_equal(hist[:, 1], oh)
    # partition on feature 2 at local bin 100 with missing going left
    (left, right), = e.partition([(root, 2, 100, True)])
    lrows, rrows = e.rows([left, right])
    fo = mtx.feature_offset
    col = mtx.columns[2]
    miss = np.isnan(x[:, 2])
    want_left = np.nonzero(miss | (~miss & (col < 100)))[0]
    np.testing.assert_array_equal(lrows, want_left)
    np.testing.assert_array_equal(rrows, np.setdiff1d(np.arange(n), want_left))
    # resident histograms: build the left child, sibling by subtraction
    assert e.reserve_hists(4)
    e.build_resident([(root, 0)])
    e.build_resident([(left, 1)], siblings=[(0, 1)])
    lh = e.read_hist(1)
    rh = e.read_hist(0)
    og, oh = _oracle_hist(x, mtx, lrows, gp, sg, sh)
    np.testing.assert_array_equal(lh[:, 0], og)
    og, oh = _oracle_hist(x, mtx, rrows, gp, sg, sh)
    np.testing.assert_array_equal(rh[:, 0], og)
    np.testing.assert_array_equal(rh[:, 1], oh)
    # scans: the device's winner equals a sequential host scan of the same
    # histogram under the reference's scoring
    e.build_resident([(root, 2)])
    params = H.TrainingParams()
    scans = e.scan_resident(params.reg(), [(2, (g, h), np.arange(7))])
    s = scans[0]
    assert s.kind == 2 and s.feature < 7 and s.loss_chg > 0
    m1 = e.read_margins()
    e.add_leaf_values([left, right], [0.5, -0.25])
    m2 = e.read_margins()
    want = m1.copy()
    want[lrows] += np.float32(0.5)
    want[rrows] += np.float32(-0.25)
    np.testing.assert_array_equal(_bits(m2), _bits(want))
    e.close()


def test_backend_build_features_and_prepare_match_oracle():
    """HistogramBackend::{build, build_features, prepare} through the C ABI
    against the oracle's fixed-point sums of the same rows."""
    e, x, mtx, gp, sg, sh = _setup_engine(n=50_021, f=9, seed=31)
    n = x.shape[0]
    rng = np.random.default_rng(2)
    try:
        rows = np.sort(rng.choice(n, 20_000, replace=False)).astype(np.uint32)
        og, oh = _oracle_hist(x, mtx, rows, gp, sg, sh)
        got = e.build(rows)
        np.testing.assert_array_equal(got[:, 0], og)
        np.testing.assert_array_equal(got[:, 1], oh)
        fo = mtx.feature_offset
        gotf = e.build_features(rows, [7, 2])
        for f in (7, 2):
            a, b = int(fo[f]), int(fo[f + 1])
            np.testing.assert_array_equal(gotf[a:b, 0], og[a:b])
            np.testing.assert_array_equal(gotf[a:b, 1], oh[a:b])
        # prepare: host gradient pairs staged as they are
        gp2 = np.stack([rng.standard_normal(n), rng.uniform(0.01, 2.0, n)], 1).astype(np.float32)
        e.prepare(gp2)
        got_gp, sg2, sh2 = e.read_gradients()
        np.testing.assert_array_equal(_bits(got_gp), _bits(gp2))
        assert sg2 == O.fixed_scale(np.abs(gp2[:, 0]).max(), n)
        assert sh2 == O.fixed_scale(np.abs(gp2[:, 1]).max(), n)
        og2, oh2 = _oracle_hist(x, mtx, rows, gp2, sg2, sh2)
        got2 = e.build(rows)
        np.testing.assert_array_equal(got2[:, 0], og2)
        np.testing.assert_array_equal(got2[:, 1], oh2)
    finally:
        e.close()


def test_monotone_training_is_monotone():
    """A constrained feature moves the prediction one way only: rows that
    differ only in feature 0 (increasing) or feature 1 (decreasing) predict
    in that order."""
    x, y = synth.logistic_c2(30_011, 6, seed=27)
    m = gpu_train(x, y, 6, objective="binary:logistic", max_depth=6, eta=0.3,
                  monotone_constraints=(1, -1, 0, 0, 0, 0))
    rng = np.random.default_rng(3)
    base = rng.standard_normal((64, 6)).astype(np.float32)
    grid = np.linspace(-3, 3, 41, dtype=np.float32)
    for f, sign in ((0, 1.0), (1, -1.0)):
        rows = np.repeat(base, grid.size, axis=0)
        rows[:, f] = np.tile(grid, base.shape[0])
        p = m.predict_margin(rows).reshape(base.shape[0], grid.size)
        assert np.all(sign * np.diff(p, axis=1) >= 0.0), f


def test_scan_resident_matches_oracle_scan():
    """RowEngine::scan_resident against the oracle's fixed-point search of
    the same histograms: the winning feature, loss change (bits), direction,
    offset and accumulated statistics, for requests in feature order, in a
    shuffled order (the merge keeps need_replace's lower-feature rule), with
    monotone directions and with finite bounds; a node with missing values
    (the backward pass scored) and one without."""
    e, x, mtx, gp, sg, sh = _setup_engine(n=20_011, f=7, seed=41, missing=0.15)
    n = x.shape[0]
    fo = mtx.feature_offset
    try:
        root = e.begin_tree(np.arange(n))
        (left, right), = e.partition([(root, 2, 90, False)])
        lrows, rrows = e.rows([left, right])
        assert e.reserve_hists(3)
        e.build_resident([(root, 0), (left, 1), (right, 2)])
        q = np.rint(gp.astype(np.float64) * [2.0 ** sg, 2.0 ** sh]).astype(np.int64)
        for params in (H.TrainingParams(), H.TrainingParams(reg_lambda=2.5, alpha=0.3, min_child_weight=5.0,
                                                            max_delta_step=0.4)):
            reg = params.reg()
            okw = dict(reg_lambda=params.reg_lambda, alpha=params.alpha,
                       min_child_weight=params.min_child_weight, max_delta_step=params.max_delta_step)
            cases = [
                (np.arange(7), None, (-np.inf, np.inf)),
                (np.array([5, 2, 6, 0, 3, 1, 4]), None, (-np.inf, np.inf)),
                (np.array([3, 1, 0, 6]), np.array([1, -1, 1, 0]), (-np.inf, np.inf)),
                (np.arange(7), np.array([1, 1, -1, 0, 1, -1, 0]), (-0.05, 0.08)),
                (np.array([4, 0, 2]), np.array([-1, 0, 1]), (-0.02, np.float32(0.3))),
            ]
            for slot, rows in ((0, np.arange(n)), (1, lrows), (2, rrows)):
                hq = O.hist(x, fo, mtx.cut_values, rows, gp, fixed_point=True, sg=sg, sh=sh)
                tq = q[rows].sum(axis=0)
                total = (tq[0] * 2.0 ** -sg, tq[1] * 2.0 ** -sh)
                reqs = [(slot, total, f, d, b) for f, d, b in cases]
                got = e.scan_resident(reg, reqs)
                for (f, d, b), r in zip(cases, got):
                    want = O.scan_node(hq, fo, mtx.dense, tq, sg, sh, f, d, b, **okw)
                    lo, up = np.float32(b[0]), np.float32(b[1])
                    assert np.float32(H.node_gain(total, reg, lo, up)) == np.float32(want.root_gain)
                    what = f"slot {slot} features {list(f)} dirs {d} bounds {b}"
                    assert r.kind == (H.HB_SCAN_NUMERIC if want.found else H.HB_SCAN_EMPTY), what
                    if not want.found:
                        continue
                    assert r.feature == want.feature, what
                    assert np.float32(r.loss_chg).view(np.uint32) == np.float32(want.loss_chg).view(np.uint32), what
                    assert r.backward == want.default_left, what
                    fs = int(fo[want.feature])
                    if want.default_left:
                        assert r.offset == (0 if want.bin < 0 else want.bin - fs + 1), what
                        acc = (tq[0] - want.left_g, tq[1] - want.left_h)
                    else:
                        assert r.offset == want.bin - fs, what
                        acc = (want.left_g, want.left_h)
                    assert r.acc.grad == acc[0] * 2.0 ** -sg and r.acc.hess == acc[1] * 2.0 ** -sh, what
    finally:
        e.close()


def test_stale_segments_are_refused():
    e, x, mtx, gp, sg, sh = _setup_engine(n=500)
    a = e.begin_tree(np.arange(500))
    e.begin_tree(np.arange(500))
    with pytest.raises(H.HbError) as ei:
        e.histograms([a])
    assert ei.value.status == H.HB_REFUSED
    e.close()


def test_non_ascending_rows_are_refused():
    e, *_ = _setup_engine(n=100)
    with pytest.raises(H.HbError):
        e.begin_tree(np.array([3, 2, 1]))
    e.close()


@pytest.mark.parametrize("n_cols,max_bin", [(28, 256), (70, 128)])
def test_histogram_kernels_agree(monkeypatch, n_cols, max_bin):
    """The 32-bit split-accumulator kernel (k_hist32) and the 64-bit-atomic
    one give the same exact int64 sums, one feature group a CTA (256 bins)
    and two (128 bins)."""
    x, y = synth.logistic_c2(1_100_000, n_cols, seed=13)
    m = H.BinnedMatrix.from_dense(x, max_bin)
    p = H.TrainingParams(objective="binary:logistic", max_depth=8, max_bin=max_bin)
    runs = []
    for kernel in ("32", "64"):
        monkeypatch.setenv("HB_HIST_KERNEL", kernel)
        runs.append(H.train(p, y=y, rounds=2, matrix=m))
    assert_forest_equal(runs[0].nodes, runs[0].tree_ptr, runs[1].nodes, runs[1].tree_ptr, "32 vs 64")


@pytest.mark.parametrize("n_cols,grow", [(6, "depthwise"), (28, "depthwise"), (28, "lossguide"), (40, "depthwise")])
def test_row_block_layout_agrees(monkeypatch, n_cols, grow):
    """Records in row blocks (5, 3 and 2 rows and their pairs to a 128-byte
    line for 16-, 32- and 48-byte records) and records apart with the pairs
    in their own array give the same forests and margins."""
    x, y = synth.logistic_c2(250_007, n_cols, seed=40 + n_cols)
    kw = dict(objective="binary:logistic", max_depth=7, eta=0.2)
    if grow == "lossguide":
        kw.update(grow_policy="lossguide", max_depth=0, max_leaves=40)
    runs = []
    for layout in ("1", "0"):
        monkeypatch.setenv("HB_ROW_BLOCKS", layout)
        runs.append(gpu_train(x, y, 3, **kw))
    assert_forest_equal(runs[0].nodes, runs[0].tree_ptr, runs[1].nodes, runs[1].tree_ptr, "blocks vs apart")
    np.testing.assert_array_equal(_bits(runs[0].predict_margin(x)), _bits(runs[1].predict_margin(x)))


@pytest.mark.parametrize("n_cols,missing", [(28, 0.05), (6, 0.2), (40, 0.0)])
def test_one_pass_partition_agrees_with_the_stable_one(monkeypatch, n_cols, missing):
    """Depthwise growth with the one-pass partition (children's rows in
    reservation order) and with the stable three-pass one grows the same
    forest and margins: nothing computed from a segment depends on the
    order of its rows."""
    x, y = synth.logistic_c2(300_007, n_cols, seed=60 + n_cols, missing=missing)
    runs = []
    for stable in ("0", "1"):
        monkeypatch.setenv("HB_STABLE_PARTITION", stable)
        runs.append(gpu_train(x, y, 4, objective="binary:logistic", max_depth=7, eta=0.3))
    assert_forest_equal(runs[0].nodes, runs[0].tree_ptr, runs[1].nodes, runs[1].tree_ptr, "one pass vs stable")
    np.testing.assert_array_equal(_bits(runs[0].predict_margin(x)), _bits(runs[1].predict_margin(x)))


@pytest.mark.parametrize("layout", ["dense", "csr"])
def test_lossguide_one_pass_partition_agrees_with_the_stable_one(monkeypatch, layout):
    """Lossguide growth with the one-pass partition (a node's children move
    to the other half of the 2n row buffer, in reservation order) and with
    the stable partition (every node in the first half) grows the same
    forest and training margins, dense with missing values and over a CSR
    index."""
    if layout == "dense":
        x, y = synth.logistic_c2(200_003, 12, seed=81, missing=0.1)
        m = H.BinnedMatrix.from_dense(x)
    else:
        indptr, indices, values, y = synth.sparse_c4(150_001, 300, density=0.05, seed=82)
        m = H.BinnedMatrix.from_csr(indptr, indices, values, 300, 64)
    p = H.TrainingParams(objective="binary:logistic", grow_policy="lossguide", max_depth=0, max_leaves=63,
                         eta=0.3, max_bin=256 if layout == "dense" else 64)
    runs = []
    for stable in ("0", "1"):
        monkeypatch.setenv("HB_STABLE_PARTITION", stable)
        e = H.Engine()
        try:
            e.upload(m)
            nodes, ptr = e.train(p, y, 4, H.base_margin(p, y))
            runs.append((nodes, ptr, e.read_margins()))
        finally:
            e.close()
    assert_forest_equal(runs[0][0], runs[0][1], runs[1][0], runs[1][1], f"lossguide {layout}")
    np.testing.assert_array_equal(_bits(runs[0][2]), _bits(runs[1][2]))


def test_engine_reused_across_uploads_of_one_shape():
    """An engine keeps its captured round graph across uploads of the same
    shape (the graph's key holds the index's constants and buffers): a
    second matrix of the same shape, with other values, cuts and labels,
    grows the forest a fresh engine grows; a matrix of another bin count
    too (its graph is captured again)."""
    p = H.TrainingParams(objective="binary:logistic", max_depth=6, eta=0.3)
    mats = []
    for seed, max_bin in ((71, 256), (72, 256), (73, 64)):
        x, y = synth.logistic_c2(60_013, 28, seed=seed)
        mats.append((H.BinnedMatrix.from_dense(x, max_bin), y))
    eng = H.Engine()
    try:
        for m, y in mats:
            got = H.train(p, y=y, rounds=3, matrix=m, engine=eng)
            want = H.train(p, y=y, rounds=3, matrix=m)
            assert_forest_equal(got.nodes, got.tree_ptr, want.nodes, want.tree_ptr, "reused engine")
    finally:
        eng.close()


@pytest.mark.parametrize("max_bin", [16, 48, 128])
def test_scan_kernels_agree(monkeypatch, max_bin):
    """The warp-per-feature split scan (features of <= 128 bins) and the
    CTA-per-feature one pick the same splits, depthwise and lossguide, with
    missing values (both directions scored)."""
    x, y = synth.logistic_c2(50_021, 20, seed=max_bin, missing=0.1)
    m = H.BinnedMatrix.from_dense(x, max_bin)
    runs = []
    for kernel in ("warp", "cta"):
        monkeypatch.setenv("HB_SCAN_KERNEL", kernel)
        for policy in ("depthwise", "lossguide"):
            p = H.TrainingParams(objective="binary:logistic", max_depth=6, max_bin=max_bin, grow_policy=policy,
                                 max_leaves=40 if policy == "lossguide" else 0)
            runs.append(H.train(p, y=y, rounds=2, matrix=m))
    for a, b in ((0, 2), (1, 3)):
        assert_forest_equal(runs[a].nodes, runs[a].tree_ptr, runs[b].nodes, runs[b].tree_ptr, "warp vs cta")


@pytest.mark.parametrize("case", ["c2_logistic", "c2_large", "regularised", "monotone_depthwise", "c1_regression"])
def test_row_engine_rounds_equal_whole_round_path(case):
    """The reference's unchanged device round (device_round +
    build_on_device, restated over the RowEngine calls in
    hessboost_b200.device_builder) grows the same trees, bit for bit, as
    hb_train_rounds, and leaves the same margins."""
    from hessboost_b200.device_builder import RowEngineTrainer

    spec = CASES[case]
    x, y = spec["gen"]()
    params = H.TrainingParams(**spec["kw"])
    mtx = H.BinnedMatrix.from_dense(x, params.max_bin)
    base = H.base_margin(params, y)
    e = H.Engine()
    try:
        e.upload(mtx)
        e.train_begin(y, base)
        want_nodes, want_ptr = e.train_rounds(params, spec["rounds"])
        want_margins = e.read_margins()
        e.load_margins(np.full(mtx.n_rows, base, np.float32))
        tr = RowEngineTrainer(e, params, y)
        got = [tr.round() for _ in range(spec["rounds"])]
        got_margins = e.read_margins()
    finally:
        e.close()
    ptr = np.concatenate([[0], np.cumsum([len(t) for t in got])]).astype(np.uint64)
    assert_forest_equal(np.concatenate(got), ptr, want_nodes, want_ptr, case)
    np.testing.assert_array_equal(_bits(got_margins), _bits(want_margins))
