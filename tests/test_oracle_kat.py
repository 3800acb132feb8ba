"""The CPU oracle against the reference's own known-answer fixtures.

The saved models under ``tests/golden/`` were written by hessboost 0.4.9's
``tests/native_format.rs`` (see ``make_golden.py``).  Two of them are full
training runs of the hist path on the 160 x 4 probe; every one of them pins
prediction.  The oracle must reproduce them bit for bit, in the reference's
f64 summation and in the int64 fixed-point summation the CUDA path uses.
"""

import numpy as np
import pytest

import oracle_lib as O

TRAIN_KATS = [("early_stopping", "y1"), ("multi_target", "y2")]


def _model(g, name):
    return [m for m in g["models"] if m["name"] == name][-1]


def _assert_trees_equal(nodes, ptr, gnodes, gptr):
    assert len(ptr) == len(gptr)
    for t in range(len(gptr) - 1):
        a = nodes[int(ptr[t]) : int(ptr[t + 1])]
        b = gnodes[int(gptr[t]) : int(gptr[t + 1])]
        assert len(a) == len(b), f"tree {t}: {len(a)} vs {len(b)} nodes"
        for k in ("left", "right", "split_feature", "default_left"):
            np.testing.assert_array_equal(a[k], b[k], err_msg=f"tree {t} {k}")
        for k in ("split_cond", "leaf_value", "sum_hess", "split_gain"):
            np.testing.assert_array_equal(O.f32_to_bits(a[k]), O.f32_to_bits(b[k]), err_msg=f"tree {t} {k}")


@pytest.mark.parametrize("fixed", [False, True], ids=["f64", "fixed_point"])
@pytest.mark.parametrize("name,ykey", TRAIN_KATS)
def test_training_kat_bit_exact(name, ykey, fixed):
    g = O.golden()
    m = _model(g, name)
    nodes, ptr, base, margins = O.train(g["x"], g[ykey], 4, max_depth=3, eta=0.3, fixed_point=fixed)
    np.testing.assert_array_equal(O.f32_to_bits(base), O.f32_to_bits(np.array(m["base_score"], np.float32)))
    gnodes, gptr = O.golden_nodes(m)
    _assert_trees_equal(nodes, ptr, gnodes, gptr)


def test_prediction_kats_bit_exact():
    g = O.golden()
    assert len(g["models"]) >= 9
    for m in g["models"]:
        nodes, ptr = O.golden_nodes(m)
        n, outs, w = O.golden_layout(m)
        got = O.predict(nodes, ptr[: n + 1], m["n_outputs"], np.array(m["base_score"], np.float32), g["x"], outs, w)
        np.testing.assert_array_equal(O.f32_to_bits(got).ravel(), np.array(m["margins_bits"], np.uint32), err_msg=m["name"])


def test_sketch_known_answers():
    # src/data/sketch.rs:876-895: the minimum is never a cut, a sentinel
    # closes the last bin, an empty feature gets the upstream placeholder.
    off, cuts = O.cuts_dense(np.array([[2.0], [0.0], [1.0], [1.0]], np.float32), 256)
    np.testing.assert_array_equal(cuts, np.array([1.0, 2.0, np.float32(2.0) + (np.float32(2.0) + np.float32(1e-5))], np.float32))
    off, cuts = O.cuts_dense(np.full((3, 1), np.nan, np.float32), 256)
    np.testing.assert_array_equal(cuts, np.array([1e-5], np.float32))
    vals = ((np.arange(5000) * 7919) % 5000).astype(np.float32) * np.float32(0.001)
    off, cuts = O.cuts_dense(vals.reshape(-1, 1), 64)
    assert len(cuts) <= 64 and np.all(np.diff(cuts) > 0) and cuts[-1] > 4.999


def test_gain_closed_forms():
    # src/tree/gain.rs:155-196 style closed form through a one-split tree:
    # two rows, g = (-1, +1), h = 1, lambda = 1 -> leaves -(-1)/(1+1) * eta.
    x = np.array([[0.0], [1.0]], np.float32)
    y = np.array([1.0, -1.0], np.float32)  # base = 0 -> g = 0 - y
    nodes, ptr, base, _ = O.train(x, y, 1, max_depth=1, eta=1.0, min_child_weight=0.0)
    assert base[0] == 0.0
    leaves = nodes[nodes["left"] == -1]["leaf_value"]
    np.testing.assert_array_equal(np.sort(leaves), np.array([-0.5, 0.5], np.float32))


def test_logistic_gradient_closed_form():
    # classification.rs:251-290: p = sigmoid(m), g = p - y, h = p(1-p).
    m = np.linspace(-6, 6, 1003).astype(np.float32)
    y = (np.arange(1003) % 2).astype(np.float32)
    gp = O.gradients(1, m, y)
    p = 1.0 / (1.0 + np.exp(-m.astype(np.float64)))
    np.testing.assert_allclose(gp[:, 0], p - y, rtol=0, atol=2e-7)
    np.testing.assert_allclose(gp[:, 1], p * (1 - p), rtol=1e-4, atol=2e-7)


def test_fixed_scale_bounds():
    for max_abs in [1e-30, 0.25, 0.9999, 1.0, 3.5, 1e20]:
        for n in [1, 2, 3, 160, 10_000_000]:
            s = O.fixed_scale(max_abs, n)
            q = np.rint(np.float64(np.float32(max_abs)) * 2.0 ** s)
            assert q * n <= 2.0 ** 62
    assert O.fixed_scale(0.0, 10) == 0


@pytest.mark.parametrize("missing", [False, True])
def test_fixed_point_matches_f64_structure(missing):
    # On data whose f64 sums are exact, the two summation modes agree.
    rng = np.random.default_rng(3)
    x = rng.integers(0, 50, size=(3000, 6)).astype(np.float32)
    if missing:
        x[rng.random(x.shape) < 0.05] = np.nan
    y = (np.nan_to_num(x[:, 0]) * 0.5 - np.nan_to_num(x[:, 1]) * 0.25).astype(np.float32)
    a = O.train(x, y, 3, max_depth=4, eta=0.5)
    b = O.train(x, y, 3, max_depth=4, eta=0.5, fixed_point=True)
    _assert_trees_equal(a[0], a[1], b[0], b[1])


# ------------------------------------------------------------ multi:softmax
def test_softmax_gradient_kat():
    """objective/multiclass.rs:124 `gradient_layout_and_values`: all margins
    0 over 3 classes -> p = 1/3, g = p - [class == label], h = 2 p (1 - p)."""
    g = O.softmax_gradients(np.zeros((2, 3), np.float32), np.array([0.0, 2.0], np.float32))
    np.testing.assert_allclose(g[0, 0, 0], 1 / 3 - 1, atol=1e-6)
    np.testing.assert_allclose(g[0, 1, 0], 1 / 3, atol=1e-6)
    np.testing.assert_allclose(g[1, 2, 0], 1 / 3 - 1, atol=1e-6)
    np.testing.assert_allclose(g[:, :, 1], 2 * (1 / 3) * (2 / 3), atol=1e-6)


def _softmax_scalar(m, y):
    """simd/mod.rs:580 `softmax_gradient_row_scalar` in numpy (exp in f64
    rounded to f32, within an ulp of expf): the comparison kernel of the
    reference's own vector-softmax tests (simd/tests.rs:33)."""
    n, k = m.shape
    out = np.zeros((n, k, 2), np.float32)
    tiny = np.float32(np.finfo(np.float32).tiny)
    with np.errstate(all="ignore"):
        for i in range(n):
            row = m[i]
            wmax = tiny
            for v in row:
                wmax = np.float32(np.fmax(v, wmax))
            e = [np.float32(np.exp(np.float64(np.float32(v - wmax)))) for v in row]
            ws = np.float32(sum(np.float64(v) for v in e))
            for j in range(k):
                p = np.float32(e[j] / ws)
                h = np.float32(np.fmax(np.float32(np.float32(2 * p) * np.float32(1 - p)), np.float32(1e-16)))
                out[i, j] = (np.float32(p - 1) if j == int(y[i]) else p, h)
    return out


@pytest.mark.parametrize("k", [2, 3, 4])
def test_short_softmax_batches_match_scalar_across_boundaries(k):
    """simd/tests.rs:133: 2 and 4 classes run x86_64's short-row vector
    kernel (whole rows per 8-lane vector, the rest scalar), 3 the scalar
    one; every row count around the batch and MIN_SIMD_LEN boundaries stays
    within 1e-6 of the scalar kernel."""
    for rows in list(range(1, 18)) + [127, 256, 257]:
        m = (((np.arange(rows * k) * 71) % 211).astype(np.float32) * np.float32(0.375)
             - np.float32(39.0)).reshape(rows, k)
        y = (np.arange(rows) % k).astype(np.float32)
        got = O.softmax_gradients(m, y)
        want = _softmax_scalar(m, y)
        assert np.all(np.abs(got - want) <= 1e-6 * np.maximum(np.abs(want), 1.0)), (k, rows)


@pytest.mark.parametrize("k", [2, 4])
def test_short_softmax_exceptional_rows_match_scalar(k):
    """simd/tests.rs:164 with class-id labels (the engine refuses others): a
    non-finite, wide (|m| > 80) or huge margin anywhere sends its vector to
    the scalar path, so NaN, infinities and values agree with the scalar
    kernel (values within 3e-7)."""
    rows = 9
    y = (np.arange(rows) % k).astype(np.float32)
    for position in range(rows * k):
        for exc in (np.nan, np.inf, -np.inf, -81.0, 81.0, -80.0, 80.0, np.finfo(np.float32).max):
            m = np.zeros(rows * k, np.float32)
            m[position] = exc
            m = m.reshape(rows, k)
            got = O.softmax_gradients(m, y)
            want = _softmax_scalar(m, y)
            assert np.array_equal(np.isnan(got), np.isnan(want)), (position, exc)
            fin = np.isfinite(want)
            assert np.array_equal(got[~fin & ~np.isnan(want)], want[~fin & ~np.isnan(want)])
            assert np.all(np.abs(got[fin] - want[fin]) <= 3e-7), (position, exc)


@pytest.mark.parametrize("k", [2, 4])
def test_short_softmax_vector_rows(k):
    """The vector kernel really runs for 2 and 4 classes: at 16 or more
    margins its rows differ from the scalar kernel's in the last bits
    somewhere (exp_f32's polynomial, p = e * (1 / sum)), while below
    MIN_SIMD_LEN (simd/mod.rs:28) every row is the scalar kernel's; a vector
    holding one irregular row computes all of its rows as the scalar
    kernel does, which the same rows reproduce as a tail."""
    rng = np.random.default_rng(k)
    m = (rng.standard_normal((4096, k)) * 3).astype(np.float32)
    y = rng.integers(0, k, 4096).astype(np.float32)
    vec = O.softmax_gradients(m, y)
    assert not np.array_equal(vec, _softmax_scalar(m, y))
    rpb = 8 // k
    small = 16 // k - 1  # n * k < 16: the whole batch scalar
    forced = m[:64].copy()
    forced[rpb - 1, 0] = np.nan  # the first vector's rows on the scalar path
    np.testing.assert_array_equal(O.softmax_gradients(m[:small], y[:small])[: rpb - 1],
                                  O.softmax_gradients(forced, y[:64])[: rpb - 1])
    tail = O.softmax_gradients(m[: 16 + rpb - 1], y[: 16 + rpb - 1])[16:]  # rows past the last whole vector
    wide = m[: 16 + rpb].copy()
    wide[16 + rpb - 1, 0] = np.inf  # the vector of rows 16.. holds an irregular row
    mixed = O.softmax_gradients(wide, y[: 16 + rpb])[16: 16 + rpb - 1]
    np.testing.assert_array_equal(mixed, tail)
    regular = O.softmax_gradients(m[: 16 + rpb], y[: 16 + rpb])[16: 16 + rpb - 1]
    assert np.all(np.abs(regular - tail) <= 1e-6)


def test_softmax_gradient_shift_and_rounding():
    """The shift is max(f32::MIN_POSITIVE, margins) and the f64 sum is
    rounded to f32 before the division (simd/mod.rs:580)."""
    rng = np.random.default_rng(2)
    m = (rng.standard_normal((50, 7)) * 3).astype(np.float32)
    m[0] = -5.0  # every margin negative: the shift stays f32::MIN_POSITIVE
    y = rng.integers(0, 7, 50).astype(np.float32)
    got = O.softmax_gradients(m, y)
    tiny = np.float32(np.finfo(np.float32).tiny)
    for i in range(50):
        wmax = max(np.float32(np.max(m[i])), tiny)
        e = [np.float32(np.exp(np.float64(np.float32(v - wmax)))) for v in m[i]]
        ws = np.float32(sum(np.float64(v) for v in e))
        for j in range(7):
            p = np.float32(e[j] / ws)
            np.testing.assert_allclose(got[i, j, 0], p - (1.0 if j == y[i] else 0.0), rtol=2e-6, atol=1e-7)
            np.testing.assert_allclose(got[i, j, 1], max(np.float32(2 * p * (1 - p)), np.float32(1e-16)), rtol=2e-6)


def test_softmax_intercepts_kat():
    """objective/multiclass.rs:146: centred log class frequencies."""
    m = O.intercepts(2, np.array([0.0, 0.0, 1.0, 2.0], np.float32), 3)
    assert abs(float(m.sum())) < 1e-6
    gap = np.log(np.float32(0.5) + np.float32(1e-6)) - np.log(np.float32(0.25) + np.float32(1e-6))
    assert abs(float(m[0] - m[1]) - gap) < 1e-6
    assert m[1] == m[2]


def test_softmax_training_fixed_matches_f64_structure():
    rng = np.random.default_rng(5)
    x = rng.uniform(-1, 1, (3000, 8)).astype(np.float32)
    w = rng.standard_normal((8, 4))
    y = np.argmax(x @ w + rng.gumbel(size=(3000, 4)), axis=1).astype(np.float32)
    kw = dict(objective=2, n_outputs=4, max_depth=4, eta=0.2, max_bin=64)
    a = O.train(x, y, 3, **kw)
    b = O.train(x, y, 3, fixed_point=True, **kw)
    assert len(a[1]) == len(b[1]) == 13  # 3 rounds x 4 classes
    for key in ("left", "right", "split_feature", "split_bin", "default_left"):
        np.testing.assert_array_equal(a[0][key], b[0][key])
    np.testing.assert_allclose(a[0]["leaf_value"], b[0]["leaf_value"], rtol=1e-5, atol=1e-7)
    np.testing.assert_array_equal(a[2], b[2])
    np.testing.assert_array_equal(a[2], O.intercepts(2, y, 4))


def _step_dataset(n):
    """training/train/tests.rs:22 `step_dataset`: x = i / n, y = [x >= 0.5]."""
    x = (np.arange(n, dtype=np.float32) / np.float32(n)).reshape(n, 1)
    return x, (x[:, 0] >= 0.5).astype(np.float32)


@pytest.mark.parametrize("fixed", [False, True], ids=["f64", "fixed_point"])
def test_lossguide_trains_end_to_end(fixed):
    """training/train/tests.rs:218 `lossguide_trains_end_to_end`: squared
    error, lossguide, max_leaves 16, eta 0.3, 60 rounds on the 120-row step
    set; RMSE below 0.06, and no tree above 16 leaves."""
    x, y = _step_dataset(120)
    nodes, ptr, base, margins = O.train(x, y, 60, grow_policy=1, max_leaves=16, eta=0.3,
                                        fixed_point=fixed)
    rmse = float(np.sqrt(np.mean((margins[:, 0].astype(np.float64) - y) ** 2)))
    assert rmse < 0.06, rmse
    sizes = np.diff(np.asarray(ptr, np.int64))
    assert sizes.max() <= 31 and sizes.min() >= 1


def test_lossguide_fixed_matches_f64_structure():
    """The fixed-point summation grows the same lossguide trees as f64 (no
    exact-gain ties on this set), leaves within 1e-5 relative."""
    rng = np.random.default_rng(4)
    x = rng.standard_normal((3000, 6)).astype(np.float32)
    y = (x[:, 0] * 2 + np.sin(x[:, 1] * 3) + 0.1 * rng.standard_normal(3000)).astype(np.float32)
    a = O.train(x, y, 3, grow_policy=1, max_leaves=20, max_depth=0, fixed_point=False)
    b = O.train(x, y, 3, grow_policy=1, max_leaves=20, max_depth=0, fixed_point=True)
    np.testing.assert_array_equal(a[1], b[1])
    for k in ("left", "right", "split_feature", "default_left", "split_bin"):
        np.testing.assert_array_equal(a[0][k], b[0][k], err_msg=k)
    np.testing.assert_allclose(a[0]["leaf_value"], b[0]["leaf_value"], rtol=1e-5, atol=1e-7)
