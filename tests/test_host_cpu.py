"""CPU-side checks of the product library: it loads without a GPU, exports
every entry point the header declares, refuses a device that is not there,
and its host binning (cuts + bins) equals the oracle's bit for bit."""

import ctypes
import math
import os
import re

import numpy as np
import pytest

import hessboost_b200 as H
import oracle_lib as O

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "hb_backend.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^(?:hb_status|const char\*)\s+(hb_\w+)\(", text, flags=re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    L = H.lib()
    names = declared_symbols()
    assert len(names) >= 30
    for name in names:
        assert hasattr(L, name), name
        assert name in H.SIGNATURES, f"{name} has no ctypes signature"
    assert set(H.SIGNATURES) == set(names)


def test_header_structs_match_bindings():
    assert ctypes.sizeof(H.TreeNode) == 40
    assert ctypes.sizeof(H.Segment) == 32
    assert ctypes.sizeof(H.GHist) == 64
    assert ctypes.sizeof(H.NodeScan) == 40


def _has_gpu():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        return False


@pytest.mark.skipif(_has_gpu(), reason="checks the no-device refusal")
def test_engine_create_refuses_without_device():
    h = ctypes.c_void_p()
    st = H.lib().hb_engine_create(0, ctypes.byref(h))
    assert st == H.HB_REFUSED
    assert not h.value


def test_invalid_arguments():
    assert H.lib().hb_engine_create(0, None) == H.HB_INVALID_ARGUMENT
    assert H.lib().hb_engine_destroy(None) == H.HB_INVALID_ARGUMENT
    assert H.lib().hb_cuts_dense(None, 0, 0, 0, None, None, 0, None) == H.HB_INVALID_ARGUMENT


def _datasets():
    rng = np.random.default_rng(7)
    yield "normal_nan", rng.standard_normal((5000, 6)).astype(np.float32), 0.05, 256
    yield "repeats", rng.integers(0, 40, (7000, 3)).astype(np.float32), 0.0, 256
    yield "few_bins", rng.standard_normal((3000, 4)).astype(np.float32), 0.1, 16
    yield "large_queue", rng.standard_normal((120_000, 2)).astype(np.float32), 0.02, 256
    yield "signed_zero", np.array([[0.0], [-0.0], [1.0], [-1.0], [0.0]] * 50, np.float32), 0.0, 256
    yield "one_row", np.array([[1.5, np.nan]], np.float32), 0.0, 256
    yield "all_missing", np.full((10, 2), np.nan, np.float32), 0.0, 256


@pytest.mark.parametrize("name,x,missing,max_bin", list(_datasets()), ids=[d[0] for d in _datasets()])
def test_cuts_and_bins_match_oracle(name, x, missing, max_bin):
    x = x.copy()
    if missing:
        x[np.random.default_rng(1).random(x.shape) < missing] = np.nan
    off_h, cuts_h = H.cuts_dense(x, max_bin)
    off_o, cuts_o = O.cuts_dense(x, max_bin)
    np.testing.assert_array_equal(off_h, off_o)
    np.testing.assert_array_equal(cuts_h.view(np.uint32), cuts_o.view(np.uint32))
    if np.max(np.diff(off_h)) <= 256:
        cols, miss, dense = H.bin_dense(x, off_h, cuts_h)
        cols_o, miss_o, dense_o = O.bin_dense(x, off_o, cuts_o)
        np.testing.assert_array_equal(cols.astype(np.uint16), cols_o)
        np.testing.assert_array_equal(miss, miss_o)
        assert dense == dense_o


def test_base_margin_matches_oracle():
    rng = np.random.default_rng(2)
    y = (rng.random(12345) < 0.3).astype(np.float32)
    out = np.zeros(1, np.float32)
    O.lib().orc_intercepts(1, O._p(y, ctypes.c_float), y.size, 1, O._p(out, ctypes.c_float))
    got = H.base_margin(H.TrainingParams(objective="binary:logistic"), y)
    assert np.float32(got).view(np.uint32) == out.view(np.uint32)[0]
    y2 = rng.standard_normal(999).astype(np.float32)
    O.lib().orc_intercepts(0, O._p(y2, ctypes.c_float), y2.size, 1, O._p(out, ctypes.c_float))
    got = H.base_margin(H.TrainingParams(), y2)
    assert np.float32(got).view(np.uint32) == out.view(np.uint32)[0]


def test_shard_split_keeps_bins_and_bitmap():
    rng = np.random.default_rng(4)
    x = rng.standard_normal((1000, 5)).astype(np.float32)
    x[rng.random(x.shape) < 0.1] = np.nan
    m = H.BinnedMatrix.from_dense(x)
    a, b = m.shard(0, 496), m.shard(496, 1000)
    np.testing.assert_array_equal(np.concatenate([a.columns, b.columns], axis=1), m.columns)
    for part, lo in ((a, 0), (b, 496)):
        bits = np.unpackbits(part.missing.view(np.uint8), bitorder="little").reshape(5, -1)[:, : part.n_rows]
        np.testing.assert_array_equal(bits.astype(bool), np.isnan(x[lo : lo + part.n_rows].T))


def test_softmax_intercepts_match_oracle():
    rng = np.random.default_rng(6)
    for n, k in ((1000, 3), (12345, 10), (7, 5)):
        y = rng.integers(0, k, n).astype(np.float32)
        np.testing.assert_array_equal(H.softmax_intercepts(y, k).view(np.uint32),
                                      O.intercepts(2, y, k).view(np.uint32))


def test_rust_ffi_module_binds_every_entry_point():
    # the Rust `extern "C"` module a maintainer would add declares exactly the
    # header's entry points
    src = open(os.path.join(os.path.dirname(HEADER), "hb_backend_ffi.rs")).read()
    assert sorted(set(re.findall(r"pub fn (hb_\w+)\(", src))) == declared_symbols()


@pytest.mark.parametrize("bad,name", [
    (dict(eta=0.0), "eta"), (dict(eta=float("nan")), "eta"), (dict(eta=1e-50), "eta"),
    (dict(gamma=-1.0), "gamma"), (dict(min_child_weight=float("inf")), "min_child_weight"),
    (dict(reg_lambda=-0.5), "reg_lambda"), (dict(alpha=1e300), "alpha"),
    (dict(max_delta_step=-1.0), "max_delta_step"), (dict(scale_pos_weight=0.0), "scale_pos_weight"),
    (dict(max_bin=1), "max_bin"), (dict(max_depth=-1), "max_depth"),
    (dict(grow_policy="lossguide", max_depth=0, max_leaves=0), "max_leaves"),
    (dict(grow_policy="symmetric"), "grow_policy"),
])
def test_training_params_validate_like_the_reference(bad, name):
    # TrainingParams::validate (src/config/params.rs:906-918, :1036): the
    # first failing parameter is named
    with pytest.raises(ValueError, match=f"`{name}`"):
        H.TrainingParams(**bad).validate()


def test_training_params_defaults_and_config_shapes_are_valid():
    H.TrainingParams().validate()
    H.TrainingParams(objective="binary:logistic", max_depth=8, eta=0.1).validate()
    H.TrainingParams(objective="multi:softmax", num_class=10, max_depth=6, eta=0.2, max_bin=128).validate()
    H.TrainingParams(grow_policy="lossguide", max_depth=0, max_leaves=255, max_bin=64).validate()
    H.TrainingParams(max_depth=5, reg_lambda=3.0, alpha=0.5, gamma=0.2, min_child_weight=20.0,
                     max_delta_step=0.7).validate()
    H.TrainingParams(max_bin=2, min_child_weight=0.0, reg_lambda=0.0).validate()
