"""The CSR index on the device (through the C ABI) against the CPU oracle.

The oracle trains on the dense matrix holding NaN in every absent cell: the
reference's CSR and dense paths share cuts (quantile.rs:199 vs sketch.rs:541)
and bins, and with exact fixed-point sums the same trees. So the CSR path
must give the oracle's fixed-point trees, leaf values and training margins
bit for bit, and the same histograms and partitions as a dense engine."""

import numpy as np
import pytest

import hessboost_b200 as H
import oracle_lib as O
from hessboost_b200 import synth

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _assert_forest_equal(nodes, ptr, onodes, optr, what=""):
    np.testing.assert_array_equal(np.asarray(ptr, np.uint64), np.asarray(optr, np.uint64), err_msg=what)
    for k in ("left", "right", "split_feature", "default_left", "split_bin"):
        np.testing.assert_array_equal(nodes[k], onodes[k], err_msg=f"{what} {k}")
    for k in ("split_cond", "leaf_value", "sum_hess", "split_gain"):
        np.testing.assert_array_equal(_bits(nodes[k]), _bits(onodes[k]), err_msg=f"{what} {k}")


def _labels(indptr, indices, values, n_cols, seed, kind):
    rng = np.random.default_rng(seed)
    x = synth.csr_to_dense(indptr, indices, values, n_cols)
    z = np.nan_to_num(x[:, : min(n_cols, 12)], nan=0.0) @ rng.standard_normal(min(n_cols, 12))
    if kind == "logistic":
        return x, (rng.random(len(z)) < 1 / (1 + np.exp(-z))).astype(np.float32)
    if kind == "softmax":
        return x, (np.digitize(z, np.quantile(z, [0.33, 0.66]))).astype(np.float32)
    return x, (z + rng.standard_normal(len(z)) * 0.1).astype(np.float32)


def _csr(n, f, density, seed):
    return synth.sparse_c4(n, f, density=density, seed=seed)[:3]


CASES = {
    # depthwise over a sparse index, missing everywhere
    "depthwise_logistic": dict(n=20_011, f=40, density=0.15, rounds=3, max_bin=256, label="logistic",
                               kw=dict(objective="binary:logistic", max_depth=6, eta=0.3)),
    # lossguide (the C4 growth) with 64-bin features
    "lossguide_regression": dict(n=15_000, f=30, density=0.3, rounds=3, max_bin=64, label="regression",
                                 kw=dict(grow_policy="lossguide", max_depth=0, max_leaves=40)),
    # many features: 700 x 64 bins, beyond every dense layout
    "wide": dict(n=8_000, f=700, density=0.03, rounds=2, max_bin=64, label="logistic",
                 kw=dict(objective="binary:logistic", grow_policy="lossguide", max_depth=0, max_leaves=31)),
    # a CSR matrix listing every cell (dense_equals_sparse, tests/properties.rs:55)
    "full_rows": dict(n=3_000, f=6, density=1.0, rounds=3, max_bin=256, label="regression",
                      kw=dict(max_depth=4)),
    # multi:softmax over CSR rows
    "softmax": dict(n=9_000, f=20, density=0.4, rounds=2, max_bin=128, label="softmax",
                    kw=dict(objective="multi:softmax", num_class=3, max_depth=4, eta=0.2)),
}


def _orc_kw(kw):
    m = dict(kw)
    obj = m.pop("objective", "reg:squarederror")
    m["objective"] = {"binary:logistic": 1, "multi:softmax": 2}.get(obj, 0)
    if obj == "multi:softmax":
        m["n_outputs"] = m.pop("num_class")
    if "grow_policy" in m:
        m["grow_policy"] = 1 if m["grow_policy"] == "lossguide" else 0
    return m


@pytest.fixture(params=["1", "0"], ids=["columns", "search"])
def csr_columns(request, monkeypatch):
    """Both ways a CSR engine reads a row's split cell: the feature-major
    copy of the index (default) and the binary search of the row's bins
    (HB_CSR_COLUMNS=0)."""
    monkeypatch.setenv("HB_CSR_COLUMNS", request.param)
    return request.param


@pytest.mark.parametrize("case", sorted(CASES))
def test_csr_training_matches_oracle(case, csr_columns):
    s = CASES[case]
    indptr, indices, values = _csr(s["n"], s["f"], s["density"], seed=len(case))
    x, y = _labels(indptr, indices, values, s["f"], 7, s["label"])
    m = H.BinnedMatrix.from_csr(indptr, indices, values, s["f"], s["max_bin"])
    params = H.TrainingParams(max_bin=s["max_bin"], **s["kw"])
    model = H.train(params, y=y, rounds=s["rounds"], matrix=m)
    on, op, ob, omarg = O.train(x, y, s["rounds"], fixed_point=True, max_bin=s["max_bin"], **_orc_kw(s["kw"]))
    np.testing.assert_array_equal(_bits(model.bases()), _bits(ob))
    _assert_forest_equal(model.nodes, model.tree_ptr, on, op, case)
    got = model.predict_margin(x).reshape(len(y), -1)
    np.testing.assert_array_equal(_bits(got), _bits(omarg.reshape(len(y), -1)))


def test_csr_engine_matches_dense_engine(csr_columns):
    """Histograms, root totals, partitions (absent = missing) and the
    no-allocation entry of a CSR engine equal a dense engine's on the same
    cells."""
    torch = pytest.importorskip("torch")
    indptr, indices, values = _csr(6_007, 9, 0.4, seed=5)
    x = synth.csr_to_dense(indptr, indices, values, 9)
    rng = np.random.default_rng(3)
    y = (rng.random(len(x)) < 0.4).astype(np.float32)
    marg = (rng.standard_normal(len(x)) * 0.5).astype(np.float32)
    dense = H.BinnedMatrix.from_dense(x)
    csr = H.BinnedMatrix.from_csr(indptr, indices, values, 9)
    np.testing.assert_array_equal(csr.cut_values.view(np.uint32), dense.cut_values.view(np.uint32))
    out = {}
    for name, mtx in (("dense", dense), ("csr", csr)):
        e = H.Engine()
        try:
            e.upload(mtx)
            e.load_margins(marg)
            assert e.gradients(H.HB_LOSS_LOGISTIC, y)
            n = len(x)
            sub = np.sort(rng.choice(n, n // 3, replace=False)) if name == "dense" else out["sub"]
            out["sub"] = sub
            root = e.begin_tree(np.arange(n))
            tot = e.root_total(root)
            hist = e.histograms([root])[0]
            part = e.build(sub)
            (left, right), = e.partition([(root, 4, 7, False)])
            lrows, rrows = e.rows([left, right])
            (ll, lr), = e.partition([(left, 1, 20, True)])
            llrows, = e.rows([ll])
            rows_dev = torch.from_numpy(sub.astype(np.int32)).cuda()
            buf = torch.zeros((mtx.total_bins, 2), dtype=torch.float64, device="cuda:0")
            torch.cuda.synchronize()
            e.build_noalloc(rows_dev.data_ptr(), sub.size, buf.data_ptr())
            out[name] = (tot, hist, part, lrows, rrows, llrows, buf.cpu().numpy())
        finally:
            e.close()
    for a, b in zip(out["dense"], out["csr"]):
        np.testing.assert_array_equal(np.asarray(a), np.asarray(b))
    # the partition's rule on absent cells: feature 4 missing goes right here
    miss = np.isnan(x[:, 4])
    assert not np.any(miss[out["csr"][3]])


def test_csr_c4_shape_lossguide(csr_columns):
    """The C4 shape at test size: 60,000 rows x 2,000 features at 2% density,
    64 bins, lossguide with 255 leaves; the oracle trains on its own CSR index
    (stored cells only). Trees, and the training margins read back from the
    device, bit for bit."""
    indptr, indices, values, y = synth.sparse_c4(60_000, 2000, seed=11)
    m = H.BinnedMatrix.from_csr(indptr, indices, values, 2000, 64)
    kw = dict(objective="binary:logistic", grow_policy="lossguide", max_depth=0, max_leaves=255, eta=0.3)
    params = H.TrainingParams(max_bin=64, **kw)
    e = H.Engine()
    try:
        e.upload(m)
        base = H.base_margin(params, y)
        nodes, ptr = e.train(params, y, 3, base)
        marg = e.read_margins()
    finally:
        e.close()
    on, op, ob, omarg = O.train_csr(indptr, indices, values, 2000, y, 3, fixed_point=True, max_bin=64, **_orc_kw(kw))
    assert np.float32(base).view(np.uint32) == ob.view(np.uint32)[0]
    _assert_forest_equal(nodes, ptr, on, op, "c4")
    np.testing.assert_array_equal(_bits(marg), _bits(omarg[:, 0]))
