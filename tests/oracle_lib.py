"""ctypes wrapper of the CPU oracle (``oracle/_build/liboracle.so``).

Test infrastructure: the oracle restates the reference's CPU hist path and is
the checker the CUDA path is compared against.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline`` leg load it.
"""

import ctypes
import json
import os
import struct
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(ROOT, "oracle")
LIB_PATH = os.path.join(ORACLE_DIR, "_build", "liboracle.so")
GOLDEN = os.path.join(ROOT, "tests", "golden", "saved_models.json")


class OrcNode(ctypes.Structure):
    _fields_ = [
        ("left", ctypes.c_int32),
        ("right", ctypes.c_int32),
        ("split_feature", ctypes.c_uint32),
        ("split_cond", ctypes.c_float),
        ("default_left", ctypes.c_uint32),
        ("leaf_value", ctypes.c_float),
        ("sum_hess", ctypes.c_float),
        ("split_gain", ctypes.c_float),
        ("split_bin", ctypes.c_int32),
        ("reserved", ctypes.c_uint32),
    ]


NODE_DTYPE = np.dtype(
    [
        ("left", "<i4"),
        ("right", "<i4"),
        ("split_feature", "<u4"),
        ("split_cond", "<f4"),
        ("default_left", "<u4"),
        ("leaf_value", "<f4"),
        ("sum_hess", "<f4"),
        ("split_gain", "<f4"),
        ("split_bin", "<i4"),
        ("reserved", "<u4"),
    ]
)
assert NODE_DTYPE.itemsize == ctypes.sizeof(OrcNode) == 40


class OrcParams(ctypes.Structure):
    _fields_ = [
        ("objective", ctypes.c_int32),
        ("n_outputs", ctypes.c_int32),
        ("max_depth", ctypes.c_int32),
        ("max_leaves", ctypes.c_int32),
        ("grow_policy", ctypes.c_int32),
        ("max_bin", ctypes.c_int32),
        ("eta", ctypes.c_float),
        ("lambda_", ctypes.c_float),
        ("alpha", ctypes.c_float),
        ("gamma", ctypes.c_float),
        ("min_child_weight", ctypes.c_float),
        ("max_delta_step", ctypes.c_float),
        ("scale_pos_weight", ctypes.c_float),
        ("base_score", ctypes.c_float),
        ("fixed_point", ctypes.c_int32),
        ("n_threads", ctypes.c_int32),
        ("monotone", ctypes.POINTER(ctypes.c_int8)),
        ("n_monotone", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class OrcScan(ctypes.Structure):
    _fields_ = [
        ("found", ctypes.c_int32),
        ("feature", ctypes.c_uint32),
        ("bin", ctypes.c_int32),
        ("default_left", ctypes.c_uint32),
        ("loss_chg", ctypes.c_float),
        ("root_gain", ctypes.c_float),
        ("left_g", ctypes.c_int64),
        ("left_h", ctypes.c_int64),
        ("w_left", ctypes.c_float),
        ("w_right", ctypes.c_float),
    ]


_lib = None


def build():
    """Compile the oracle with its committed Makefile (no reference sources)."""
    subprocess.run(["make", "-s", "-C", ORACLE_DIR], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.POINTER
        f32p, u32p, u64p = P(ctypes.c_float), P(ctypes.c_uint32), P(ctypes.c_uint64)
        L.orc_cuts_dense.restype = ctypes.c_int64
        L.orc_cuts_dense.argtypes = [f32p, ctypes.c_uint64, ctypes.c_uint64, f32p, ctypes.c_uint32, u32p, f32p, ctypes.c_uint64]
        L.orc_bin_dense.restype = ctypes.c_int32
        L.orc_bin_dense.argtypes = [f32p, ctypes.c_uint64, ctypes.c_uint64, u32p, f32p, P(ctypes.c_uint16), u64p]
        L.orc_gradients.restype = None
        L.orc_gradients.argtypes = [ctypes.c_int32, f32p, f32p, ctypes.c_uint64, ctypes.c_float, f32p]
        L.orc_intercepts.restype = None
        L.orc_intercepts.argtypes = [ctypes.c_int32, f32p, ctypes.c_uint64, ctypes.c_int32, f32p]
        L.orc_train.restype = ctypes.c_int64
        L.orc_train.argtypes = [P(OrcParams), f32p, ctypes.c_uint64, ctypes.c_uint64, f32p, ctypes.c_int32, P(OrcNode), ctypes.c_uint64, u64p, f32p, f32p]
        L.orc_softmax_gradients.restype = None
        L.orc_softmax_gradients.argtypes = [f32p, f32p, ctypes.c_uint64, ctypes.c_int32, f32p]
        L.orc_intercepts.restype = None
        L.orc_intercepts.argtypes = [ctypes.c_int32, f32p, ctypes.c_uint64, ctypes.c_int32, f32p]
        L.orc_predict.restype = None
        L.orc_predict.argtypes = [P(OrcNode), u64p, ctypes.c_uint64, ctypes.c_int32, u32p, f32p, f32p, f32p, ctypes.c_uint64, ctypes.c_uint64, f32p]
        L.orc_hist.restype = None
        L.orc_hist.argtypes = [f32p, ctypes.c_uint64, ctypes.c_uint64, u32p, f32p, u32p, ctypes.c_uint64, f32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, P(ctypes.c_double), P(ctypes.c_int64)]
        L.orc_trainer_new.restype = ctypes.c_void_p
        L.orc_trainer_new.argtypes = [P(OrcParams), f32p, ctypes.c_uint64, ctypes.c_uint64, f32p]
        L.orc_trainer_rounds.restype = ctypes.c_int64
        L.orc_trainer_rounds.argtypes = [ctypes.c_void_p, ctypes.c_int32, P(OrcNode), ctypes.c_uint64, u64p]
        L.orc_trainer_free.restype = None
        L.orc_trainer_free.argtypes = [ctypes.c_void_p]
        L.orc_trainer_new_csr.restype = ctypes.c_void_p
        L.orc_trainer_new_csr.argtypes = [P(OrcParams), u64p, u32p, f32p, ctypes.c_uint64, ctypes.c_uint64, f32p]
        L.orc_train_csr.restype = ctypes.c_int64
        L.orc_train_csr.argtypes = [P(OrcParams), u64p, u32p, f32p, ctypes.c_uint64, ctypes.c_uint64, f32p,
                                    ctypes.c_int32, P(OrcNode), ctypes.c_uint64, u64p, f32p, f32p]
        L.orc_cuts_csr.restype = ctypes.c_int64
        L.orc_cuts_csr.argtypes = [u64p, u32p, f32p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int32, u32p, f32p,
                                   ctypes.c_uint64]
        L.orc_trainer_margins.restype = ctypes.c_uint64
        L.orc_trainer_margins.argtypes = [ctypes.c_void_p, f32p, ctypes.c_uint64]
        L.orc_trainer_set_margins.restype = ctypes.c_int32
        L.orc_trainer_set_margins.argtypes = [ctypes.c_void_p, f32p, ctypes.c_uint64]
        L.orc_scan_node.restype = ctypes.c_int32
        L.orc_scan_node.argtypes = [P(OrcParams), u32p, ctypes.c_uint32, ctypes.c_int32, P(ctypes.c_int64),
                                    ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_float,
                                    ctypes.c_float, u32p, P(ctypes.c_int8), ctypes.c_uint32, P(OrcScan)]
        L.orc_fixed_scale.restype = ctypes.c_int32
        L.orc_fixed_scale.argtypes = [ctypes.c_float, ctypes.c_uint64]
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(ctypes.POINTER(t))


def cuts_dense(x, max_bin):
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, f = x.shape
    cap = f * (max_bin + 1)
    off = np.zeros(f + 1, np.uint32)
    vals = np.zeros(cap, np.float32)
    total = lib().orc_cuts_dense(_p(x, ctypes.c_float), n, f, None, max_bin, _p(off, ctypes.c_uint32), _p(vals, ctypes.c_float), cap)
    assert total >= 0
    return off, vals[:total].copy()


def bin_dense(x, off, cuts):
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, f = x.shape
    bins = np.zeros(f * n, np.uint16)
    words = (n + 63) // 64
    miss = np.zeros(f * words, np.uint64)
    dense = lib().orc_bin_dense(_p(x, ctypes.c_float), n, f, _p(off, ctypes.c_uint32), _p(cuts, ctypes.c_float), _p(bins, ctypes.c_uint16), _p(miss, ctypes.c_uint64))
    return bins.reshape(f, n), miss.reshape(f, words), bool(dense)


def gradients(objective, margins, labels, spw=1.0):
    m = np.ascontiguousarray(margins, np.float32)
    y = np.ascontiguousarray(labels, np.float32)
    out = np.zeros(2 * m.size, np.float32)
    lib().orc_gradients(objective, _p(m, ctypes.c_float), _p(y, ctypes.c_float), m.size, spw, _p(out, ctypes.c_float))
    return out.reshape(-1, 2)


def softmax_gradients(margins, labels):
    """multi:softmax pairs (n, k, 2) at margins (n, k), labels class ids (n,)."""
    m = np.ascontiguousarray(margins, np.float32)
    y = np.ascontiguousarray(labels, np.float32)
    n, k = m.shape
    out = np.zeros(2 * m.size, np.float32)
    lib().orc_softmax_gradients(_p(m, ctypes.c_float), _p(y, ctypes.c_float), n, k, _p(out, ctypes.c_float))
    return out.reshape(n, k, 2)


def intercepts(objective, labels, n_outputs):
    y = np.ascontiguousarray(labels, np.float32)
    n = y.shape[0]
    out = np.zeros(n_outputs, np.float32)
    lib().orc_intercepts(objective, _p(y, ctypes.c_float), n, n_outputs, _p(out, ctypes.c_float))
    return out


def fixed_scale(max_abs, n):
    return int(lib().orc_fixed_scale(float(max_abs), int(n)))


def params(**kw):
    p = OrcParams()
    p.objective = kw.get("objective", 0)
    p.n_outputs = kw.get("n_outputs", 1)
    p.max_depth = kw.get("max_depth", 6)
    p.max_leaves = kw.get("max_leaves", 0)
    p.grow_policy = kw.get("grow_policy", 0)
    p.max_bin = kw.get("max_bin", 256)
    p.eta = kw.get("eta", 0.3)
    p.lambda_ = kw.get("reg_lambda", 1.0)
    p.alpha = kw.get("alpha", 0.0)
    p.gamma = kw.get("gamma", 0.0)
    p.min_child_weight = kw.get("min_child_weight", 1.0)
    p.max_delta_step = kw.get("max_delta_step", 0.0)
    p.scale_pos_weight = kw.get("scale_pos_weight", 1.0)
    p.base_score = kw.get("base_score", float("nan"))
    p.fixed_point = 1 if kw.get("fixed_point", False) else 0
    p.n_threads = kw.get("n_threads", 0)
    mono = kw.get("monotone")
    if mono is not None:
        p._mono = np.ascontiguousarray(mono, np.int8)  # kept alive with the struct
        p.monotone = p._mono.ctypes.data_as(ctypes.POINTER(ctypes.c_int8))
        p.n_monotone = p._mono.size
    return p


def train(x, y, rounds, **kw):
    """Returns (nodes structured array, tree_ptr, base (n_out,), margins (n, n_out))."""
    x = np.ascontiguousarray(x, np.float32)
    n, f = x.shape
    if kw.get("objective", 0) == 2:  # multi:softmax: class ids, n_outputs classes
        y = np.ascontiguousarray(y, np.float32).reshape(n)
        k = kw["n_outputs"]
    else:
        y = np.ascontiguousarray(y, np.float32).reshape(n, -1)
        k = y.shape[1]
    kw.setdefault("n_outputs", k)
    p = params(**kw)
    n_trees_max = rounds * k
    depth = p.max_depth if p.max_depth > 0 else 16
    per_tree = (2 ** (depth + 1)) if p.grow_policy == 0 else 2 * max(p.max_leaves, 2 ** depth) + 1
    cap = n_trees_max * per_tree + 1
    nodes = np.zeros(cap, NODE_DTYPE)
    tree_ptr = np.zeros(n_trees_max + 1, np.uint64)
    base = np.zeros(k, np.float32)
    margins = np.zeros(n * k, np.float32)
    got = lib().orc_train(ctypes.byref(p), _p(x, ctypes.c_float), n, f, _p(y, ctypes.c_float), rounds,
                          nodes.ctypes.data_as(ctypes.POINTER(OrcNode)), cap, _p(tree_ptr, ctypes.c_uint64),
                          _p(base, ctypes.c_float), _p(margins, ctypes.c_float))
    assert got >= 0, got
    tree_ptr = tree_ptr[: got + 1]
    return nodes[: int(tree_ptr[-1])].copy(), tree_ptr.copy(), base, margins.reshape(n, k)


def _csr(indptr, indices, values):
    return (np.ascontiguousarray(indptr, np.uint64), np.ascontiguousarray(indices, np.uint32),
            np.ascontiguousarray(values, np.float32))


def cuts_csr(indptr, indices, values, n_cols, max_bin):
    ip, ix, vs = _csr(indptr, indices, values)
    cap = n_cols * (max_bin + 1)
    off = np.zeros(n_cols + 1, np.uint32)
    vals = np.zeros(cap, np.float32)
    total = lib().orc_cuts_csr(_p(ip, ctypes.c_uint64), _p(ix, ctypes.c_uint32), _p(vs, ctypes.c_float),
                               ip.size - 1, n_cols, max_bin, _p(off, ctypes.c_uint32), _p(vals, ctypes.c_float), cap)
    assert total >= 0
    return off, vals[:total].copy()


def _tree_cap(p):
    depth = p.max_depth if p.max_depth > 0 else 16
    if p.grow_policy == 0:
        return 2 ** (depth + 1)
    return 2 * (p.max_leaves if p.max_leaves > 0 else 2 ** depth) + 1


def train_csr(indptr, indices, values, n_cols, y, rounds, **kw):
    """`train` on CSR arrays (absent cells missing): the oracle's CSR index."""
    ip, ix, vs = _csr(indptr, indices, values)
    n = ip.size - 1
    if kw.get("objective", 0) == 2:
        y = np.ascontiguousarray(y, np.float32).reshape(n)
        k = kw["n_outputs"]
    else:
        y = np.ascontiguousarray(y, np.float32).reshape(n, -1)
        k = y.shape[1]
    kw.setdefault("n_outputs", k)
    p = params(**kw)
    cap = rounds * k * _tree_cap(p) + 1
    nodes = np.zeros(cap, NODE_DTYPE)
    tree_ptr = np.zeros(rounds * k + 1, np.uint64)
    base = np.zeros(k, np.float32)
    margins = np.zeros(n * k, np.float32)
    got = lib().orc_train_csr(ctypes.byref(p), _p(ip, ctypes.c_uint64), _p(ix, ctypes.c_uint32), _p(vs, ctypes.c_float),
                              n, n_cols, _p(y, ctypes.c_float), rounds, nodes.ctypes.data_as(ctypes.POINTER(OrcNode)),
                              cap, _p(tree_ptr, ctypes.c_uint64), _p(base, ctypes.c_float), _p(margins, ctypes.c_float))
    assert got >= 0, got
    tree_ptr = tree_ptr[: got + 1]
    return nodes[: int(tree_ptr[-1])].copy(), tree_ptr.copy(), base, margins.reshape(n, k)


def predict(nodes, tree_ptr, n_outputs, base, x, tree_output=None, tree_weight=None):
    x = np.ascontiguousarray(x, np.float32)
    n, f = x.shape
    nodes = np.ascontiguousarray(nodes, NODE_DTYPE)
    tree_ptr = np.ascontiguousarray(tree_ptr, np.uint64)
    base = np.ascontiguousarray(base, np.float32)
    out = np.zeros(n * n_outputs, np.float32)
    to = None if tree_output is None else np.ascontiguousarray(tree_output, np.uint32)
    tw = None if tree_weight is None else np.ascontiguousarray(tree_weight, np.float32)
    lib().orc_predict(nodes.ctypes.data_as(ctypes.POINTER(OrcNode)), _p(tree_ptr, ctypes.c_uint64), len(tree_ptr) - 1,
                      n_outputs, None if to is None else _p(to, ctypes.c_uint32), None if tw is None else _p(tw, ctypes.c_float),
                      _p(base, ctypes.c_float), _p(x, ctypes.c_float), n, f, _p(out, ctypes.c_float))
    return out.reshape(n, n_outputs)


def golden_layout(model):
    """(n_trees used, tree_output, tree_weight) of a saved model's effective
    iterations (BoostedModel::effective_num_trees, model/mod.rs:1238)."""
    n_out, npt = model["n_outputs"], model["num_parallel_tree"]
    per = n_out * npt
    n = len(model["trees"])
    if model["best_iteration"] is not None:
        n = min((model["best_iteration"] + 1) * per, n)
    outputs = np.array([(t // npt) % n_out for t in range(n)], np.uint32)
    weights = np.array(model["tree_weights"][:n], np.float32)
    return n, outputs, weights


def hist(x, off, cuts, rows, gpair, fixed_point=False, sg=0, sh=0):
    x = np.ascontiguousarray(x, np.float32)
    n, f = x.shape
    rows = np.ascontiguousarray(rows, np.uint32)
    gp = np.ascontiguousarray(gpair, np.float32).reshape(-1)
    nb = int(off[-1])
    o64 = np.zeros(2 * nb, np.float64)
    oi = np.zeros(2 * nb, np.int64)
    lib().orc_hist(_p(x, ctypes.c_float), n, f, _p(off, ctypes.c_uint32), _p(cuts, ctypes.c_float), _p(rows, ctypes.c_uint32),
                   len(rows), _p(gp, ctypes.c_float), 1 if fixed_point else 0, sg, sh,
                   _p(o64, ctypes.c_double), _p(oi, ctypes.c_int64))
    return (oi if fixed_point else o64).reshape(nb, 2)


# ---------------------------------------------------------------- golden data
def scan_node(hist_q, feature_offset, dense, total_q, sg, sh, features, directions=None,
              bounds=(-np.inf, np.inf), **kw):
    """One node's fixed-point split search (orc_scan_node): `hist_q` the
    int64 (g, h) histogram, `total_q` the node's int64 totals."""
    p = params(**kw)
    h = np.ascontiguousarray(hist_q, np.int64)
    off = np.ascontiguousarray(feature_offset, np.uint32)
    f = np.ascontiguousarray(features, np.uint32)
    d = None if directions is None else np.ascontiguousarray(directions, np.int8)
    out = OrcScan()
    st = lib().orc_scan_node(ctypes.byref(p), _p(off, ctypes.c_uint32), off.size - 1, 1 if dense else 0,
                             _p(h, ctypes.c_int64), int(total_q[0]), int(total_q[1]), sg, sh,
                             float(bounds[0]), float(bounds[1]), _p(f, ctypes.c_uint32),
                             None if d is None else _p(d, ctypes.c_int8), f.size, ctypes.byref(out))
    assert st == 0, st
    return out


def bits_to_f32(bits):
    return np.array(bits, dtype=np.uint32).view(np.float32)


def golden():
    with open(GOLDEN) as fh:
        g = json.load(fh)
    g["x"] = bits_to_f32(g["probe_x_bits"]).reshape(-1, 4)
    g["y1"] = bits_to_f32(g["labels_k1_bits"]).reshape(-1, 1)
    g["y2"] = bits_to_f32(g["labels_k2_bits"]).reshape(-1, 2)
    return g


def golden_nodes(model):
    """A saved model's trees as (nodes structured array, tree_ptr)."""
    parts, ptr = [], [0]
    for t in model["trees"]:
        n = len(t["left"])
        a = np.zeros(n, NODE_DTYPE)
        for k in ("left", "right", "split_feature", "split_cond", "leaf_value", "sum_hess", "split_gain"):
            a[k] = t[k]
        a["default_left"] = np.array(t["default_left"], dtype=np.uint32)
        a["split_bin"] = -1
        parts.append(a)
        ptr.append(ptr[-1] + n)
    return np.concatenate(parts), np.array(ptr, np.uint64)


def f32_to_bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def struct_f32(v):
    return struct.unpack("<I", struct.pack("<f", v))[0]


class Trainer:
    """An oracle training session: preparation (cuts, bins, intercepts) in
    the constructor, timed rounds in ``rounds``."""

    def __init__(self, x, y, csr=None, **kw):
        """`x` dense f32 rows, or None with `csr` = (indptr, indices, values, n_cols)."""
        if csr is not None:
            self._csr = _csr(*csr[:3])
            n, f = self._csr[0].size - 1, csr[3]
            self._x = None
        else:
            self._x = np.ascontiguousarray(x, np.float32)
            n, f = self._x.shape
        if kw.get("objective", 0) == 2:  # multi:softmax: class ids, n_outputs classes
            self._y = np.ascontiguousarray(y, np.float32).reshape(n)
        else:
            self._y = np.ascontiguousarray(y, np.float32).reshape(n, -1)
            kw.setdefault("n_outputs", self._y.shape[1])
        self.p = params(**kw)
        if self._x is None:
            ip, ix, vs = self._csr
            self.h = lib().orc_trainer_new_csr(ctypes.byref(self.p), _p(ip, ctypes.c_uint64), _p(ix, ctypes.c_uint32),
                                               _p(vs, ctypes.c_float), n, f, _p(self._y, ctypes.c_float))
        else:
            self.h = lib().orc_trainer_new(ctypes.byref(self.p), _p(self._x, ctypes.c_float), n, f,
                                           _p(self._y, ctypes.c_float))
        assert self.h

    def rounds(self, k):
        cap = max(k, 1) * self.p.n_outputs * _tree_cap(self.p) + 1
        nodes = np.zeros(cap, NODE_DTYPE)
        ptr = np.zeros(k * self.p.n_outputs + 1, np.uint64)
        got = lib().orc_trainer_rounds(self.h, k, nodes.ctypes.data_as(ctypes.POINTER(OrcNode)), cap, _p(ptr, ctypes.c_uint64))
        assert got >= 0, got
        return nodes[: int(ptr[got])].copy(), ptr[: got + 1].copy()

    def margins(self):
        """The session's training margins, (n, n_outputs)."""
        n = int(lib().orc_trainer_margins(self.h, None, 0))
        out = np.zeros(n, np.float32)
        lib().orc_trainer_margins(self.h, _p(out, ctypes.c_float), n)
        return out.reshape(-1, self.p.n_outputs)

    def set_margins(self, m):
        m = np.ascontiguousarray(m, np.float32).ravel()
        assert lib().orc_trainer_set_margins(self.h, _p(m, ctypes.c_float), m.size) == 0

    def close(self):
        if self.h:
            lib().orc_trainer_free(self.h)
            self.h = None

    def __del__(self):
        self.close()
