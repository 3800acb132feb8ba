"""hessboost_b200: hessboost's ``tree_method = hist`` path on B200 GPUs.

The product is ``_lib/libhb_cuda.so``, a C-ABI library (``include/hb_backend.h``)
whose entry points mirror hessboost's ``HistogramBackend`` / ``RowEngine``
backend seam (``src/tree/hist/mod.rs:73-295``) and its GPU prediction model.
This module binds it with ctypes and offers the reference's user-level verbs
on top: cuts and binning of a dense matrix, ``train`` of a single-output
squared-error or logistic model, and batch ``predict_margin``.

There is no CPU fallback: every computing call goes to the CUDA library, and
importing a missing library raises.
"""

import ctypes
import math
import os
from dataclasses import dataclass

import numpy as np

from . import build as _build

__all__ = [
    "HbError",
    "lib",
    "TrainingParams",
    "BinnedMatrix",
    "Engine",
    "Model",
    "Predictor",
    "cuts_dense",
    "bin_dense",
    "train",
    "NODE_DTYPE",
]

HB_OK, HB_REFUSED, HB_DEVICE_FAILED, HB_INVALID_ARGUMENT = 0, 1, 2, 3
HB_LOSS_SQUARED_ERROR, HB_LOSS_LOGISTIC, HB_LOSS_SOFTMAX = 0, 1, 2
HB_GROW_DEPTHWISE, HB_GROW_LOSSGUIDE = 0, 1
HB_SCAN_EMPTY, HB_SCAN_REPLAY, HB_SCAN_NUMERIC = 0, 1, 2  # NodeScan kinds


class HbError(RuntimeError):
    """A call into libhb_cuda returned a status other than HB_OK."""

    def __init__(self, status, where, detail=""):
        self.status = status
        names = {1: "refused", 2: "device failed", 3: "invalid argument"}
        super().__init__(f"{where}: {names.get(status, status)}" + (f" ({detail})" if detail else ""))


# ---------------------------------------------------------------- C structs
class GradStats(ctypes.Structure):
    _fields_ = [("grad", ctypes.c_double), ("hess", ctypes.c_double)]


class Segment(ctypes.Structure):
    _fields_ = [
        ("offset", ctypes.c_uint64),
        ("len", ctypes.c_uint64),
        ("contiguous", ctypes.c_uint32),
        ("reserved", ctypes.c_uint32),
        ("tree", ctypes.c_uint64),
    ]


class RowSplit(ctypes.Structure):
    _fields_ = [
        ("seg", Segment),
        ("feature", ctypes.c_uint32),
        ("limit", ctypes.c_uint32),
        ("default_left", ctypes.c_uint32),
        ("reserved", ctypes.c_uint32),
    ]


class Partitioned(ctypes.Structure):
    _fields_ = [("left", Segment), ("right", Segment)]


class RegParams(ctypes.Structure):
    _fields_ = [
        ("lambda_", ctypes.c_double),
        ("alpha", ctypes.c_double),
        ("max_delta_step", ctypes.c_double),
        ("min_child_weight", ctypes.c_double),
    ]


def node_gain(total, reg, lower=-math.inf, upper=math.inf):
    """xgb_node_gain (src/tree/builder/shared.rs:136) of a node with
    statistics `total` = (G, H) and monotone bounds [lower, upper]: the
    scorer's root gain a ScanRequest carries (f32)."""
    g, h = float(total[0]), float(total[1])
    if h <= 0.0:
        return 0.0
    a = reg.alpha
    t = g - a if g > a else (g + a if g < -a else 0.0)
    w = -t / (h + reg.lambda_)
    if reg.max_delta_step != 0.0 and abs(w) > reg.max_delta_step:
        w = math.copysign(reg.max_delta_step, w)
    w32 = np.float32(w)
    lo, up = np.float32(lower), np.float32(upper)
    w32 = lo if w32 < lo else (up if w32 > up else w32)
    wf = float(w32)
    gain = -(2.0 * g * wf + (h + reg.lambda_) * float(np.float32(w32 * w32)) + 2.0 * a * abs(wf))
    return float(np.float32(gain))


class ScanRequest(ctypes.Structure):
    _fields_ = [
        ("slot", ctypes.c_uint32),
        ("n_features", ctypes.c_uint32),
        ("features", ctypes.POINTER(ctypes.c_uint32)),
        ("directions", ctypes.POINTER(ctypes.c_int8)),
        ("total", GradStats),
        ("root_gain", ctypes.c_float),
        ("lower", ctypes.c_float),
        ("upper", ctypes.c_float),
        ("reserved", ctypes.c_uint32),
    ]


class NodeScan(ctypes.Structure):
    _fields_ = [
        ("kind", ctypes.c_uint32),
        ("feature", ctypes.c_uint32),
        ("loss_chg", ctypes.c_float),
        ("backward", ctypes.c_uint32),
        ("offset", ctypes.c_uint32),
        ("reserved", ctypes.c_uint32),
        ("acc", GradStats),
    ]


class DeviceLoss(ctypes.Structure):
    _fields_ = [
        ("kind", ctypes.c_int32),
        ("scale_pos_weight", ctypes.c_float),
        ("min_hess", ctypes.c_float),
        ("reserved", ctypes.c_int32),
    ]


class GHist(ctypes.Structure):
    _fields_ = [
        ("n_rows", ctypes.c_uint64),
        ("n_cols", ctypes.c_uint32),
        ("dense", ctypes.c_uint32),
        ("feature_offset", ctypes.POINTER(ctypes.c_uint32)),
        ("cut_values", ctypes.POINTER(ctypes.c_float)),
        ("columns", ctypes.POINTER(ctypes.c_uint8)),
        ("missing", ctypes.POINTER(ctypes.c_uint64)),
        ("row_ptr", ctypes.POINTER(ctypes.c_uint64)),
        ("row_bins", ctypes.POINTER(ctypes.c_uint32)),
    ]


class TreeNode(ctypes.Structure):
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


class TrainParamsC(ctypes.Structure):
    _fields_ = [
        ("objective", ctypes.c_int32),
        ("max_depth", ctypes.c_int32),
        ("max_leaves", ctypes.c_int32),
        ("grow_policy", ctypes.c_int32),
        ("eta", ctypes.c_float),
        ("lambda_", ctypes.c_float),
        ("alpha", ctypes.c_float),
        ("gamma", ctypes.c_float),
        ("min_child_weight", ctypes.c_float),
        ("max_delta_step", ctypes.c_float),
        ("scale_pos_weight", ctypes.c_float),
        ("base_score", ctypes.c_float),
        ("num_class", ctypes.c_int32),
        ("n_monotone", ctypes.c_int32),
        ("monotone", ctypes.POINTER(ctypes.c_int8)),
    ]


class EngineStats(ctypes.Structure):
    _fields_ = [
        ("ms", ctypes.c_double * 8),
        ("timed_launches", ctypes.c_uint64 * 8),
        ("kernel_launches", ctypes.c_uint64),
        ("rows_built_contiguous", ctypes.c_uint64),
        ("rows_built_gathered", ctypes.c_uint64),
        ("rounds", ctypes.c_uint64),
        ("last_rounds_ms", ctypes.c_double),
    ]


TIMER_NAMES = ["gradients", "root_hist", "scan", "apply", "partition", "hist", "subtract", "other"]

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
assert NODE_DTYPE.itemsize == ctypes.sizeof(TreeNode) == 40

# Every entry point include/hb_backend.h declares, with its ctypes signature.
_P = ctypes.POINTER
_u8p, _u32p, _u64p, _f32p = _P(ctypes.c_uint8), _P(ctypes.c_uint32), _P(ctypes.c_uint64), _P(ctypes.c_float)
_vp, _i32p = ctypes.c_void_p, _P(ctypes.c_int32)
SIGNATURES = {
    "hb_engine_create": [ctypes.c_int32, _P(_vp)],
    "hb_engine_destroy": [_vp],
    "hb_engine_upload": [_vp, _P(GHist)],
    "hb_engine_last_error": [_vp],
    "hb_engine_set_shard": [_vp, ctypes.c_uint64, ctypes.c_uint64],
    "hb_prepare": [_vp, _f32p, ctypes.c_uint64],
    "hb_build": [_vp, _u32p, ctypes.c_uint64, _P(GradStats)],
    "hb_build_features": [_vp, _u32p, ctypes.c_uint64, _u32p, ctypes.c_uint32, _P(GradStats)],
    "hb_build_noalloc": [_vp, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p],
    "hb_begin_tree": [_vp, _u32p, ctypes.c_uint64, _P(Segment)],
    "hb_root_total": [_vp, _P(Segment), _P(GradStats)],
    "hb_partition": [_vp, _P(RowSplit), ctypes.c_uint32, _P(Partitioned)],
    "hb_histograms": [_vp, _P(Segment), ctypes.c_uint32, _P(GradStats)],
    "hb_rows": [_vp, _P(Segment), ctypes.c_uint32, _u32p],
    "hb_load_margins": [_vp, _f32p, ctypes.c_uint64],
    "hb_gradients": [_vp, _P(DeviceLoss), _f32p, _f32p, ctypes.c_uint64, _i32p],
    "hb_add_leaf_values": [_vp, _P(Segment), _f32p, ctypes.c_uint32],
    "hb_read_margins": [_vp, _f32p, ctypes.c_uint64],
    "hb_reserve_hists": [_vp, ctypes.c_uint32, _i32p],
    "hb_build_resident": [_vp, _P(Segment), _u32p, ctypes.c_uint32, _u32p, ctypes.c_uint32],
    "hb_scan_resident": [_vp, _P(RegParams), _P(ScanRequest), ctypes.c_uint32, _P(NodeScan)],
    "hb_read_hist": [_vp, ctypes.c_uint32, _P(GradStats)],
    "hb_read_gradients": [_vp, _f32p, ctypes.c_uint64, _i32p, _i32p],
    "hb_grow_tree": [_vp, _P(TrainParamsC), _P(TreeNode), ctypes.c_uint32, _u32p],
    "hb_train": [_vp, _P(TrainParamsC), _f32p, ctypes.c_uint64, ctypes.c_float, ctypes.c_int32, _P(TreeNode), ctypes.c_uint64, _u64p],
    "hb_train_begin_classes": [_vp, _f32p, ctypes.c_uint64, _f32p, ctypes.c_int32],
    "hb_train_begin": [_vp, _f32p, ctypes.c_uint64, ctypes.c_float],
    "hb_train_rounds": [_vp, _P(TrainParamsC), ctypes.c_int32, _P(TreeNode), ctypes.c_uint64, _u64p],
    "hb_engine_reset_stats": [_vp, ctypes.c_int32],
    "hb_engine_get_stats": [_vp, _P(EngineStats)],
    "hb_engine_stream": [_vp, _P(_vp)],
    "hb_comm_unique_id": [_u8p],
    "hb_comm_init": [_vp, ctypes.c_int32, ctypes.c_int32, _u8p, ctypes.c_uint64],
    "hb_predictor_create": [ctypes.c_int32, _P(TreeNode), _u64p, ctypes.c_uint64, _u32p, _f32p, ctypes.c_int32, _f32p, ctypes.c_uint32, _P(_vp)],
    "hb_predictor_destroy": [_vp],
    "hb_predict_margin": [_vp, _f32p, ctypes.c_uint64, _f32p],
    "hb_predict_margin_device": [_vp, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, _vp],
    "hb_cuts_dense": [_f32p, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, _u32p, _f32p, ctypes.c_uint64, _u64p],
    "hb_bin_dense": [_f32p, ctypes.c_uint64, ctypes.c_uint32, _u32p, _f32p, _u8p, _u64p, _i32p],
    "hb_cuts_csr": [_u64p, _u32p, _f32p, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, _u32p, _f32p,
                    ctypes.c_uint64, _u64p],
    "hb_bin_csr": [_u64p, _u32p, _f32p, ctypes.c_uint64, ctypes.c_uint32, _u32p, _f32p, _u64p, _u32p, _i32p],
    "hb_sketch_dense": [ctypes.c_int32, _f32p, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, _u32p, _f32p,
                        ctypes.c_uint64, _u64p, _u8p, _u64p, _i32p],
    "hb_sketch_csr": [ctypes.c_int32, _u64p, _u32p, _f32p, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, _u32p,
                      _f32p, ctypes.c_uint64, _u64p, _u32p, _i32p],
    "hb_sketch_last_error": [],
    "hb_xxh64": [ctypes.c_void_p, ctypes.c_uint64, _u64p],
    "hb_engine_upload_dense": [_vp, _f32p, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, _u32p, _f32p,
                               ctypes.c_uint64, _u64p],
    "hb_engine_upload_csr": [_vp, _u64p, _u32p, _f32p, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, _u32p,
                             _f32p, ctypes.c_uint64, _u64p],
    "hb_engine_inject_fault": [_vp, ctypes.c_int32],
    "hb_probe_smem": [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                      ctypes.POINTER(ctypes.c_double)],
    "hb_peer_wait_probe": [ctypes.c_int32, ctypes.c_int32, _u64p, ctypes.POINTER(ctypes.c_double)],
}
_STRING_RESULT = ("hb_engine_last_error", "hb_sketch_last_error")

_lib = None


def lib():
    """The loaded libhb_cuda.so (built in-tree on first use if absent)."""
    global _lib
    if _lib is None:
        path = _build.LIB
        if not os.path.exists(path):
            _build.build()
        L = ctypes.CDLL(path)
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_char_p if name in _STRING_RESULT else ctypes.c_int32
        _lib = L
    return _lib


def _ptr(a, t):
    return a.ctypes.data_as(ctypes.POINTER(t))


def _check(status, where, handle=None):
    if status != HB_OK:
        detail = ""
        try:
            msg = lib().hb_engine_last_error(handle)
            detail = msg.decode() if msg else ""
        except Exception:  # noqa: BLE001 - best effort detail
            pass
        raise HbError(status, where, detail)


# ---------------------------------------------------------------- params
@dataclass
class TrainingParams:
    """The ``TrainingParams`` fields of the hist path
    (src/config/params.rs:653; defaults as the reference's)."""

    objective: str = "reg:squarederror"
    max_depth: int = 6
    max_leaves: int = 0
    grow_policy: str = "depthwise"
    eta: float = 0.3
    reg_lambda: float = 1.0
    alpha: float = 0.0
    gamma: float = 0.0
    min_child_weight: float = 1.0
    max_delta_step: float = 0.0
    scale_pos_weight: float = 1.0
    base_score: float = float("nan")
    max_bin: int = 256
    num_class: int = 0
    monotone_constraints: tuple = ()  # per feature: 1 increasing, -1 decreasing, 0 none

    def validate(self):
        """The reference's parameter checks for these fields
        (TrainingParams::validate, src/config/params.rs:906-918 and :1036;
        the helpers of src/check.rs; scale_pos_weight,
        src/objective/params.rs:330): ValueError naming the first
        parameter that fails. Returns self."""
        def ensure(name, ok, reason):
            if not ok:
                raise ValueError(f"invalid parameter `{name}`: {reason}")

        def finite(v):
            return math.isfinite(float(v))

        def narrows(name, v, positive):
            # stays finite (and > 0) once narrowed to f32
            with np.errstate(over="ignore"):
                n = np.float32(v)
            ensure(name, np.isfinite(n) and (not positive or n > 0),
                   f"must stay {'positive and ' if positive else ''}finite in f32, got {v}")

        ensure("eta", finite(self.eta) and self.eta > 0, f"must be > 0, got {self.eta}")
        narrows("eta", self.eta, True)
        for name in ("gamma", "min_child_weight", "reg_lambda", "alpha"):
            v = getattr(self, name)
            ensure(name, finite(v) and v >= 0, f"must be >= 0, got {v}")
            narrows(name, v, False)
        # 0 is "no bound"; a bound must be finite and > 0
        ensure("max_delta_step", finite(self.max_delta_step) and self.max_delta_step >= 0,
               f"a bound must be > 0 (0 for none), got {self.max_delta_step}")
        if self.max_delta_step > 0:
            narrows("max_delta_step", self.max_delta_step, True)
        ensure("scale_pos_weight", finite(self.scale_pos_weight) and self.scale_pos_weight > 0,
               f"must be > 0, got {self.scale_pos_weight}")
        narrows("scale_pos_weight", self.scale_pos_weight, True)
        ensure("max_bin", self.max_bin >= 2, f"must be >= 2, got {self.max_bin}")
        ensure("max_depth", self.max_depth >= 0, f"must be >= 0 (0 for no limit), got {self.max_depth}")
        ensure("max_leaves", self.max_leaves >= 0, f"must be >= 0 (0 for no limit), got {self.max_leaves}")
        ensure("max_leaves", not (self.grow_policy == "lossguide" and self.max_leaves == 0 and self.max_depth == 0),
               "lossguide growth needs a bound: set max_leaves or max_depth")
        ensure("grow_policy", self.grow_policy in ("depthwise", "lossguide"),
               f"must be depthwise or lossguide, got {self.grow_policy!r}")
        ensure("monotone_constraints", all(int(v) in (-1, 0, 1) and int(v) == v for v in self.monotone_constraints),
               "every entry must be 1 (increasing), -1 (decreasing) or 0 (none)")
        return self

    def validate_for(self, n_features):
        """validate_constraints (src/training/validate.rs:283): the
        constraints name only features of the training matrix."""
        if len(self.monotone_constraints) > n_features:
            raise ValueError("invalid parameter `monotone_constraints`: contains more entries than the "
                             "training matrix has features")
        return self

    def loss_kind(self):
        if self.objective in ("reg:squarederror",):
            return HB_LOSS_SQUARED_ERROR
        if self.objective in ("binary:logistic", "reg:logistic", "binary:logitraw"):
            return HB_LOSS_LOGISTIC
        if self.objective in ("multi:softmax", "multi:softprob"):
            return HB_LOSS_SOFTMAX
        raise ValueError(f"objective {self.objective!r} is not on the device path")

    def n_outputs(self):
        return self.num_class if self.loss_kind() == HB_LOSS_SOFTMAX else 1

    def tree_slots(self):
        """Nodes one grown tree can have: 2 * leaves (lossguide: max_leaves,
        else 2^max_depth; depthwise 2^max_depth)."""
        if self.grow_policy == "lossguide":
            return 2 * (self.max_leaves if self.max_leaves > 0 else 1 << self.max_depth)
        return 2 << self.max_depth

    def to_c(self):
        c = TrainParamsC()
        c.objective = self.loss_kind()
        c.max_depth = self.max_depth
        c.max_leaves = self.max_leaves
        if self.grow_policy not in ("depthwise", "lossguide"):
            raise ValueError(f"grow_policy {self.grow_policy!r}")
        c.grow_policy = HB_GROW_DEPTHWISE if self.grow_policy == "depthwise" else HB_GROW_LOSSGUIDE
        c.eta = self.eta
        c.lambda_ = self.reg_lambda
        c.alpha = self.alpha
        c.gamma = self.gamma
        c.min_child_weight = self.min_child_weight
        c.max_delta_step = self.max_delta_step
        c.scale_pos_weight = self.scale_pos_weight
        c.base_score = self.base_score
        c.num_class = self.num_class
        if len(self.monotone_constraints):
            c._mono = np.ascontiguousarray(self.monotone_constraints, np.int8)  # kept alive with the struct
            c.n_monotone = c._mono.size
            c.monotone = c._mono.ctypes.data_as(ctypes.POINTER(ctypes.c_int8))
        return c

    def reg(self):
        """RegParams (gain.rs:83): every value rounded to f32."""
        r = RegParams()
        r.lambda_ = float(np.float32(self.reg_lambda))
        r.alpha = float(np.float32(self.alpha))
        r.max_delta_step = float(np.float32(self.max_delta_step))
        r.min_child_weight = float(np.float32(self.min_child_weight))
        return r


# ---------------------------------------------------------------- binning
def cuts_dense(x, max_bin=256):
    """HistCuts::from_dmatrix of a dense f32 matrix (NaN missing)."""
    x = np.ascontiguousarray(x, np.float32)
    n, f = x.shape
    cap = f * (max_bin + 1)
    off = np.zeros(f + 1, np.uint32)
    vals = np.zeros(cap, np.float32)
    total = ctypes.c_uint64()
    _check(lib().hb_cuts_dense(_ptr(x, ctypes.c_float), n, f, max_bin, _ptr(off, ctypes.c_uint32),
                               _ptr(vals, ctypes.c_float), cap, ctypes.byref(total)), "hb_cuts_dense")
    return off, vals[: total.value].copy()


def bin_dense(x, feature_offset, cut_values):
    """One-byte feature-local bins (feature-major) and the missing bitmap."""
    x = np.ascontiguousarray(x, np.float32)
    n, f = x.shape
    cols = np.zeros(f * n, np.uint8)
    words = (n + 63) // 64
    miss = np.zeros(f * words, np.uint64)
    dense = ctypes.c_int32()
    off = np.ascontiguousarray(feature_offset, np.uint32)
    cuts = np.ascontiguousarray(cut_values, np.float32)
    _check(lib().hb_bin_dense(_ptr(x, ctypes.c_float), n, f, _ptr(off, ctypes.c_uint32), _ptr(cuts, ctypes.c_float),
                              _ptr(cols, ctypes.c_uint8), _ptr(miss, ctypes.c_uint64), ctypes.byref(dense)), "hb_bin_dense")
    return cols.reshape(f, n), miss.reshape(f, words), bool(dense.value)


def _csr_arrays(indptr, indices, values):
    return (np.ascontiguousarray(indptr, np.uint64), np.ascontiguousarray(indices, np.uint32),
            np.ascontiguousarray(values, np.float32))


def cuts_csr(indptr, indices, values, n_cols, max_bin=256):
    """HistCuts::from_dmatrix of a CSR matrix (absent entries missing)."""
    ip, ix, vs = _csr_arrays(indptr, indices, values)
    cap = n_cols * (max_bin + 1)
    off = np.zeros(n_cols + 1, np.uint32)
    vals = np.zeros(cap, np.float32)
    total = ctypes.c_uint64()
    _check(lib().hb_cuts_csr(_ptr(ip, ctypes.c_uint64), _ptr(ix, ctypes.c_uint32), _ptr(vs, ctypes.c_float),
                             ip.size - 1, n_cols, max_bin, _ptr(off, ctypes.c_uint32), _ptr(vals, ctypes.c_float),
                             cap, ctypes.byref(total)), "hb_cuts_csr")
    return off, vals[: total.value].copy()


def bin_csr(indptr, indices, values, n_cols, feature_offset, cut_values):
    """The CSR index: row offsets and each entry's global bin (ascending in a row)."""
    ip, ix, vs = _csr_arrays(indptr, indices, values)
    n = ip.size - 1
    row_ptr = np.zeros(n + 1, np.uint64)
    row_bins = np.zeros(max(int(ip[-1]), 1), np.uint32)
    dense = ctypes.c_int32()
    off = np.ascontiguousarray(feature_offset, np.uint32)
    cuts = np.ascontiguousarray(cut_values, np.float32)
    _check(lib().hb_bin_csr(_ptr(ip, ctypes.c_uint64), _ptr(ix, ctypes.c_uint32), _ptr(vs, ctypes.c_float), n,
                            n_cols, _ptr(off, ctypes.c_uint32), _ptr(cuts, ctypes.c_float),
                            _ptr(row_ptr, ctypes.c_uint64), _ptr(row_bins, ctypes.c_uint32), ctypes.byref(dense)),
           "hb_bin_csr")
    return row_ptr, row_bins[: int(ip[-1])], bool(dense.value)


def _sketch_check(status, where):
    if status != HB_OK:
        msg = lib().hb_sketch_last_error()
        raise HbError(status, where, msg.decode() if msg else "")


def sketch_dense(x, max_bin=256, device=0, bins=True):
    """hb_cuts_dense (+ hb_bin_dense when ``bins``) computed on ``device``:
    returns (feature_offset, cut_values, columns, missing, dense), the last
    three None without ``bins``."""
    x = np.ascontiguousarray(x, np.float32)
    n, f = x.shape
    cap = f * max(max_bin, 1)
    off = np.zeros(f + 1, np.uint32)
    vals = np.zeros(cap, np.float32)
    total = ctypes.c_uint64()
    cols = miss = None
    dense = ctypes.c_int32()
    if bins:
        cols = np.empty((f, n), np.uint8)
        miss = np.zeros((f, (n + 63) // 64), np.uint64)
    _sketch_check(lib().hb_sketch_dense(device, _ptr(x, ctypes.c_float), n, f, max_bin, _ptr(off, ctypes.c_uint32),
                                        _ptr(vals, ctypes.c_float), cap, ctypes.byref(total),
                                        None if cols is None else _ptr(cols, ctypes.c_uint8),
                                        None if miss is None else _ptr(miss, ctypes.c_uint64),
                                        ctypes.byref(dense) if bins else None), "hb_sketch_dense")
    vals = vals[: total.value].copy()
    if not bins:
        return off, vals, None, None, None
    return off, vals, cols, miss, bool(dense.value)


def sketch_csr(indptr, indices, values, n_cols, max_bin=256, device=0, bins=True):
    """hb_cuts_csr (+ hb_bin_csr when ``bins``) computed on ``device``:
    returns (feature_offset, cut_values, row_bins, dense)."""
    ip, ix, vs = _csr_arrays(indptr, indices, values)
    n = ip.size - 1
    cap = n_cols * max(max_bin, 1)
    off = np.zeros(n_cols + 1, np.uint32)
    vals = np.zeros(cap, np.float32)
    total = ctypes.c_uint64()
    dense = ctypes.c_int32()
    rb = np.empty(max(int(ip[-1]), 1), np.uint32) if bins else None
    _sketch_check(lib().hb_sketch_csr(device, _ptr(ip, ctypes.c_uint64), _ptr(ix, ctypes.c_uint32),
                                      _ptr(vs, ctypes.c_float), n, n_cols, max_bin, _ptr(off, ctypes.c_uint32),
                                      _ptr(vals, ctypes.c_float), cap, ctypes.byref(total),
                                      None if rb is None else _ptr(rb, ctypes.c_uint32),
                                      ctypes.byref(dense) if bins else None), "hb_sketch_csr")
    vals = vals[: total.value].copy()
    if not bins:
        return off, vals, None, None
    return off, vals, rb[: int(ip[-1])], bool(dense.value)


class DeviceIndex:
    """What the host keeps of an index the engine sketched and binned on its
    own device (hb_engine_upload_dense / _csr): the cuts and the shape."""

    def __init__(self, feature_offset, cut_values, n_rows, n_cols):
        self.feature_offset = feature_offset
        self.cut_values = cut_values
        self.n_rows = n_rows
        self.n_cols = n_cols

    @property
    def total_bins(self):
        return int(self.feature_offset[-1])


class BinnedMatrix:
    """A GHistIndex-equivalent: cuts plus either one-byte feature-major bins
    and the missing bitmap, or (``from_csr``) the CSR rows of global bins."""

    def __init__(self, feature_offset, cut_values, columns, missing, dense, row_ptr=None, row_bins=None):
        self.feature_offset = np.ascontiguousarray(feature_offset, np.uint32)
        self.cut_values = np.ascontiguousarray(cut_values, np.float32)
        self.dense = bool(dense)
        if columns is None:
            self.columns = self.missing = None
            self.row_ptr = np.ascontiguousarray(row_ptr, np.uint64)
            self.row_bins = np.ascontiguousarray(row_bins, np.uint32)
            self.n_cols = self.feature_offset.size - 1
            self.n_rows = self.row_ptr.size - 1
            return
        self.row_ptr = self.row_bins = None
        self.columns = np.ascontiguousarray(columns, np.uint8)
        self.missing = None if dense else np.ascontiguousarray(missing, np.uint64)
        self.n_cols, self.n_rows = self.columns.shape

    @property
    def is_csr(self):
        return self.columns is None

    @classmethod
    def from_dense(cls, x, max_bin=256, cuts=None, device=None):
        """Host sketch and binning; with ``device`` (a GPU ordinal) and no
        given cuts, both run on that GPU (hb_sketch_dense). A matrix whose
        features may take more than 256 bins (max_bin > 256) is binned into
        the CSR index instead (present cells stored, NaN absent: the same
        cuts and trees as the dense index, src/data/ghist.rs:6-21)."""
        if max_bin > 256:
            x = np.ascontiguousarray(x, np.float32)
            present = ~np.isnan(x)
            indptr = np.concatenate([[0], np.cumsum(present.sum(axis=1))]).astype(np.uint64)
            indices = np.nonzero(present)[1].astype(np.uint32)
            return cls.from_csr(indptr, indices, x[present], x.shape[1], max_bin, cuts=cuts)
        if device is not None and cuts is None:
            off, vals, cols, miss, dense = sketch_dense(x, max_bin, device)
            return cls(off, vals, cols, miss, dense)
        off, vals = cuts if cuts is not None else cuts_dense(x, max_bin)
        cols, miss, dense = bin_dense(x, off, vals)
        return cls(off, vals, cols, miss, dense)

    @classmethod
    def from_csr(cls, indptr, indices, values, n_cols, max_bin=256, cuts=None, device=None):
        """DMatrix::from_csr + GHistIndex: absent entries are missing. With
        ``device`` and no given cuts, sketch and bins come from the GPU."""
        if device is not None and cuts is None:
            off, vals, rb, dense = sketch_csr(indptr, indices, values, n_cols, max_bin, device)
            return cls(off, vals, None, None, dense, np.asarray(indptr, np.uint64), rb)
        off, vals = cuts if cuts is not None else cuts_csr(indptr, indices, values, n_cols, max_bin)
        row_ptr, row_bins, dense = bin_csr(indptr, indices, values, n_cols, off, vals)
        return cls(off, vals, None, None, dense, row_ptr, row_bins)

    def shard(self, begin, end):
        """Rows [begin, end) as their own matrix (the cut table is shared)."""
        if self.is_csr:
            a, b = int(self.row_ptr[begin]), int(self.row_ptr[end])
            ptr = self.row_ptr[begin : end + 1] - np.uint64(a)
            full = bool(np.all(np.diff(ptr) == self.n_cols))
            return BinnedMatrix(self.feature_offset, self.cut_values, None, None, full, ptr, self.row_bins[a:b])
        cols = self.columns[:, begin:end]
        n = end - begin
        miss = None
        dense = self.dense
        if not dense:
            bits = np.unpackbits(self.missing.view(np.uint8), bitorder="little").reshape(self.n_cols, -1)
            sub = bits[:, begin:end]
            dense = not sub.any()
            pad = (-n) % 64
            sub = np.concatenate([sub, np.zeros((self.n_cols, pad), np.uint8)], axis=1)
            miss = np.packbits(sub, axis=1, bitorder="little").view(np.uint64)
        return BinnedMatrix(self.feature_offset, self.cut_values, cols, miss, dense)

    @property
    def total_bins(self):
        return int(self.feature_offset[-1])

    def to_c(self):
        g = GHist()
        g.n_rows = self.n_rows
        g.n_cols = self.n_cols
        g.dense = 1 if self.dense else 0
        g.feature_offset = _ptr(self.feature_offset, ctypes.c_uint32)
        g.cut_values = _ptr(self.cut_values, ctypes.c_float)
        if self.is_csr:
            g.columns = None
            g.missing = None
            g.row_ptr = _ptr(self.row_ptr, ctypes.c_uint64)
            g.row_bins = _ptr(self.row_bins, ctypes.c_uint32) if self.row_bins.size else None
            return g
        g.columns = _ptr(self.columns, ctypes.c_uint8)
        g.missing = None if self.missing is None else _ptr(self.missing, ctypes.c_uint64)
        return g


# ---------------------------------------------------------------- engine
class Engine:
    """One GPU's CudaHistBackend + RowEngine (the C ABI's hb_engine)."""

    def __init__(self, device=0):
        h = ctypes.c_void_p()
        _check(lib().hb_engine_create(device, ctypes.byref(h)), "hb_engine_create")
        self.h = h
        self.device = device
        self.matrix = None

    def close(self):
        if self.h:
            lib().hb_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    def _c(self, status, where):
        _check(status, where, self.h)

    def set_shard(self, row_begin, global_rows):
        self._c(lib().hb_engine_set_shard(self.h, row_begin, global_rows), "hb_engine_set_shard")

    def comm_init(self, nranks, rank, uid, global_rows):
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(bytes(uid))
        self._c(lib().hb_comm_init(self.h, nranks, rank, buf, global_rows), "hb_comm_init")

    def upload(self, m):
        self.matrix = m
        g = m.to_c()
        self._c(lib().hb_engine_upload(self.h, ctypes.byref(g)), "hb_engine_upload")

    def upload_dense(self, x, max_bin=256):
        """Sketch, bin and keep a raw dense matrix on this engine's GPU
        (hb_engine_upload_dense); returns the DeviceIndex (cuts and shape)."""
        x = np.ascontiguousarray(x, np.float32)
        n, f = x.shape
        cap = f * max(max_bin, 1)
        off = np.zeros(f + 1, np.uint32)
        vals = np.zeros(cap, np.float32)
        total = ctypes.c_uint64()
        self._c(lib().hb_engine_upload_dense(self.h, _ptr(x, ctypes.c_float), n, f, max_bin, _ptr(off, ctypes.c_uint32),
                                             _ptr(vals, ctypes.c_float), cap, ctypes.byref(total)),
                "hb_engine_upload_dense")
        self.matrix = DeviceIndex(off, vals[: total.value].copy(), n, f)
        return self.matrix

    def upload_csr(self, indptr, indices, values, n_cols, max_bin=256):
        """The CSR twin of upload_dense (hb_engine_upload_csr)."""
        ip, ix, vs = _csr_arrays(indptr, indices, values)
        n = ip.size - 1
        cap = n_cols * max(max_bin, 1)
        off = np.zeros(n_cols + 1, np.uint32)
        vals = np.zeros(cap, np.float32)
        total = ctypes.c_uint64()
        self._c(lib().hb_engine_upload_csr(self.h, _ptr(ip, ctypes.c_uint64), _ptr(ix, ctypes.c_uint32),
                                           _ptr(vs, ctypes.c_float), n, n_cols, max_bin, _ptr(off, ctypes.c_uint32),
                                           _ptr(vals, ctypes.c_float), cap, ctypes.byref(total)),
                "hb_engine_upload_csr")
        self.matrix = DeviceIndex(off, vals[: total.value].copy(), n, n_cols)
        return self.matrix

    # HistogramBackend
    def prepare(self, gpair):
        gp = np.ascontiguousarray(gpair, np.float32).reshape(-1)
        self._c(lib().hb_prepare(self.h, _ptr(gp, ctypes.c_float), gp.size // 2), "hb_prepare")

    def build(self, rows):
        rows = np.ascontiguousarray(rows, np.uint32)
        out = (GradStats * self.matrix.total_bins)()
        self._c(lib().hb_build(self.h, _ptr(rows, ctypes.c_uint32), rows.size, out), "hb_build")
        return np.ctypeslib.as_array(out).view(np.float64).reshape(-1, 2).copy()

    def build_features(self, rows, features):
        """hb_build_features: the histogram of `rows`; the bins of `features`
        are the ones the caller reads."""
        rows = np.ascontiguousarray(rows, np.uint32)
        feats = np.ascontiguousarray(features, np.uint32)
        out = (GradStats * self.matrix.total_bins)()
        self._c(lib().hb_build_features(self.h, _ptr(rows, ctypes.c_uint32), rows.size,
                                        _ptr(feats, ctypes.c_uint32), feats.size, out), "hb_build_features")
        return np.ctypeslib.as_array(out).view(np.float64).reshape(-1, 2).copy()

    def inject_fault(self, after_calls):
        """Arm a host-side fault: the engine's `after_calls`-th checked CUDA
        call outside stream capture fails as a device error (-1 disarms)."""
        self._c(lib().hb_engine_inject_fault(self.h, int(after_calls)), "hb_engine_inject_fault")

    def build_noalloc(self, rows_ptr, n, out_ptr):
        """hb_build_noalloc on caller-owned device buffers: `rows_ptr` holds n
        ascending u32 row ids, `out_ptr` receives total_bins (g, h) f64 pairs."""
        self._c(lib().hb_build_noalloc(self.h, rows_ptr, n, out_ptr), "hb_build_noalloc")

    # RowEngine
    def begin_tree(self, rows):
        rows = np.ascontiguousarray(rows, np.uint32)
        seg = Segment()
        self._c(lib().hb_begin_tree(self.h, _ptr(rows, ctypes.c_uint32), rows.size, ctypes.byref(seg)), "hb_begin_tree")
        return seg

    def root_total(self, seg):
        out = GradStats()
        self._c(lib().hb_root_total(self.h, ctypes.byref(seg), ctypes.byref(out)), "hb_root_total")
        return out.grad, out.hess

    def partition(self, splits):
        arr = (RowSplit * len(splits))()
        for i, (seg, feature, limit, default_left) in enumerate(splits):
            arr[i].seg = seg
            arr[i].feature = feature
            arr[i].limit = limit
            arr[i].default_left = 1 if default_left else 0
        out = (Partitioned * len(splits))()
        self._c(lib().hb_partition(self.h, arr, len(splits), out), "hb_partition")
        return [(out[i].left, out[i].right) for i in range(len(splits))]

    def histograms(self, segs):
        arr = (Segment * len(segs))(*segs)
        out = (GradStats * (len(segs) * self.matrix.total_bins))()
        self._c(lib().hb_histograms(self.h, arr, len(segs), out), "hb_histograms")
        return np.ctypeslib.as_array(out).view(np.float64).reshape(len(segs), -1, 2).copy()

    def rows(self, segs):
        arr = (Segment * len(segs))(*segs)
        total = sum(int(s.len) for s in segs)
        out = np.zeros(max(total, 1), np.uint32)
        self._c(lib().hb_rows(self.h, arr, len(segs), _ptr(out, ctypes.c_uint32)), "hb_rows")
        res, at = [], 0
        for s in segs:
            res.append(out[at : at + int(s.len)].copy())
            at += int(s.len)
        return res

    def load_margins(self, margins):
        m = np.ascontiguousarray(margins, np.float32)
        self._c(lib().hb_load_margins(self.h, _ptr(m, ctypes.c_float), m.size), "hb_load_margins")

    def gradients(self, kind, labels, weights=None, scale_pos_weight=1.0):
        self._labels = np.ascontiguousarray(labels, np.float32)
        self._weights = None if weights is None else np.ascontiguousarray(weights, np.float32)
        loss = DeviceLoss(kind, scale_pos_weight, 1e-16, 0)
        ok = ctypes.c_int32()
        self._c(lib().hb_gradients(self.h, ctypes.byref(loss), _ptr(self._labels, ctypes.c_float),
                                   None if self._weights is None else _ptr(self._weights, ctypes.c_float),
                                   self._labels.size, ctypes.byref(ok)), "hb_gradients")
        return bool(ok.value)

    def add_leaf_values(self, segs, values):
        arr = (Segment * len(segs))(*segs)
        v = np.ascontiguousarray(values, np.float32)
        self._c(lib().hb_add_leaf_values(self.h, arr, _ptr(v, ctypes.c_float), len(segs)), "hb_add_leaf_values")

    def read_margins(self):
        out = np.zeros(self.matrix.n_rows, np.float32)
        self._c(lib().hb_read_margins(self.h, _ptr(out, ctypes.c_float), out.size), "hb_read_margins")
        return out

    def reserve_hists(self, slots):
        ok = ctypes.c_int32()
        self._c(lib().hb_reserve_hists(self.h, slots, ctypes.byref(ok)), "hb_reserve_hists")
        return bool(ok.value)

    def build_resident(self, nodes, siblings=()):
        segs = (Segment * max(len(nodes), 1))(*[s for s, _ in nodes])
        slots = np.array([slot for _, slot in nodes] or [0], np.uint32)
        sib = np.array([v for pair in siblings for v in pair] or [0], np.uint32)
        self._c(lib().hb_build_resident(self.h, segs, _ptr(slots, ctypes.c_uint32), len(nodes),
                                        _ptr(sib, ctypes.c_uint32), len(siblings)), "hb_build_resident")

    def scan_resident(self, reg, requests):
        """requests: (slot, (G, H), features[, directions[, (lower, upper)[, root_gain]]]);
        root_gain defaults to the node's gain at its bounds under `reg`."""
        keep = []
        arr = (ScanRequest * len(requests))()
        for i, req in enumerate(requests):
            slot, total, features = req[:3]
            f = np.ascontiguousarray(features, np.uint32)
            keep.append(f)
            arr[i].slot = slot
            arr[i].n_features = f.size
            arr[i].features = _ptr(f, ctypes.c_uint32)
            if len(req) > 3 and req[3] is not None:
                d = np.ascontiguousarray(req[3], np.int8)
                assert d.size == f.size
                keep.append(d)
                arr[i].directions = d.ctypes.data_as(ctypes.POINTER(ctypes.c_int8))
            arr[i].total = GradStats(*total)
            lo, up = req[4] if len(req) > 4 and req[4] is not None else (-math.inf, math.inf)
            arr[i].lower = lo
            arr[i].upper = up
            arr[i].root_gain = req[5] if len(req) > 5 else node_gain(total, reg, lo, up)
        out = (NodeScan * len(requests))()
        self._c(lib().hb_scan_resident(self.h, ctypes.byref(reg), arr, len(requests), out), "hb_scan_resident")
        return [out[i] for i in range(len(requests))]

    def read_hist(self, slot):
        out = (GradStats * self.matrix.total_bins)()
        self._c(lib().hb_read_hist(self.h, slot, out), "hb_read_hist")
        return np.ctypeslib.as_array(out).view(np.float64).reshape(-1, 2).copy()

    def read_gradients(self):
        out = np.zeros(2 * self.matrix.n_rows, np.float32)
        sg, sh = ctypes.c_int32(), ctypes.c_int32()
        self._c(lib().hb_read_gradients(self.h, _ptr(out, ctypes.c_float), self.matrix.n_rows,
                                        ctypes.byref(sg), ctypes.byref(sh)), "hb_read_gradients")
        return out.reshape(-1, 2), sg.value, sh.value

    # whole-tree growth
    def grow_tree(self, params):
        cap = params.tree_slots()
        nodes = np.zeros(cap, NODE_DTYPE)
        n = ctypes.c_uint32()
        p = params.to_c()
        self._c(lib().hb_grow_tree(self.h, ctypes.byref(p), nodes.ctypes.data_as(ctypes.POINTER(TreeNode)), cap,
                                   ctypes.byref(n)), "hb_grow_tree")
        return nodes[: n.value].copy()

    def train(self, params, labels, rounds, base_margin):
        self.train_begin(labels, base_margin)
        return self.train_rounds(params, rounds)

    def train_begin(self, labels, base_margin):
        self._labels = np.ascontiguousarray(labels, np.float32)
        self._classes = 1
        self._c(lib().hb_train_begin(self.h, _ptr(self._labels, ctypes.c_float), self._labels.size,
                                     float(base_margin)), "hb_train_begin")

    def train_begin_classes(self, labels, base_margins):
        """A multi:softmax run: labels are class ids, one base margin per class."""
        self._labels = np.ascontiguousarray(labels, np.float32)
        self._bases = np.ascontiguousarray(base_margins, np.float32)
        self._classes = self._bases.size
        self._c(lib().hb_train_begin_classes(self.h, _ptr(self._labels, ctypes.c_float), self._labels.size,
                                             _ptr(self._bases, ctypes.c_float), self._classes),
                "hb_train_begin_classes")

    def train_rounds(self, params, rounds):
        """`rounds` rounds; returns every tree's nodes and the tree offsets
        (a softmax round's trees are its classes', in class order)."""
        trees = rounds * getattr(self, "_classes", 1)
        cap = max(trees, 1) * params.tree_slots()
        nodes = np.zeros(cap, NODE_DTYPE)
        tree_ptr = np.zeros(trees + 1, np.uint64)
        p = params.to_c()
        self._c(lib().hb_train_rounds(self.h, ctypes.byref(p), rounds, nodes.ctypes.data_as(ctypes.POINTER(TreeNode)),
                                      cap, _ptr(tree_ptr, ctypes.c_uint64)), "hb_train_rounds")
        return nodes[: int(tree_ptr[-1])].copy(), tree_ptr

    def reset_stats(self, timing=0):
        """timing: 0 off, 1 events around the histogram kernel, 2 around every family."""
        self._c(lib().hb_engine_reset_stats(self.h, int(timing)), "hb_engine_reset_stats")

    def stats(self):
        st = EngineStats()
        self._c(lib().hb_engine_get_stats(self.h, ctypes.byref(st)), "hb_engine_get_stats")
        return {
            "ms": {k: st.ms[i] for i, k in enumerate(TIMER_NAMES)},
            "timed_launches": {k: int(st.timed_launches[i]) for i, k in enumerate(TIMER_NAMES)},
            "kernel_launches": int(st.kernel_launches),
            "rows_built_contiguous": int(st.rows_built_contiguous),
            "rows_built_gathered": int(st.rows_built_gathered),
            "rounds": int(st.rounds),
            "last_rounds_ms": float(st.last_rounds_ms),
        }

    def stream(self):
        s = ctypes.c_void_p()
        self._c(lib().hb_engine_stream(self.h, ctypes.byref(s)), "hb_engine_stream")
        return s.value


# ---------------------------------------------------------------- model
def softmax_intercepts(labels, n_classes):
    """multi:softmax class intercepts (objective/multiclass.rs:68 in its
    precision): class counts accumulated in f32 (saturating at 2^24 as
    sequential f32 adds of 1 do), divided by the f64 row count rounded to
    f32 first, ln(p + 1e-6) with the C library's logf, centred by the f32
    mean of m / k summed in class order."""
    y = np.asarray(labels, np.float32)
    ids = y[(y >= 0) & (y < n_classes)].astype(np.int64)
    counts = np.minimum(np.bincount(ids, minlength=n_classes), 2**24).astype(np.float32)
    inv = 1.0 / np.float64(np.float32(len(y)))
    m = [np.float32(_libm().logf(float(np.float32(np.float32(np.float64(c) * inv) + np.float32(1e-6)))))
         for c in counts]
    kk = np.float32(n_classes)
    mean = np.float32(0.0)
    for v in m:
        mean = np.float32(mean + np.float32(v / kk))
    return np.array([np.float32(v - mean) for v in m], np.float32)


def base_margin(params, labels):
    """The intercept (train.rs:408 `initial_intercepts`): the label mean for
    squared error, its logit for logistic (objective/mod.rs:645,
    classification.rs:69), computed as the reference does in f64 then f32."""
    y = np.asarray(labels, np.float32)
    if not math.isnan(params.base_score):
        p = np.float32(params.base_score)
    elif len(y) == 0:
        p = np.float32(0.0)
    else:
        # a sequential f64 sum of y / n (np.cumsum adds in order)
        p = np.float32(np.cumsum(y.astype(np.float64) / float(len(y)))[-1])
    if params.loss_kind() == HB_LOSS_LOGISTIC and params.objective != "binary:logitraw":
        eps = np.float32(1e-6)
        p = np.minimum(np.maximum(p, eps), np.float32(1.0) - eps)
        # -(1/p - 1).ln() in f32 with the C library's logf, as Rust's f32::ln
        return np.float32(-_libm().logf(float(np.float32(np.float32(1.0) / p - np.float32(1.0)))))
    return np.float32(p)


_libm_handle = None


def _libm():
    global _libm_handle
    if _libm_handle is None:
        _libm_handle = ctypes.CDLL("libm.so.6")
        _libm_handle.logf.restype = ctypes.c_float
        _libm_handle.logf.argtypes = [ctypes.c_float]
    return _libm_handle


@dataclass
class Model:
    """A trained ensemble: nodes back to back, per-tree offsets, the base
    margin (one per output). Tree t adds to output
    (t // num_parallel_tree) % outputs, scaled by tree_weights[t] when the
    model has per-tree weights (a DART model read from a file)."""

    nodes: np.ndarray
    tree_ptr: np.ndarray
    base: object
    n_features: int
    num_parallel_tree: int = 1
    tree_weights: object = None

    def bases(self):
        return np.atleast_1d(np.asarray(self.base, np.float32))

    def tree_layout(self):
        """(output of each tree, weight of each tree or None), the layout
        BoostedModel::predict_margin walks (model/predict.rs:701)."""
        n_trees = len(self.tree_ptr) - 1
        outs = (np.arange(n_trees) // max(int(self.num_parallel_tree), 1)) % self.bases().size
        w = None if self.tree_weights is None else np.asarray(self.tree_weights, np.float32)
        if w is not None and w.size != n_trees:
            raise ValueError("tree_weights needs one weight per tree")
        return outs.astype(np.uint32), w

    def predictor(self, device=0):
        outs, w = self.tree_layout()
        return Predictor(self.nodes, self.tree_ptr, self.bases(), self.n_features,
                         tree_output=outs if self.num_parallel_tree != 1 else None, tree_weight=w,
                         device=device)

    def predict_margin(self, x, device=0):
        p = self.predictor(device)
        try:
            out = p.predict_margin(x)
            return out[:, 0] if out.shape[1] == 1 else out
        finally:
            p.close()

    def save_native(self, path, params, format="json"):
        """Write the reference's native model file (loads unchanged in
        hessboost's Python and Rust APIs): `format` "json" (the pretty
        serde form) or "binary" (the checksummed section container as a
        zstd frame, BoostedModel::save with ModelFormat::Binary); `params`
        the TrainingParams the model was trained with."""
        from . import model_io

        softmax = params.loss_kind() == HB_LOSS_SOFTMAX
        kw = dict(objective=params.objective, num_class=params.num_class if softmax else 0,
                  scale_pos_weight=params.scale_pos_weight,
                  max_delta_step=float(np.float32(params.max_delta_step)),
                  num_parallel_tree=self.num_parallel_tree, tree_weights=self.tree_weights)
        if format == "json":
            data = model_io.to_native_json(self.nodes, self.tree_ptr, self.bases(), self.n_features,
                                           **kw).encode()
        elif format == "binary":
            data = model_io.to_native_binary(self.nodes, self.tree_ptr, self.bases(), self.n_features, **kw)
        else:
            raise ValueError(f"unknown model format {format!r} (json or binary)")
        with open(path, "wb") as fh:
            fh.write(data)

    @staticmethod
    def load_native(path):
        """A gbtree model (numeric scalar-leaf trees) from a native JSON or
        binary file, told apart by their first bytes (ModelFormat::detect)."""
        from . import model_io

        with open(path, "rb") as fh:
            data = fh.read()
        kind = model_io.detect(data)
        if kind == "binary":
            nodes, ptr, base, nf, fields = model_io.from_native_binary(data)
        elif kind == "json":
            nodes, ptr, base, nf, fields = model_io.from_native_json(data.decode())
        else:
            raise ValueError(f"{path}: not a native hessboost model file")
        npt = int(fields.get("num_parallel_tree") or 1)
        weights = np.asarray(fields.get("tree_weights") or np.ones(len(ptr) - 1), np.float32)
        if fields.get("best_iteration") is not None:
            # predictions stop at the best iteration (model/predict.rs:701)
            n = (int(fields["best_iteration"]) + 1) * int(fields["n_outputs"]) * npt
            nodes, ptr, weights = nodes[: int(ptr[n])], ptr[: n + 1], weights[:n]
        return Model(nodes, ptr, base if base.size > 1 else float(base[0]), nf, num_parallel_tree=npt,
                     tree_weights=None if np.all(weights == 1.0) else weights)


def train(params, x=None, y=None, rounds=10, device=0, matrix=None, engine=None):
    """Train ``rounds`` rounds on one GPU (train_trees, train.rs:222).

    With a raw matrix ``x`` (and no ``matrix``) the engine sketches and bins
    it on its own GPU (hb_engine_upload_dense); where the device sketch
    refuses the input (a feature with 2^24 or more present values), the
    reference's host sketch bins it instead, with the same cuts."""
    params.validate()
    if x is not None or matrix is not None:
        params.validate_for((matrix.n_cols if matrix is not None else np.asarray(x).shape[1]))
    y = np.ascontiguousarray(y, np.float32)
    eng = engine or Engine(device)
    try:
        if matrix is None:
            try:
                matrix = eng.upload_dense(x, params.max_bin)
            except HbError as err:
                if err.status != HB_REFUSED:
                    raise
                matrix = BinnedMatrix.from_dense(x, params.max_bin)
                eng.upload(matrix)
        else:
            eng.upload(matrix)
        if params.loss_kind() == HB_LOSS_SOFTMAX:
            if math.isnan(params.base_score):
                base = softmax_intercepts(y, params.num_class)
            else:
                base = np.full(params.num_class, params.base_score, np.float32)
            eng.train_begin_classes(y, base)
            nodes, tree_ptr = eng.train_rounds(params, rounds)
            return Model(nodes, tree_ptr, base, matrix.n_cols)
        base = base_margin(params, y)
        nodes, tree_ptr = eng.train(params, y, rounds, base)
    finally:
        if engine is None:
            eng.close()
    return Model(nodes, tree_ptr, float(base), matrix.n_cols)


class Predictor:
    """BoostedModel::to_cuda's GpuModel (src/backend/cuda/predict.rs:501)."""

    def __init__(self, nodes, tree_ptr, base, n_features, tree_output=None, tree_weight=None, device=0):
        nodes = np.ascontiguousarray(nodes, NODE_DTYPE)
        tree_ptr = np.ascontiguousarray(tree_ptr, np.uint64)
        base = np.ascontiguousarray(base, np.float32)
        self.n_outputs = base.size
        self.n_features = n_features
        to = None if tree_output is None else np.ascontiguousarray(tree_output, np.uint32)
        tw = None if tree_weight is None else np.ascontiguousarray(tree_weight, np.float32)
        h = ctypes.c_void_p()
        _check(lib().hb_predictor_create(device, nodes.ctypes.data_as(ctypes.POINTER(TreeNode)), _ptr(tree_ptr, ctypes.c_uint64),
                                         len(tree_ptr) - 1, None if to is None else _ptr(to, ctypes.c_uint32),
                                         None if tw is None else _ptr(tw, ctypes.c_float), base.size,
                                         _ptr(base, ctypes.c_float), n_features, ctypes.byref(h)), "hb_predictor_create")
        self.h = h

    def predict_margin(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros((x.shape[0], self.n_outputs), np.float32)
        _check(lib().hb_predict_margin(self.h, _ptr(x, ctypes.c_float), x.shape[0], _ptr(out, ctypes.c_float)),
               "hb_predict_margin")
        return out

    def predict_margin_into(self, x, out):
        """hb_predict_margin from host rows `x` (n x n_features f32, C order)
        into the host array `out` (n x n_outputs f32); pinned buffers make
        the copies asynchronous."""
        if x.dtype != np.float32 or not x.flags.c_contiguous or out.dtype != np.float32:
            raise ValueError("x and out must be C-contiguous float32")
        if out.size != x.shape[0] * self.n_outputs:
            raise ValueError("out must hold n_rows x n_outputs values")
        _check(lib().hb_predict_margin(self.h, _ptr(x, ctypes.c_float), x.shape[0], _ptr(out, ctypes.c_float)),
               "hb_predict_margin")

    def predict_margin_device(self, d_rows, n_rows, d_out, stream=None):
        _check(lib().hb_predict_margin_device(self.h, d_rows, n_rows, d_out, stream), "hb_predict_margin_device")

    def close(self):
        if self.h:
            lib().hb_predictor_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass
