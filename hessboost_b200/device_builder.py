"""Device-resident rounds through the RowEngine entry points, call for call as
the reference's unchanged trainer makes them.

`device_round` (src/training/round.rs:117-160) with
`HistTreeBuilder::build_on_device` (src/tree/builder/hist/device.rs:147-300,
depthwise growth with resident histograms: `resident_children` :451,
`resident_search` :553, `resident_best` :642) is restated here over this
library's C ABI:

  gradients -> begin_tree -> root_total -> reserve_hists -> build_resident
  (root) -> scan_resident (root), then per level partition (every split of
  the level) -> build_resident (the smaller children, their siblings by
  subtraction) -> scan_resident (every child), and add_leaf_values.

The host keeps the tree (RegTree) and the per-node statistics and monotone
bounds, decodes each NodeScan into a split exactly as `resident_best` does
(children from `acc` and the node total, weights from the host scorer), and
finishes the leaves (`finalize_leaf_values`, `scale_leaves`). This is the
path a drop-in binding under the reference's `train()` runs; the trees it
grows equal those of the whole-round entry point (hb_train_rounds) bit for
bit, because every histogram sum is an integer the f64 ABI carries exactly.
"""

import math
import time

import numpy as np

from . import (HB_LOSS_LOGISTIC, HB_LOSS_SQUARED_ERROR, HB_SCAN_EMPTY, NODE_DTYPE, HbError,
               node_gain)

BELOW_ALL = float(np.float32(-3.40282347e38))  # src/tree/builder/mod.rs:308 (f32::MIN)
RT_EPS = 1e-6                                   # src/lib.rs:366


def _threshold_l1(g, alpha):  # src/tree/gain.rs:96
    if g > alpha:
        return g - alpha
    if g < -alpha:
        return g + alpha
    return 0.0


def xgb_weight(g, h, reg, lower, upper):
    """shared.rs:113: the f64 weight rounded to f32, clamped to the f32 bounds."""
    if h <= 0.0:
        w = 0.0
    else:
        w = -_threshold_l1(g, reg.alpha) / (h + reg.lambda_)
        if reg.max_delta_step != 0.0 and abs(w) > reg.max_delta_step:
            w = math.copysign(reg.max_delta_step, w)
    w32 = np.float32(w)
    lo, up = np.float32(lower), np.float32(upper)
    return lo if w32 < lo else (up if w32 > up else w32)


def calc_weight_bounded(g, h, reg, lower, upper):
    """constraints.rs:70 over gain.rs:107 (leaf values; min_child_weight
    applies), clamped to the bounds in f64."""
    if h < reg.min_child_weight or h <= 0.0:
        w = 0.0
    else:
        w = -_threshold_l1(g, reg.alpha) / (h + reg.lambda_)
        if reg.max_delta_step > 0.0:
            w = min(max(w, -reg.max_delta_step), reg.max_delta_step)
    return lower if w < lower else (upper if w > upper else w)


def child_bounds(lower, upper, direction, wl, wr):
    """constraints.rs:82 (f64::midpoint of the bounded child weights)."""
    if direction == 0:
        return (lower, upper), (lower, upper)
    a, b = float(wl), float(wr)
    mid = (a + b) / 2.0 if max(abs(a), abs(b)) <= 1.7976931348623157e308 / 2 else a / 2.0 + b / 2.0
    if direction > 0:
        return (lower, mid), (mid, upper)
    return (mid, upper), (lower, mid)


class _Slots:
    """device.rs:69 `Slots`: histogram slots taken from a free list first."""

    def __init__(self, reserved):
        self.next, self.reserved, self.free = 0, reserved, []

    def take(self):
        if self.free:
            return self.free.pop()
        if self.next >= self.reserved:
            raise HbError(1, "slots", "more histogram slots than reserved")
        self.next += 1
        return self.next - 1

    def release(self, slot):
        if slot is not None:
            self.free.append(slot)


class RowEngineTrainer:
    """`device_round` over an Engine whose matrix is uploaded and whose
    margins are loaded: one round per `round()` call, depthwise growth."""

    def __init__(self, engine, params, labels):
        params.validate()
        if params.grow_policy != "depthwise" or params.max_depth < 1:
            raise ValueError("RowEngineTrainer grows depthwise trees of bounded depth")
        self.e = engine
        self.p = params
        self.kind = params.loss_kind()
        if self.kind not in (HB_LOSS_SQUARED_ERROR, HB_LOSS_LOGISTIC):
            raise ValueError("single-output objectives only")
        self.labels = np.ascontiguousarray(labels, np.float32)
        m = engine.matrix
        self.fo = np.asarray(m.feature_offset, np.int64)
        self.cuts = np.asarray(m.cut_values, np.float32)
        self.n_cols = int(m.n_cols)
        self.n_rows = int(m.n_rows)
        self.all_rows = np.arange(self.n_rows, dtype=np.uint32)
        self.reg = params.reg()
        self.mono = [int(v) for v in params.monotone_constraints] + [0] * self.n_cols
        self.features = np.arange(self.n_cols, dtype=np.uint32)
        self.dirs = np.array(self.mono[: self.n_cols], np.int8)
        self.calls = 0
        self.seconds = {}  # host wall time by entry point
        # resident_slots (device.rs:123): 2^(max_depth - 1) for depthwise
        self.n_slots = min(1 << (params.max_depth - 1), max(self.n_rows, 1))

    def _t(self, name, fn, *a, **kw):
        """One C-ABI call, counted and timed (host wall clock)."""
        t0 = time.perf_counter()
        out = fn(*a, **kw)
        self.seconds[name] = self.seconds.get(name, 0.0) + time.perf_counter() - t0
        self.calls += 1
        return out

    # -- one node's scan decoded (resident_best, device.rs:642) -------------
    def _best(self, scan, total, bounds):
        if scan.kind == HB_SCAN_EMPTY:
            return None
        f = int(scan.feature)
        first = int(self.fo[f])
        acc = (scan.acc.grad, scan.acc.hess)
        rest = (total[0] - acc[0], total[1] - acc[1])
        if scan.backward:
            left, right = rest, acc
            bin_ = -1 if scan.offset == 0 else first + int(scan.offset) - 1
        else:
            left, right = acc, rest
            bin_ = first + int(scan.offset)
        wl = xgb_weight(left[0], left[1], self.reg, *bounds)
        wr = xgb_weight(right[0], right[1], self.reg, *bounds)
        return dict(feature=f, bin=bin_, default_left=bool(scan.backward), left=left, right=right,
                    wl=wl, wr=wr, loss=np.float32(scan.loss_chg))

    def _valid(self, b):  # builder/mod.rs:167 `BestSplit::valid`
        if b is None:
            return False
        mcw = self.reg.min_child_weight
        return (float(b["loss"]) > RT_EPS and float(b["loss"]) >= float(np.float32(self.p.gamma))
                and b["left"][1] > 0.0 and b["right"][1] > 0.0 and b["left"][1] >= mcw and b["right"][1] >= mcw)

    def _scan(self, nodes):
        """resident_search (device.rs:553): one request per node."""
        if not nodes:
            return []
        reqs = [(n["slot"], n["stats"], self.features, self.dirs, n["bounds"],
                 node_gain(n["stats"], self.reg, *n["bounds"])) for n in nodes]
        scans = self._t("scan_resident", self.e.scan_resident, self.reg, reqs)
        return [self._best(s, n["stats"], n["bounds"]) for s, n in zip(scans, nodes)]

    def round(self):
        """One boosting round; returns the tree as an hb_tree_node array."""
        e = self.e
        if not self._t("gradients", e.gradients, self.kind, self.labels, scale_pos_weight=self.p.scale_pos_weight):
            raise HbError(1, "gradients", "non-finite gradients: the host grows this round")
        seg = self._t("begin_tree", e.begin_tree, self.all_rows)
        g, h = self._t("root_total", e.root_total, seg)
        if not self._t("reserve_hists", e.reserve_hists, self.n_slots):
            raise HbError(1, "reserve_hists", "the device declined the slots")
        slots = _Slots(self.n_slots)
        root_slot = slots.take()
        self._t("build_resident", e.build_resident, [(seg, root_slot)])
        inf = (-math.inf, math.inf)
        nodes = [dict(nid=0, depth=0, seg=seg, slot=root_slot, stats=(g, h), bounds=inf)]
        nodes[0]["best"] = self._scan(nodes)[0]
        tree = [dict(left=-1, right=-1, feature=0, cond=0.0, default_left=1,
                     leaf=np.float32(0.0), hess=np.float32(h), gain=np.float32(0.0), bin=-1)]
        stats, bounds = [(g, h)], [inf]
        leaves = []
        limit = self.p.max_depth
        frontier, depth = nodes, 0
        while depth < limit and frontier:
            pending = []
            for n in frontier:
                b = n["best"]
                if self._valid(b):
                    # prepare_split (hist/mod.rs:639): expand, child bounds
                    left_id = len(tree)
                    t = tree[n["nid"]]
                    t.update(left=left_id, right=left_id + 1, feature=b["feature"],
                             cond=BELOW_ALL if b["bin"] < 0 else float(self.cuts[b["bin"]]),
                             default_left=1 if b["default_left"] else 0, gain=b["loss"], bin=b["bin"])
                    for st, w in ((b["left"], b["wl"]), (b["right"], b["wr"])):
                        tree.append(dict(left=-1, right=-1, feature=0, cond=0.0, default_left=1, leaf=w,
                                         hess=np.float32(st[1]), gain=np.float32(0.0), bin=-1))
                    lb, rb = child_bounds(*n["bounds"], self.mono[b["feature"]], b["wl"], b["wr"])
                    stats += [b["left"], b["right"]]
                    bounds += [lb, rb]
                    pending.append((n, left_id, lb, rb, depth + 1 >= limit))
                else:
                    slots.release(n["slot"])
                    leaves.append((n["nid"], n["seg"]))
            frontier = self._children(pending, slots)
            depth += 1
        leaves += [(n["nid"], n["seg"]) for n in frontier]
        # finalize_leaf_values (shared.rs:174) then scale_leaves(eta)
        eta = np.float32(self.p.eta)
        for nid, t in enumerate(tree):
            if t["left"] == -1:
                w = np.float32(calc_weight_bounded(*stats[nid], self.reg, *bounds[nid]))
                t["leaf"] = np.float32(w * eta)
        self._t("add_leaf_values", e.add_leaf_values, [s for _, s in leaves], [tree[nid]["leaf"] for nid, _ in leaves])
        out = np.zeros(len(tree), NODE_DTYPE)
        for i, t in enumerate(tree):
            out[i] = (t["left"], t["right"], t["feature"], t["cond"], t["default_left"], t["leaf"],
                      t["hess"], t["gain"], t["bin"], 0)
        return out

    def _children(self, pending, slots):
        """resident_children (device.rs:451)."""
        if not pending:
            return []
        e = self.e
        splits = []
        for n, _, _, _, _ in pending:
            b = n["best"]
            first = int(self.fo[b["feature"]])
            limit = 0 if b["bin"] < 0 else b["bin"] + 1 - first
            splits.append((n["seg"], b["feature"], limit, b["default_left"]))
        parts = self._t("partition", e.partition, splits)
        for n, _, _, _, terminal in pending:
            if terminal:
                slots.release(n["slot"])
        build, siblings, kids = [], [], []
        for (n, left_id, lb, rb, terminal), (lseg, rseg) in zip(pending, parts):
            b = n["best"]
            kl = dict(nid=left_id, seg=lseg, stats=b["left"], bounds=lb, slot=None)
            kr = dict(nid=left_id + 1, seg=rseg, stats=b["right"], bounds=rb, slot=None)
            if not terminal:
                built = slots.take()
                left_smaller = lseg.len <= rseg.len
                build.append((lseg if left_smaller else rseg, built))
                siblings.append((n["slot"], built))
                kl["slot"], kr["slot"] = (built, n["slot"]) if left_smaller else (n["slot"], built)
            kids.append((kl, kr, terminal))
        if build:
            self._t("build_resident", e.build_resident, build, siblings=siblings)
        searched = [k for kl, kr, t in kids if not t for k in (kl, kr)]
        for k, best in zip(searched, self._scan(searched)):
            k["best"] = best
        out = []
        for kl, kr, t in kids:
            if t:
                kl["best"] = kr["best"] = None
            out += [kl, kr]
        return out
