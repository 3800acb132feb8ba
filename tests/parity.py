"""North-star parity of GPU-trained forests against the CPU oracle.

TEST INFRASTRUCTURE ONLY: imported by tests/ and by bench.py's parity leg,
never by the product package. The criteria:

* against the oracle's fixed-point mode (the same int64 sums by
  construction): every node field bit for bit;
* against the oracle's f64 mode (the reference's own summation order):
  identical tree structure (split feature, bin threshold, default
  direction) except exact-gain ties, leaf values within 1e-5 relative, leaf
  indices bit-exact (implied: identical structure and bins route every row
  the same way), predictions within 1e-6 relative.

Tolerances, written once here and used by every caller:
  LEAF_RTOL = 1e-5 with LEAF_ATOL = 1e-7 (a leaf of |w| < 1e-2 is compared
  to 1e-5 of 1e-2; leaves are f32 of magnitude eta * G / (H + lambda));
  MARGIN_RTOL = 1e-6 with MARGIN_ATOL = 1e-7 (margins near zero);
  TIE_RTOL = 1e-5: a structural difference counts as a tie when the two
  chosen splits' gains agree to 1e-5 relative (f32 scores of equal f64
  gains rounded apart).

`forced_f64_rounds` compares round by round with both sides started from
the same margins every round (the oracle's f64 trajectory), so a tie in
round r does not hide rounds r+1, r+2, ...: every later tree is compared
from identical inputs.
"""

import numpy as np

LEAF_RTOL, LEAF_ATOL = 1e-5, 1e-7
MARGIN_RTOL, MARGIN_ATOL = 1e-6, 1e-7
TIE_RTOL = 1e-5

STRUCT_FIELDS = ("split_feature", "split_bin", "default_left")
INT_FIELDS = ("left", "right", "split_feature", "default_left", "split_bin")
F32_FIELDS = ("split_cond", "leaf_value", "sum_hess", "split_gain")


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def trees(nodes, ptr):
    return [nodes[int(ptr[i]):int(ptr[i + 1])] for i in range(len(ptr) - 1)]


def forest_bit_exact(nodes, ptr, onodes, optr):
    """(True, "") when every node field of every tree is equal bit for bit,
    else (False, where)."""
    if len(ptr) != len(optr) or not np.array_equal(np.asarray(ptr, np.uint64), np.asarray(optr, np.uint64)):
        return False, "tree sizes differ"
    for k in INT_FIELDS:
        if not np.array_equal(nodes[k], onodes[k]):
            return False, k
    for k in F32_FIELDS:
        if not np.array_equal(_bits(nodes[k]), _bits(onodes[k])):
            return False, k
    return True, ""


def first_structural_difference(a, b):
    """Index of the first node whose split (feature, bin, direction) or
    leafness differs between trees a and b, else None."""
    n = min(len(a), len(b))
    for i in range(n):
        if (a[i]["left"] == -1) != (b[i]["left"] == -1):
            return i
        if a[i]["left"] != -1 and any(a[i][k] != b[i][k] for k in STRUCT_FIELDS):
            return i
    return None if len(a) == len(b) else n


def compare_tree_f64(g, o):
    """One GPU tree `g` against the oracle's f64-mode tree `o` grown from
    the same margins. Returns a dict: structure equal, tie (a structural
    difference whose two gains agree to TIE_RTOL), leaf error (over the
    nodes before the first difference)."""
    k = first_structural_difference(g, o)
    upto = len(g) if k is None else k
    gl, ol = g[:upto], o[:upto]
    leaf = gl["left"] == -1
    lg, lo = gl["leaf_value"][leaf].astype(np.float64), ol["leaf_value"][leaf].astype(np.float64)
    err = np.abs(lg - lo)
    leaf_ok = bool(np.all(err <= LEAF_ATOL + LEAF_RTOL * np.abs(lo)))
    rel = float(np.max(err / np.maximum(np.abs(lo), 1e-30))) if err.size else 0.0
    tie, gain_rel = False, None
    if k is not None and k < min(len(g), len(o)):
        a, b = float(o[k]["split_gain"]), float(g[k]["split_gain"])
        gain_rel = abs(a - b) / max(abs(a), 1e-30)
        tie = gain_rel <= TIE_RTOL
    return {"structure_equal": k is None, "first_difference": k, "tie": tie, "gain_rel": gain_rel,
            "leaf_ok": leaf_ok, "leaf_max_rel": rel}


def margins_ok(got, want):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    err = np.abs(got - want)
    ok = bool(np.all(err <= MARGIN_ATOL + MARGIN_RTOL * np.abs(want)))
    nz = np.abs(want) > 1e-3
    rel = float(np.max(err[nz] / np.abs(want[nz]))) if nz.any() else 0.0
    exact = float(np.mean(_bits(got.astype(np.float32)) == _bits(want.astype(np.float32))))
    return ok, rel, exact


def forced_f64_rounds(engine, params, trainer_f64, rounds):
    """`rounds` rounds, each grown by the GPU engine and by the oracle's
    f64-mode trainer from the same margins (the oracle's trajectory). The
    engine must have had train_begin; the trainer is an oracle Trainer in
    f64 mode on the same matrix and labels. Returns a summary dict."""
    out = {"rounds": 0, "trees_structure_equal": 0, "ties": [], "not_ties": [], "leaf_ok": True,
           "leaf_max_rel": 0.0, "margins_ok": True, "margin_max_rel": 0.0, "margin_bit_exact_frac": 1.0}
    for r in range(rounds):
        m = trainer_f64.margins()[:, 0].copy()
        engine.load_margins(m)
        gn, gp = engine.train_rounds(params, 1)
        gm = engine.read_margins()
        on, op = trainer_f64.rounds(1)
        om = trainer_f64.margins()[:, 0]
        c = compare_tree_f64(gn[int(gp[0]):int(gp[1])], on[int(op[0]):int(op[1])])
        out["rounds"] += 1
        out["leaf_ok"] &= c["leaf_ok"]
        out["leaf_max_rel"] = max(out["leaf_max_rel"], c["leaf_max_rel"])
        if c["structure_equal"]:
            out["trees_structure_equal"] += 1
            ok, rel, exact = margins_ok(gm, om)
            out["margins_ok"] &= ok
            out["margin_max_rel"] = max(out["margin_max_rel"], rel)
            out["margin_bit_exact_frac"] = min(out["margin_bit_exact_frac"], exact)
        elif c["tie"]:
            out["ties"].append({"round": r, "node": c["first_difference"], "gain_rel": c["gain_rel"]})
        else:
            out["not_ties"].append({"round": r, "node": c["first_difference"], "gain_rel": c["gain_rel"]})
    out["pass"] = bool(out["leaf_ok"] and out["margins_ok"] and not out["not_ties"])
    return out


def compare_forests(nodes, ptr, onodes, optr):
    """Tree-by-tree north-star comparison of two forests grown from the same
    margins (one round, or the first round of several): structure equal
    except ties, leaf error before the first difference of each tree."""
    out = {"trees": 0, "trees_structure_equal": 0, "ties": [], "not_ties": [], "leaf_ok": True,
           "leaf_max_rel": 0.0}
    for t, (g, o) in enumerate(zip(trees(nodes, ptr), trees(onodes, optr))):
        c = compare_tree_f64(g, o)
        out["trees"] += 1
        out["leaf_ok"] &= c["leaf_ok"]
        out["leaf_max_rel"] = max(out["leaf_max_rel"], c["leaf_max_rel"])
        if c["structure_equal"]:
            out["trees_structure_equal"] += 1
        elif c["tie"]:
            out["ties"].append({"tree": t, "node": c["first_difference"], "gain_rel": c["gain_rel"]})
        else:
            out["not_ties"].append({"tree": t, "node": c["first_difference"], "gain_rel": c["gain_rel"]})
    out["pass"] = bool(out["leaf_ok"] and not out["not_ties"] and len(ptr) == len(optr))
    return out
