"""Native JSON model files: the reference's `BoostedModel` serde form
(src/model/serde.rs:12 `SerializedBoostedModel`, fields in that order),
written pretty the way its JSON writer writes them (src/model/io.rs:101:
two-space indent, one element per line, f32 and f64 values in their
shortest round-trip decimal form). A model trained here and saved with
`save_native` loads unchanged in the reference's Python and Rust APIs; a
reference JSON model loads here with `load_native`.

Only what this library trains is written: numeric scalar-leaf trees of
reg:squarederror, binary:logistic and multi:softmax (no categories, vector
leaves, linear leaves, DART weights or boosters besides gbtree).
"""

import json

import numpy as np

from . import NODE_DTYPE

# StoredObjectiveParams (src/model/objective.rs:166) as the 0.4.9 files
# store them; the loader fills any missing one from the objective's defaults
_DEFAULT_PARAMS = [
    ("scale_pos_weight", ("f32", 1.0)),
    ("max_delta_step", ("f64", 0.0)),
    ("tweedie_variance_power", ("f64", 1.5)),
    ("huber_slope", ("f32", 1.0)),
    ("lambdarank_num_pair_per_sample", ("int", 32)),
    ("quantile_alpha", ("raw", [])),
    ("expectile_alpha", ("raw", [])),
    ("aft_loss_distribution", ("str", "normal")),
    ("aft_loss_distribution_scale", ("f64", 1.0)),
    ("dist_gradient", ("str", "fisher")),
    ("dist_split_direction", ("str", "random")),
    ("distribution", ("raw", None)),
]


def _shortest(v, single):
    """Shortest round-trip decimal of an f32 (single) or f64, laid out as
    the ryu algorithm's writer lays it out (Ulf Adams, "Ryu: fast
    float-to-string conversion", PLDI 2018): plain decimal while the
    decimal exponent allows it, else d.ddde<exp>."""
    x = np.float32(v) if single else np.float64(v)
    if not np.isfinite(x):
        raise ValueError("non-finite values have no JSON form")
    if x == 0:
        return "-0.0" if np.signbit(x) else "0.0"
    s = np.format_float_scientific(x, unique=True, trim="-")
    mant, exp = s.split("e")
    sign = "-" if mant.startswith("-") else ""
    digits = mant.lstrip("-").replace(".", "")
    e10 = int(exp) - (len(digits) - 1)  # x = digits * 10^e10
    n = len(digits)
    kk = n + e10                        # 10^(kk-1) <= |x| < 10^kk
    limit = 13 if single else 16
    if 0 <= e10 and kk <= limit:
        out = digits + "0" * e10 + ".0"
    elif 0 < kk <= limit:
        out = digits[:kk] + "." + digits[kk:]
    elif -6 < kk <= 0:
        out = "0." + "0" * (-kk) + digits
    elif n == 1:
        out = digits + "e" + str(kk - 1)
    else:
        out = digits[0] + "." + digits[1:] + "e" + str(kk - 1)
    return sign + out


class _F32:
    def __init__(self, v):
        self.v = v


class _F64:
    def __init__(self, v):
        self.v = v


def _write(v, indent, out):
    pad = "  " * indent
    if isinstance(v, _F32):
        out.append(_shortest(v.v, True))
    elif isinstance(v, _F64):
        out.append(_shortest(v.v, False))
    elif v is None:
        out.append("null")
    elif isinstance(v, bool):
        out.append("true" if v else "false")
    elif isinstance(v, (int, np.integer)):
        out.append(str(int(v)))
    elif isinstance(v, str):
        out.append(json.dumps(v))
    elif isinstance(v, list):
        if not v:
            out.append("[]")
            return
        out.append("[\n")
        for i, item in enumerate(v):
            out.append(pad + "  ")
            _write(item, indent + 1, out)
            out.append(",\n" if i + 1 < len(v) else "\n")
        out.append(pad + "]")
    elif isinstance(v, dict):
        if not v:
            out.append("{}")
            return
        out.append("{\n")
        items = list(v.items())
        for i, (k, item) in enumerate(items):
            out.append(pad + "  " + json.dumps(k) + ": ")
            _write(item, indent + 1, out)
            out.append(",\n" if i + 1 < len(items) else "\n")
        out.append(pad + "}")
    else:
        raise TypeError(f"no JSON form for {type(v).__name__}")


def to_native_json(nodes, tree_ptr, base, n_features, objective="reg:squarederror",
                   num_class=0, best_iteration=None, scale_pos_weight=1.0, max_delta_step=0.0,
                   tree_weights=None):
    """The native JSON text of a gbtree model: `nodes` (NODE_DTYPE) back to
    back, tree t at nodes[tree_ptr[t] : tree_ptr[t + 1]], feeding output
    t % n_outputs; `base` one margin per output."""
    nodes = np.asarray(nodes, NODE_DTYPE)
    tree_ptr = np.asarray(tree_ptr, np.uint64)
    base = np.atleast_1d(np.asarray(base, np.float32))
    n_outputs = int(base.size)
    n_trees = len(tree_ptr) - 1
    if objective.startswith("multi:") and num_class != n_outputs:
        raise ValueError("a multiclass model has one output per class")
    trees = []
    for t in range(n_trees):
        seg = nodes[int(tree_ptr[t]):int(tree_ptr[t + 1])]
        trees.append({
            "nodes": [{
                "split_feature": int(nd["split_feature"]) if nd["left"] >= 0 else 0,
                "split_cond": _F32(nd["split_cond"]),
                "default_left": bool(nd["default_left"]),
                "left": int(nd["left"]),
                "right": int(nd["right"]),
                "leaf_value": _F32(nd["leaf_value"]),
                "sum_hess": _F32(nd["sum_hess"]),
                "split_gain": _F32(nd["split_gain"]),
                "is_categorical": False,
                "cat_begin": 0,
                "cat_end": 0,
            } for nd in seg],
            "categories": [],
            "size_leaf_vector": 0,
            "leaf_vectors": [],
            "linear": None,
        })
    params = {}
    for k, (kind, dv) in _DEFAULT_PARAMS:
        v = {"scale_pos_weight": scale_pos_weight, "max_delta_step": max_delta_step}.get(k, dv)
        params[k] = _F32(v) if kind == "f32" else _F64(v) if kind == "f64" else v
    weights = np.ones(n_trees, np.float32) if tree_weights is None else np.asarray(tree_weights, np.float32)
    doc = {
        "trees": trees,
        "base_score": [_F32(b) for b in base],
        "objective": objective,
        "objective_params": params,
        "num_class": int(num_class),
        "n_outputs": n_outputs,
        "n_targets": 1 if objective.startswith("multi:") else n_outputs,
        "n_features": int(n_features),
        "best_iteration": None if best_iteration is None else int(best_iteration),
        "tree_weights": [_F32(w) for w in weights],
        "num_parallel_tree": 1,
        "linear": None,
        "shrinkage": None,
        "boulevard": None,
        "ebm": None,
    }
    out = []
    _write(doc, 0, out)
    return "".join(out)


def from_native_json(text):
    """(nodes, tree_ptr, base, n_features, fields) of a native JSON gbtree
    model with numeric scalar-leaf trees; `fields` holds objective,
    num_class, n_outputs, best_iteration, tree_weights and
    num_parallel_tree."""
    doc = json.loads(text)
    if doc.get("linear") is not None:
        raise ValueError("gblinear models have no trees to load")
    counts = [len(t["nodes"]) for t in doc["trees"]]
    nodes = np.zeros(sum(counts), NODE_DTYPE)
    at = 0
    for t in doc["trees"]:
        if t.get("size_leaf_vector", 0) or t.get("linear") or t.get("categories"):
            raise ValueError("only numeric scalar-leaf trees load here")
        for nd in t["nodes"]:
            if nd.get("is_categorical"):
                raise ValueError("categorical splits do not load here")
            rec = nodes[at]
            rec["left"], rec["right"] = nd["left"], nd["right"]
            rec["split_feature"] = nd["split_feature"]
            rec["split_cond"] = np.float32(nd["split_cond"])
            rec["default_left"] = 1 if nd["default_left"] else 0
            rec["leaf_value"] = np.float32(nd["leaf_value"])
            rec["sum_hess"] = np.float32(nd["sum_hess"])
            rec["split_gain"] = np.float32(nd["split_gain"])
            rec["split_bin"] = -1
            at += 1
    tree_ptr = np.concatenate([[0], np.cumsum(counts)]).astype(np.uint64)
    base = np.asarray(doc["base_score"], np.float32)
    fields = {k: doc.get(k) for k in ("objective", "num_class", "n_outputs", "best_iteration",
                                       "tree_weights", "num_parallel_tree")}
    return nodes, tree_ptr, base, int(doc["n_features"]), fields
