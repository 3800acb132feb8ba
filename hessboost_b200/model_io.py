"""Native model files, in both of the reference's native formats.

* JSON: the `BoostedModel` serde form (src/model/serde.rs:12
  `SerializedBoostedModel`, fields in that order), written pretty the way
  its JSON writer writes them (src/model/io.rs:101: two-space indent, one
  element per line, f32 and f64 values in their shortest round-trip decimal
  form).
* Binary: the checksummed section container (src/model/native.rs,
  container.rs, sections.rs) as one zstd frame.

A model trained here and saved with `Model.save_native` loads unchanged in
the reference's Python and Rust APIs; a reference model file of either
format loads here with `Model.load_native`.

Only what this library trains is written: numeric scalar-leaf trees of
reg:squarederror, binary:logistic and multi:softmax (no categories, vector
leaves, linear leaves, DART weights or boosters besides gbtree).
"""

import ctypes
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
                   tree_weights=None, num_parallel_tree=1):
    """The native JSON text of a gbtree model: `nodes` (NODE_DTYPE) back to
    back, tree t at nodes[tree_ptr[t] : tree_ptr[t + 1]], feeding output
    (t // num_parallel_tree) % n_outputs; `base` one margin per output."""
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
        "num_parallel_tree": int(num_parallel_tree),
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


# ---------------------------------------------------------------- binary form
# The native binary container (src/model/native.rs:1-60,
# src/model/container.rs:1-13, src/model/sections.rs:1-17):
#
#   b"HBM\0", u8 container version 3,
#   u32 section count, per section: u8 name length, name, u8 flags,
#   u64 payload length; the payloads back to back in table order;
#   u64 XXH64 (seed 0) of every byte before it,
#
# little-endian throughout, stored as one zstd frame (or uncompressed, which
# the reader accepts as well). Sections are written in the order the
# reference's writer emits them (native.rs:413 `write_model_sections`, :463
# `write_tree_sections`), so a model written here with the reference's
# writer string is the reference's file byte for byte.

WRITER = "hessboost_b200 0.1"
_MAGIC = b"HBM\0"
_LEGACY_MAGIC = b"SQB\0"
_CONTAINER_VERSION = 3
_ZSTD_MAGIC = b"\x28\xb5\x2f\xfd"
_REQUIRED = 1
_DEFAULT_LEFT, _CATEGORICAL = 1, 2
# decompressed containers up to 256 MiB always load, larger ones within
# 4096x of their frame (container.rs:38-44)
_ALWAYS_ALLOWED = 256 << 20
_MAX_EXPANSION = 1 << 12
# the zstd level the reference seals with (the zstd crate's default)
_ZSTD_LEVEL = 3

# every section the reference's reader knows (native.rs:121 `KNOWN`, plus the
# objective sections :767); the ones marked False make a model this library
# does not load (gblinear, shrinkage, EBM terms change predictions)
_KNOWN = {
    "model.objective", "model.writer", "model.base_score", "model.num_class", "model.n_outputs",
    "model.n_targets", "model.n_features", "model.best_iteration", "model.tree_weights",
    "model.num_parallel_tree", "shrinkage.factors", "shrinkage.base_score", "gblinear.weights",
    "gblinear.bias", "tree.node_count", "node.split_feature", "node.split_cond", "node.left",
    "node.right", "node.leaf_value", "node.sum_hess", "node.split_gain", "node.cat_begin",
    "node.cat_end", "node.flags", "tree.category_count", "tree.categories", "tree.size_leaf_vector",
    "tree.leaf_vectors", "tree.has_linear", "tree.leaf_divisor", "leaf_linear.offsets",
    "leaf_linear.intercepts", "leaf_linear.features", "leaf_linear.coeffs", "leaf_linear.lower",
    "leaf_linear.upper", "boulevard.dropout", "boulevard.learning_rate", "boulevard.subsample",
    "boulevard.reg_lambda", "boulevard.truncation", "boulevard.seed",
    "boulevard.intercept_from_labels", "ebm.term_sizes", "ebm.term_features", "ebm.tree_terms",
    "ebm.term_means", "ebm.boulevard",
    "objective.scale_pos_weight", "objective.max_delta_step", "objective.tweedie_variance_power",
    "objective.huber_slope", "objective.lambdarank_num_pair_per_sample", "objective.quantile_alpha",
    "objective.expectile_alpha", "objective.exceedance_threshold", "objective.aft_loss_distribution",
    "objective.aft_loss_distribution_scale", "objective.dist_gradient",
    "objective.dist_split_direction", "objective.distribution",
}
_UNSUPPORTED = ("gblinear.weights", "gblinear.bias", "shrinkage.factors", "shrinkage.base_score",
                "leaf_linear.lower", "leaf_linear.upper", "ebm.term_sizes")


def xxh64(data):
    """XXH64 (seed 0) of `data`, the container's checksum (hb_xxh64)."""
    from . import lib

    buf = bytes(data)
    out = ctypes.c_uint64()
    st = lib().hb_xxh64(buf, len(buf), ctypes.byref(out))
    if st != 0:
        raise RuntimeError(f"hb_xxh64 failed with status {st}")
    return out.value


class _SectionWriter:
    """A section table (sections.rs:28 `Writer`)."""

    def __init__(self):
        self.sections = []

    def raw(self, name, payload, flags=_REQUIRED):
        enc = name.encode()
        if len(enc) > 255:
            raise ValueError(f"section name {name!r} is too long")
        self.sections.append((enc, flags, bytes(payload)))

    def str(self, name, value):
        self.raw(name, value.encode())

    def u64(self, name, value):
        self.raw(name, int(value).to_bytes(8, "little"))

    def f64(self, name, value):
        self.raw(name, np.float64(value).tobytes())

    def array(self, name, values, dtype):
        self.raw(name, np.ascontiguousarray(values, np.dtype(dtype).newbyteorder("<")).tobytes())

    def container(self):
        """magic, version, table, payloads, checksum (container.rs:66)."""
        parts = [_MAGIC, bytes([_CONTAINER_VERSION]), len(self.sections).to_bytes(4, "little")]
        for name, flags, payload in self.sections:
            parts += [bytes([len(name)]), name, bytes([flags]), len(payload).to_bytes(8, "little")]
        parts += [payload for _, _, payload in self.sections]
        body = b"".join(parts)
        return body + xxh64(body).to_bytes(8, "little")


def _zstd():
    """pyarrow's zstd codec, or None where pyarrow is absent."""
    try:
        import pyarrow as pa
    except ImportError:
        return None
    return pa if pa.Codec.is_available("zstd") else None


def _expansion_accepted(compressed, decompressed):
    return decompressed <= max(compressed * _MAX_EXPANSION, _ALWAYS_ALLOWED)


def to_native_binary(nodes, tree_ptr, base, n_features, objective="reg:squarederror", num_class=0,
                     best_iteration=None, scale_pos_weight=1.0, max_delta_step=0.0, tree_weights=None,
                     num_parallel_tree=1, writer=WRITER, compress=True, n_targets=None,
                     objective_sections=None):
    """The native binary file of a gbtree model (arguments as
    `to_native_json`): the section container as one zstd frame when
    `compress` and a zstd codec is present (the reference's `seal`,
    container.rs:81, keeps it uncompressed when the frame would expand past
    what its reader accepts), else the container itself.

    `n_targets` defaults to 1 for multi:* objectives and to the output
    count otherwise; `objective_sections` ([(name, payload)], as
    `from_native_binary` returns them), when given, replaces the objective
    parameters written from `scale_pos_weight` and `max_delta_step`, so a
    model read here writes back unchanged."""
    nodes = np.asarray(nodes, NODE_DTYPE)
    tree_ptr = np.asarray(tree_ptr, np.uint64)
    base = np.atleast_1d(np.asarray(base, np.float32))
    n_outputs = int(base.size)
    n_trees = len(tree_ptr) - 1
    if objective.startswith("multi:") and num_class != n_outputs:
        raise ValueError("a multiclass model has one output per class")
    if n_trees >= 1 << 32 or len(nodes) >= 1 << 32:
        raise ValueError("model is too large for the native format")
    nodes = nodes[: int(tree_ptr[-1])] if n_trees else nodes[:0]
    weights = np.ones(n_trees, np.float32) if tree_weights is None else np.asarray(tree_weights, np.float32)
    w = _SectionWriter()
    # model.* (native.rs:413)
    w.str("model.objective", objective)
    w.raw("model.writer", writer.encode(), flags=0)
    w.array("model.base_score", base, np.float32)
    w.u64("model.num_class", num_class)
    w.u64("model.n_outputs", n_outputs)
    if n_targets is None:
        n_targets = 1 if objective.startswith("multi:") else n_outputs
    w.u64("model.n_targets", n_targets)
    w.u64("model.n_features", n_features)
    if best_iteration is not None:
        w.u64("model.best_iteration", best_iteration)
    w.array("model.tree_weights", weights, np.float32)
    w.u64("model.num_parallel_tree", num_parallel_tree)
    # objective.* (native.rs:767), the objective's stored defaults otherwise
    if objective_sections is not None:
        for name, payload in objective_sections:
            if not name.startswith("objective.") or name not in _KNOWN:
                raise ValueError(f"{name!r} is not an objective section")
            w.raw(name, payload)
    else:
        _default_objective_sections(w, scale_pos_weight, max_delta_step)
    _tree_sections(w, nodes, tree_ptr, n_trees)
    container = w.container()
    pa = _zstd() if compress else None
    if pa is None:
        return container
    frame = pa.Codec("zstd", compression_level=_ZSTD_LEVEL).compress(container, asbytes=True)
    return frame if _expansion_accepted(len(frame), len(container)) else container


def _default_objective_sections(w, scale_pos_weight, max_delta_step):
    """The objective parameters this library trains with, the others at
    the reference's stored defaults (objective.rs:166)."""
    w.f64("objective.scale_pos_weight", np.float32(scale_pos_weight))
    w.f64("objective.max_delta_step", max_delta_step)
    w.f64("objective.tweedie_variance_power", 1.5)
    w.f64("objective.huber_slope", np.float32(1.0))
    w.u64("objective.lambdarank_num_pair_per_sample", 32)
    w.array("objective.quantile_alpha", [], np.float64)
    w.array("objective.expectile_alpha", [], np.float64)
    w.str("objective.aft_loss_distribution", "normal")
    w.f64("objective.aft_loss_distribution_scale", 1.0)
    w.str("objective.dist_gradient", "fisher")
    w.str("objective.dist_split_direction", "random")


def _tree_sections(w, nodes, tree_ptr, n_trees):
    """The trees column-wise (native.rs:463 `write_tree_sections`), numeric
    scalar-leaf trees only: no categories, leaf vectors or linear leaves."""
    counts = np.diff(tree_ptr.astype(np.int64)).astype(np.uint32)
    leaf = nodes["left"] < 0
    w.array("tree.node_count", counts, np.uint32)
    w.array("node.split_feature", np.where(leaf, 0, nodes["split_feature"]), np.uint32)
    w.array("node.split_cond", nodes["split_cond"], np.float32)
    w.array("node.left", nodes["left"], np.int32)
    w.array("node.right", nodes["right"], np.int32)
    w.array("node.leaf_value", nodes["leaf_value"], np.float32)
    w.array("node.sum_hess", nodes["sum_hess"], np.float32)
    w.array("node.split_gain", nodes["split_gain"], np.float32)
    zeros = np.zeros(len(nodes), np.uint32)
    w.array("node.cat_begin", zeros, np.uint32)
    w.array("node.cat_end", zeros, np.uint32)
    w.array("node.flags", np.where(nodes["default_left"] != 0, _DEFAULT_LEFT, 0), np.uint8)
    per_tree = np.zeros(n_trees, np.uint32)
    w.array("tree.category_count", per_tree, np.uint32)
    w.array("tree.categories", [], np.uint32)
    w.array("tree.size_leaf_vector", per_tree, np.uint32)
    w.array("tree.leaf_vectors", [], np.float32)
    w.array("tree.has_linear", np.zeros(n_trees, np.uint8), np.uint8)
    w.array("leaf_linear.offsets", [], np.uint32)
    w.array("leaf_linear.intercepts", [], np.float64)
    w.array("leaf_linear.features", [], np.uint32)
    w.array("leaf_linear.coeffs", [], np.float64)


def _zstd_content_size(frame):
    """The decompressed size a zstd frame header declares (RFC 8878 3.1.1.1),
    or None when the header leaves it out."""
    if len(frame) < 6:
        raise ValueError("truncated zstd frame")
    fhd = frame[4]
    fcs_flag, single = fhd >> 6, (fhd >> 5) & 1
    if fhd & 0x08:
        raise ValueError("zstd frame header has its reserved bit set")
    at = 5 + (0 if single else 1) + (0, 1, 2, 4)[fhd & 3]
    width = (1 if single else 0, 2, 4, 8)[fcs_flag]
    if width == 0:
        return None
    if len(frame) < at + width:
        raise ValueError("truncated zstd frame")
    size = int.from_bytes(frame[at:at + width], "little")
    return size + 256 if width == 2 else size


def _unpack(data):
    """The container in `data`: decompressed from its zstd frame, within
    the reader's expansion bound (container.rs:170 `unpack`), or as is."""
    if not data.startswith(_ZSTD_MAGIC):
        return data
    size = _zstd_content_size(data)
    if size is None:
        raise ValueError("zstd frame without a content size")
    if not _expansion_accepted(len(data), size):
        raise ValueError("zstd frame expands too far")
    pa = _zstd()
    if pa is None:
        raise ValueError("a zstd-compressed model needs pyarrow's zstd codec")
    out = pa.decompress(data, decompressed_size=size, codec="zstd", asbytes=True)
    if len(out) != size:
        raise ValueError("zstd frame disagrees with its content size")
    return out


def _sections(container):
    """name -> payload of a checked container (container.rs:183
    `section_table`, sections.rs:103 `Sections::parse`)."""
    if container.startswith(_LEGACY_MAGIC):
        raise ValueError("a native model from hessboost 0.1.x, which this format cannot read")
    if not container.startswith(_MAGIC):
        raise ValueError("invalid native model header")
    if len(container) < 5:
        raise ValueError("truncated native model")
    if container[4] != _CONTAINER_VERSION:
        raise ValueError(f"unsupported native model version {container[4]}")
    if len(container) - 8 <= len(_MAGIC):
        raise ValueError("truncated native model")
    body, checksum = container[:-8], container[-8:]
    if xxh64(body).to_bytes(8, "little") != checksum:
        raise ValueError("native model checksum mismatch")
    table = memoryview(body)[5:]
    at = 0

    def take(n):
        nonlocal at
        if at + n > len(table):
            raise ValueError("truncated data")
        at += n
        return table[at - n:at]

    count = int.from_bytes(take(4), "little")
    entries = []
    for _ in range(count):
        name = bytes(take(take(1)[0]))
        try:
            name = name.decode()
        except UnicodeDecodeError:
            raise ValueError("section name is not UTF-8") from None
        flags = take(1)[0]
        entries.append((name, flags, int.from_bytes(take(8), "little")))
    out = {}
    for name, flags, n in entries:
        payload = bytes(take(n))
        if name not in _KNOWN:
            if flags & _REQUIRED:
                raise ValueError(f"the data needs section `{name}`, which this version cannot read")
            continue
        if name in out:
            raise ValueError(f"section `{name}` appears twice")
        out[name] = payload
    if at != len(table):
        raise ValueError(f"{len(table) - at} unexpected bytes after the last section")
    return out


def from_native_binary(data):
    """(nodes, tree_ptr, base, n_features, fields) of a native binary gbtree
    model with numeric scalar-leaf trees (as `from_native_json`); `data` a
    zstd frame or an uncompressed container. The checks are the reference
    reader's (native.rs:633 `read_trees`): every column's length, the
    defined flag bits, nothing left in a pool."""
    s = _sections(_unpack(bytes(data)))

    def need(name):
        if name not in s:
            raise ValueError(f"missing section `{name}`")
        return s[name]

    def u64(name):
        v = need(name)
        if len(v) != 8:
            raise ValueError(f"section `{name}` is not one value")
        return int.from_bytes(v, "little")

    def arr(name, dtype, count=None):
        v = need(name)
        dt = np.dtype(dtype).newbyteorder("<")
        if len(v) % dt.itemsize or (count is not None and len(v) != count * dt.itemsize):
            raise ValueError(f"section `{name}` has the wrong length")
        return np.frombuffer(v, dt).astype(np.dtype(dtype))

    for name in _UNSUPPORTED:
        if name in s:
            raise ValueError(f"section `{name}`: only numeric scalar-leaf gbtree models load here")
    try:
        objective = need("model.objective").decode()
    except UnicodeDecodeError:
        raise ValueError("section `model.objective` is not UTF-8") from None
    counts = arr("tree.node_count", np.uint32).astype(np.int64)
    n_trees, n_nodes = len(counts), int(counts.sum())
    nodes = np.zeros(n_nodes, NODE_DTYPE)
    nodes["split_feature"] = arr("node.split_feature", np.uint32, n_nodes)
    nodes["split_cond"] = arr("node.split_cond", np.float32, n_nodes)
    nodes["left"] = arr("node.left", np.int32, n_nodes)
    nodes["right"] = arr("node.right", np.int32, n_nodes)
    nodes["leaf_value"] = arr("node.leaf_value", np.float32, n_nodes)
    nodes["sum_hess"] = arr("node.sum_hess", np.float32, n_nodes)
    nodes["split_gain"] = arr("node.split_gain", np.float32, n_nodes)
    arr("node.cat_begin", np.uint32, n_nodes)
    arr("node.cat_end", np.uint32, n_nodes)
    flags = arr("node.flags", np.uint8, n_nodes)
    if np.any(flags & ~np.uint8(_DEFAULT_LEFT | _CATEGORICAL)):
        raise ValueError("`node.flags` holds undefined bits")
    if np.any(flags & _CATEGORICAL):
        raise ValueError("categorical splits do not load here")
    nodes["default_left"] = (flags & _DEFAULT_LEFT) != 0
    nodes["split_bin"] = -1
    if np.any(arr("tree.category_count", np.uint32, n_trees)) or len(need("tree.categories")):
        raise ValueError("categorical splits do not load here")
    if np.any(arr("tree.size_leaf_vector", np.uint32, n_trees)) or len(need("tree.leaf_vectors")):
        raise ValueError("only numeric scalar-leaf trees load here")
    has_linear = arr("tree.has_linear", np.uint8, n_trees)
    if np.any(has_linear > 2):
        raise ValueError("`tree.has_linear` holds a value other than 0, 1 or 2")
    if np.any(has_linear) or any(len(need(n)) for n in ("leaf_linear.offsets", "leaf_linear.intercepts",
                                                         "leaf_linear.features", "leaf_linear.coeffs")):
        raise ValueError("linear leaves do not load here")
    if "tree.leaf_divisor" in s:
        div = arr("tree.leaf_divisor", np.uint64, n_trees)
        if np.any((div < 1) | (div > np.uint64(1 << 53))):
            raise ValueError("`tree.leaf_divisor` holds a value outside 1 to 2^53")
    tree_ptr = np.concatenate([[0], np.cumsum(counts)]).astype(np.uint64)
    base = arr("model.base_score", np.float32)
    fields = {
        "objective": objective,
        "num_class": u64("model.num_class"),
        "n_outputs": u64("model.n_outputs"),
        "n_targets": u64("model.n_targets"),
        "best_iteration": u64("model.best_iteration") if "model.best_iteration" in s else None,
        "tree_weights": [float(v) for v in arr("model.tree_weights", np.float32)],
        "num_parallel_tree": u64("model.num_parallel_tree"),
        "writer": s["model.writer"].decode(errors="replace") if "model.writer" in s else None,
        "objective_sections": [(k, v) for k, v in s.items() if k.startswith("objective.")],
    }
    for name in ("scale_pos_weight", "max_delta_step"):
        key = "objective." + name
        if key in s:
            fields[name] = float(np.frombuffer(s[key], "<f8")[0]) if len(s[key]) == 8 else None
    return nodes, tree_ptr, base, u64("model.n_features"), fields


def detect(data):
    """"binary" or "json" for a native model file's bytes (io.rs:55
    `ModelFormat::detect`, native formats only), else None (XGBoost JSON or
    UBJSON, LightGBM text, or none of them)."""
    data = bytes(data)
    if data.startswith((_ZSTD_MAGIC, _MAGIC, _LEGACY_MAGIC)):
        return "binary"
    ws = b" \t\r\n\x0c\x0b"
    text = data.lstrip(ws)
    if text.startswith(b"{") and text[1:].lstrip(ws)[:1] in (b'"', b"}"):
        return None if b'"learner"' in data else "json"
    return None
