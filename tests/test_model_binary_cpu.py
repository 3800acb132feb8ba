"""Native binary model files (src/model/native.rs, container.rs, sections.rs).

* the checksum: XXH64 against the reference's own digests
  (container.rs:283 `xxh64_matches_the_reference`);
* byte for byte: the reference's saved `.bin` files (hessboost 0.4.9) read
  here and written back are the same bytes, container and zstd frame; the
  oracle's early_stopping forest (the training known answer) writes the
  reference's file;
* the reader's refusals (container.rs:150 `read`, sections.rs:103 `parse`,
  native.rs:633 `read_trees`) and its frame-expansion policy
  (container.rs:302 `frame_expansion_policy_boundaries`);
* `Model.save_native` / `load_native` in both formats.
"""

import os

import numpy as np
import pytest

import hessboost_b200 as H
import oracle_lib as O
from hessboost_b200 import model_io as M

NATIVE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "native")
REF_WRITER = "hessboost 0.4.9"
BIN_FIXTURES = ("early_stopping", "multi_target", "multiclass_forest")

needs_zstd = pytest.mark.skipif(M._zstd() is None, reason="pyarrow's zstd codec is absent")


def _bin(name):
    with open(os.path.join(NATIVE, name + ".bin"), "rb") as fh:
        return fh.read()


def _write_back(data, **extra):
    nodes, ptr, base, nf, f = M.from_native_binary(data)
    kw = dict(objective=f["objective"], num_class=f["num_class"], best_iteration=f["best_iteration"],
              tree_weights=f["tree_weights"], num_parallel_tree=f["num_parallel_tree"],
              scale_pos_weight=f["scale_pos_weight"], max_delta_step=f["max_delta_step"],
              writer=REF_WRITER)
    kw.update(extra)
    return M.to_native_binary(nodes, ptr, base, nf, **kw)


def test_xxh64_matches_the_reference_digests():
    data = bytes(range(100))
    for chunk, want in [(b"", 0xEF46DB3751D8E999), (b"a", 0xD24EC4F1A98C6E5B), (b"abc", 0x44BC2CF5AD770999),
                        (b"0123456789abcdef", 0x5C5B90C34E376D0B), (data[:31], 0xC346D2B59B4D8EE1),
                        (data[:32], 0xCBF59C5116FF32B4), (data, 0x6AC1E58032166597)]:
        assert M.xxh64(chunk) == want, len(chunk)


@needs_zstd
@pytest.mark.parametrize("name", BIN_FIXTURES)
def test_reference_file_writes_back_byte_for_byte(name):
    data = _bin(name)
    container = M._unpack(data)
    assert container[:5] == b"HBM\0\x03"
    assert _write_back(data, compress=False) == container
    # the same container sealed at the reference's zstd level is its frame
    assert _write_back(data) == data


@needs_zstd
def test_oracle_training_known_answer_writes_the_reference_binary_file():
    g = O.golden()
    for fixed in (False, True):
        nodes, ptr, base, _ = O.train(g["x"], g["y1"], 4, max_depth=3, fixed_point=fixed)
        out = M.to_native_binary(nodes.view(H.NODE_DTYPE), ptr, base, 4, objective="reg:squarederror",
                                 best_iteration=1, writer=REF_WRITER)
        assert out == _bin("early_stopping")


@needs_zstd
@pytest.mark.parametrize("name", ["early_stopping", "multiclass_forest"])
def test_binary_and_json_readers_agree(name):
    a = M.from_native_binary(_bin(name))
    with open(os.path.join(NATIVE, name + ".json")) as fh:
        b = M.from_native_json(fh.read())
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])
    np.testing.assert_array_equal(a[2].view(np.uint32), b[2].view(np.uint32))
    assert a[3] == b[3]
    for k in ("objective", "num_class", "n_outputs", "best_iteration", "tree_weights", "num_parallel_tree"):
        assert a[4][k] == b[4][k], k


@needs_zstd
def test_loaded_binary_model_predicts_its_margins():
    g = O.golden()
    nodes, ptr, base, nf, f = M.from_native_binary(_bin("early_stopping"))
    ref = next(m for m in g["models"] if m["name"] == "early_stopping")
    n = f["best_iteration"] + 1
    got = O.predict(nodes[: int(ptr[n])].view(O.NODE_DTYPE), ptr[: n + 1], 1, base, g["x"])[:, 0]
    np.testing.assert_array_equal(got.view(np.uint32), np.array(ref["margins_bits"], np.uint32))


def test_uncompressed_container_loads_and_default_writer():
    g = O.golden()
    nodes, ptr, base, _ = O.train(g["x"], g["y1"], 2, max_depth=3)
    data = M.to_native_binary(nodes.view(H.NODE_DTYPE), ptr, base, 4, compress=False)
    assert data.startswith(b"HBM\0\x03")
    back = M.from_native_binary(data)
    assert back[4]["writer"] == M.WRITER
    np.testing.assert_array_equal(back[0][["left", "right", "split_feature"]],
                                  nodes.view(H.NODE_DTYPE)[["left", "right", "split_feature"]])


# ---------------------------------------------------------------- refusals
def _container(sections, version=3, magic=b"HBM\0", tail=b""):
    """A container of `sections` [(name, flags, payload)], checksummed."""
    w = M._SectionWriter()
    for name, flags, payload in sections:
        w.raw(name, payload, flags)
    body = w.container()[:-8]
    body = magic + bytes([version]) + body[5:] + tail
    return body + M.xxh64(body).to_bytes(8, "little")


def _sections_of(container):
    """The [(name, flags, payload)] table of an uncompressed container."""
    at = 5
    count = int.from_bytes(container[at:at + 4], "little")
    at += 4
    table = []
    for _ in range(count):
        n = container[at]
        name = container[at + 1:at + 1 + n].decode()
        flags = container[at + 1 + n]
        size = int.from_bytes(container[at + 2 + n:at + 10 + n], "little")
        table.append((name, flags, size))
        at += 10 + n
    out = []
    for name, flags, size in table:
        out.append((name, flags, container[at:at + size]))
        at += size
    return out


@pytest.fixture(scope="module")
def plain():
    g = O.golden()
    nodes, ptr, base, _ = O.train(g["x"], g["y1"], 2, max_depth=3)
    return M.to_native_binary(nodes.view(H.NODE_DTYPE), ptr, base, 4, compress=False)


def test_rebuilt_container_is_identical(plain):
    assert _container(_sections_of(plain)) == plain


@pytest.mark.parametrize("case,message", [
    ("checksum", "checksum mismatch"),
    ("version", "unsupported native model version 2"),
    ("legacy", "0.1.x"),
    ("magic", "invalid native model header"),
    ("trailing", "unexpected bytes after the last section"),
    ("truncated", "truncated"),
    ("required_unknown", "cannot read"),
    ("duplicate", "appears twice"),
    ("flags", "undefined bits"),
    ("length", "wrong length"),
    ("missing", "missing section `node.left`"),
    ("gblinear", "only numeric scalar-leaf gbtree models load here"),
    ("categorical", "categorical splits do not load here"),
    ("has_linear", "other than 0, 1 or 2"),
    ("divisor", "outside 1 to 2^53"),
])
def test_reader_refusals(plain, case, message):
    secs = _sections_of(plain)
    idx = {name: i for i, (name, _, _) in enumerate(secs)}

    def put(name, payload, flags=1):
        if name in idx:
            secs[idx[name]] = (name, secs[idx[name]][1], payload)
        else:
            secs.append((name, flags, payload))

    n_nodes = len(dict((n, p) for n, _, p in secs)["node.flags"])
    n_trees = len(dict((n, p) for n, _, p in secs)["tree.has_linear"])
    data = None
    if case == "checksum":
        data = bytearray(plain)
        data[20] ^= 1
        data = bytes(data)
    elif case == "version":
        data = _container(secs, version=2)
    elif case == "legacy":
        data = _container(secs, magic=b"SQB\0")
    elif case == "magic":
        data = _container(secs, magic=b"XYZ\0")
    elif case == "trailing":
        data = _container(secs, tail=b"\0")
    elif case == "truncated":
        data = _container(secs)[:40]
        data = data + M.xxh64(data).to_bytes(8, "little")
    elif case == "required_unknown":
        put("model.future_field", b"\1", flags=1)
    elif case == "duplicate":
        secs.append(secs[idx["model.n_features"]])
    elif case == "flags":
        put("node.flags", bytes([4] + [0] * (n_nodes - 1)))
    elif case == "length":
        put("node.split_cond", secs[idx["node.split_cond"]][2][:-4])
    elif case == "missing":
        del secs[idx["node.left"]]
    elif case == "gblinear":
        put("gblinear.weights", np.zeros(4, np.float32).tobytes())
    elif case == "categorical":
        put("node.flags", bytes([2] + [0] * (n_nodes - 1)))
    elif case == "has_linear":
        put("tree.has_linear", bytes([3] + [0] * (n_trees - 1)))
    elif case == "divisor":
        put("tree.leaf_divisor", np.zeros(n_trees, np.uint64).tobytes(), flags=0)
    if data is None:
        data = _container(secs)
    with pytest.raises(ValueError, match=message.replace("^", r"\^")):
        M.from_native_binary(data)


def test_unknown_optional_section_is_skipped(plain):
    secs = _sections_of(plain)
    secs.insert(3, ("model.some_later_note", 0, b"anything"))
    back = M.from_native_binary(_container(secs))
    ref = M.from_native_binary(plain)
    np.testing.assert_array_equal(back[0], ref[0])


def test_frame_expansion_policy_boundaries():
    always = M._ALWAYS_ALLOWED
    assert M._expansion_accepted(1, always)
    assert not M._expansion_accepted(1, always + 1)
    frame = always // M._MAX_EXPANSION + 1
    assert M._expansion_accepted(frame, frame * M._MAX_EXPANSION)
    assert not M._expansion_accepted(frame, frame * M._MAX_EXPANSION + 1)


@needs_zstd
def test_frame_that_declares_too_much_is_refused():
    data = _bin("early_stopping")
    assert data[4] == 0x60  # single segment, a 2-byte content size (+256)
    # the same frame with a 4-byte content size one past what its length allows
    hdr = bytes([0x28, 0xB5, 0x2F, 0xFD, 0xA0]) + (M._ALWAYS_ALLOWED + 1).to_bytes(4, "little")
    with pytest.raises(ValueError, match="expands too far"):
        M.from_native_binary(hdr + data[7:])


def test_detect():
    assert M.detect(b"\x28\xb5\x2f\xfd....") == "binary"
    assert M.detect(b"HBM\0\x03") == "binary"
    assert M.detect(b' \n{\n  "trees": []}') == "json"
    assert M.detect(b"{}") == "json"
    assert M.detect(b'{"learner": {}}') is None  # XGBoost JSON
    assert M.detect(b"{i\x05trees") is None       # UBJSON
    assert M.detect(b"tree\nversion=v4") is None  # LightGBM text
    assert M.detect(b"") is None


@pytest.mark.parametrize("fmt", ["json", "binary"])
def test_model_save_load_both_formats(tmp_path, fmt):
    g = O.golden()
    nodes, ptr, base, margins = O.train(g["x"], g["y1"], 3, max_depth=3)
    m = H.Model(nodes.view(H.NODE_DTYPE).copy(), ptr, float(base[0]), 4)
    path = tmp_path / ("model." + fmt)
    m.save_native(path, H.TrainingParams(), format=fmt)
    back = H.Model.load_native(path)
    assert M.detect(open(path, "rb").read()) == fmt
    np.testing.assert_array_equal(back.tree_ptr, m.tree_ptr)
    for k in ("left", "right", "split_feature", "default_left"):
        np.testing.assert_array_equal(back.nodes[k], m.nodes[k])
    for k in ("split_cond", "leaf_value", "sum_hess", "split_gain"):
        np.testing.assert_array_equal(back.nodes[k].view(np.uint32), m.nodes[k].view(np.uint32))
    got = O.predict(back.nodes.view(O.NODE_DTYPE), back.tree_ptr, 1, back.bases(), g["x"])
    np.testing.assert_array_equal(got.view(np.uint32), margins.view(np.uint32))
    with pytest.raises(ValueError):
        m.save_native(tmp_path / "x", H.TrainingParams(), format="ubjson")


def _saved_models():
    return [(m["version"], m["name"]) for m in O.golden()["models"]]


@needs_zstd
@pytest.mark.parametrize("version,name", _saved_models(), ids=[f"{v}-{n}" for v, n in _saved_models()])
def test_every_saved_model_reads_predicts_and_writes_back(version, name):
    # every prediction known answer, through its binary file: the trees
    # equal the JSON file's, the margins are the recorded ones bit for bit,
    # and the file writes back to the same container
    g = O.golden()
    m = next(x for x in g["models"] if (x["version"], x["name"]) == (version, name))
    data = _bin(f"saved_{version}_{name}")
    nodes, ptr, base, nf, f = M.from_native_binary(data)
    gnodes, gptr = O.golden_nodes(m)
    np.testing.assert_array_equal(ptr, gptr)
    for k in ("left", "right", "default_left"):
        np.testing.assert_array_equal(nodes[k], gnodes[k], err_msg=k)
    inner = nodes["left"] >= 0
    np.testing.assert_array_equal(nodes["split_feature"][inner], gnodes["split_feature"][inner])
    for k in ("split_cond", "leaf_value"):
        np.testing.assert_array_equal(nodes[k].view(np.uint32), gnodes[k].view(np.uint32), err_msg=k)
    np.testing.assert_array_equal(base.view(np.uint32), O.f32_to_bits(np.array(m["base_score"], np.float32)))
    n, outs, w = O.golden_layout(m)
    got = O.predict(nodes.view(O.NODE_DTYPE), ptr[: n + 1], m["n_outputs"], base, g["x"], outs, w)
    np.testing.assert_array_equal(O.f32_to_bits(got).ravel(), np.array(m["margins_bits"], np.uint32))
    out = M.to_native_binary(nodes, ptr, base, nf, objective=f["objective"], num_class=f["num_class"],
                             best_iteration=f["best_iteration"], tree_weights=f["tree_weights"],
                             num_parallel_tree=f["num_parallel_tree"], n_targets=f["n_targets"],
                             objective_sections=f["objective_sections"], writer=f["writer"], compress=False)
    assert out == M._unpack(data)
    assert f["writer"] == f"hessboost {version}"


def test_objective_sections_must_be_objective_sections():
    g = O.golden()
    nodes, ptr, base, _ = O.train(g["x"], g["y1"], 1, max_depth=2)
    with pytest.raises(ValueError, match="not an objective section"):
        M.to_native_binary(nodes.view(H.NODE_DTYPE), ptr, base, 4, objective_sections=[("model.n_features", b"")])


@needs_zstd
@pytest.mark.parametrize("version,name,ext", [("0.4.9", "multiclass_forest", ".bin"), ("0.4.9", "multiclass_forest", ".json"),
                                              ("0.2.0", "dart", ".bin"), ("0.4.3", "dart", ".bin"),
                                              ("0.4.9", "early_stopping", ".bin")])
def test_model_load_native_keeps_the_tree_layout(tmp_path, version, name, ext):
    # Model.load_native keeps num_parallel_tree (the softprob forest grows 3
    # trees per class and round) and DART's per-tree weights, stops at the
    # best iteration, and its layout predicts the recorded margins
    g = O.golden()
    src = name + ext if version == "0.4.9" else f"saved_{version}_{name}{ext}"
    m = H.Model.load_native(os.path.join(NATIVE, src))
    ref = next(x for x in g["models"] if x["name"] == name and (x["version"] == version or version == "0.4.9"))
    n, outs, w = O.golden_layout(ref)
    got_outs, got_w = m.tree_layout()
    assert len(m.tree_ptr) - 1 == n
    np.testing.assert_array_equal(got_outs, outs)
    np.testing.assert_array_equal(np.ones(n, np.float32) if got_w is None else got_w, w)
    pred = O.predict(m.nodes.view(O.NODE_DTYPE), m.tree_ptr, m.bases().size, m.bases(), g["x"], got_outs, got_w)
    np.testing.assert_array_equal(O.f32_to_bits(pred).ravel(), np.array(ref["margins_bits"], np.uint32))
    # and saves with that layout
    path = tmp_path / "again.bin"
    m.save_native(path, H.TrainingParams(objective="multi:softmax", num_class=3) if name == "multiclass_forest"
                  else H.TrainingParams(), format="binary")
    back = H.Model.load_native(path)
    assert back.num_parallel_tree == m.num_parallel_tree
    np.testing.assert_array_equal(back.tree_layout()[0], got_outs)


def test_c5_forest_round_trips_at_full_size():
    # the prediction workload's forest (1,000 complete depth-8 trees,
    # 511,000 nodes): the binary file gives back every node bit for bit
    from hessboost_b200 import synth

    nodes, ptr = synth.forest_c5()
    base = np.array([0.25], np.float32)
    data = M.to_native_binary(nodes, ptr, base, 50)
    back = M.from_native_binary(data)
    assert len(back[0]) == len(nodes) == 1000 * 511
    np.testing.assert_array_equal(back[1], ptr)
    for k in ("left", "right", "default_left"):
        np.testing.assert_array_equal(back[0][k], nodes[k])
    inner = nodes["left"] >= 0
    np.testing.assert_array_equal(back[0]["split_feature"][inner], nodes["split_feature"][inner])
    for k in ("split_cond", "leaf_value", "sum_hess", "split_gain"):
        np.testing.assert_array_equal(back[0][k].view(np.uint32), nodes[k].view(np.uint32))
