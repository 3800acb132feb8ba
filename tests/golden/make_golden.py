"""Regenerate ``saved_models.json`` from the reference checkout's saved models.

The reference (hessboost 0.4.9) keeps, under ``tests/data/saved/<version>/``,
models trained by its own ``tests/native_format.rs`` on a fixed 160 x 4 probe
(``tests/common/mod.rs:29-39`` ``four_features``) together with the raw
margins each model predicted on that probe when it was saved (f32
little-endian, ``<name>.margins``).  This script extracts, for every model
whose trees are scalar-leaf numeric trees (the only kind the CUDA prediction
path serves), the node arrays, base scores, tree weights, output layout and
recorded margins, and adds the probe rows and labels computed as the
reference's tests compute them (f32 arithmetic throughout).

* ``early_stopping`` and ``multi_target`` (0.4.9) are full *training*
  known-answer tests: ``train(hist, max_depth 3, seed 11, defaults)`` for 4
  rounds on the probe (``tests/native_format.rs:441-489``), labels
  ``y_t = 2a - b + t*c + 0.1``.
* every extracted model (all versions) is a *prediction* known-answer test.
* ``native/early_stopping.json`` and ``native/multiclass_forest.json`` are
  two of those files verbatim, the native JSON writer's byte-level fixtures;
  ``native/{early_stopping,multi_target,multiclass_forest}.bin`` likewise for
  the native binary format, and ``native/saved_<version>_<name>.bin`` is the
  binary file of every extracted prediction model.

Usage: ``python tests/golden/make_golden.py /path/to/reference`` (the root of
a hessboost 0.4.9 checkout).  The output is committed, so the tests never
need the reference at run time.
"""

import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
MODELS = [
    "early_stopping",
    "multi_target",
    "dart",
    "quantiles",
    "expectiles",
    "aft",
    "dist_normal",
    "dist_negbinomial",
    "multiclass_forest",
]
NODE_FIELDS = [
    "split_feature",
    "split_cond",
    "default_left",
    "left",
    "right",
    "leaf_value",
    "sum_hess",
    "split_gain",
]


def probe(n=160):
    """``four_features`` rows (tests/common/mod.rs:31) in f32 arithmetic."""
    i = np.arange(n)
    a = ((i * 37) % 101).astype(np.float32) / np.float32(101.0)
    b = ((i * 53) % 97).astype(np.float32) / np.float32(97.0)
    c = ((i * 11) % 89).astype(np.float32) / np.float32(89.0)
    d = ((i * 29) % 83).astype(np.float32) / np.float32(83.0)
    d[i % 7 == 0] = np.float32("nan")
    return np.stack([a, b, c, d], axis=1).astype(np.float32)


def labels(x, k):
    """``train_data`` labels (tests/native_format.rs:441): 2a - b + t*c + 0.1."""
    a, b, c = x[:, 0], x[:, 1], x[:, 2]
    cols = []
    for t in range(k):
        y = np.float32(2.0) * a - b + np.float32(t) * c + np.float32(0.1)
        cols.append(y.astype(np.float32))
    return np.stack(cols, axis=1).astype(np.float32)


def f32_bits(values):
    return [struct.unpack("<I", struct.pack("<f", float(v)))[0] for v in values]


def main(ref):
    saved = os.path.join(ref, "tests", "data", "saved")
    x = probe()
    out = {
        "source": "hessboost 0.4.9 tests/data/saved (extracted by make_golden.py)",
        "probe_x_bits": f32_bits(x.ravel()),
        "labels_k1_bits": f32_bits(labels(x, 1).ravel()),
        "labels_k2_bits": f32_bits(labels(x, 2).ravel()),
        "models": [],
    }
    seen = set()
    for version in sorted(os.listdir(saved)):
        for name in MODELS:
            path = os.path.join(saved, version, name + ".json")
            if not os.path.exists(path):
                continue
            with open(path) as fh:
                doc = json.load(fh)
            with open(os.path.join(saved, version, name + ".margins"), "rb") as fh:
                raw = fh.read()
            margins = list(struct.unpack("<%dI" % (len(raw) // 4), raw))
            trees = [
                {f: [node[f] for node in t["nodes"]] for f in NODE_FIELDS} for t in doc["trees"]
            ]
            for t in doc["trees"]:
                assert t["size_leaf_vector"] == 0 and not t.get("linear")
                assert not any(n["is_categorical"] for n in t["nodes"])
            key = json.dumps([trees, doc["base_score"], margins], sort_keys=True)
            if key in seen:
                continue
            seen.add(key)
            # the same model's native binary file, for the binary reader
            os.makedirs(os.path.join(HERE, "native"), exist_ok=True)
            with open(os.path.join(saved, version, name + ".bin"), "rb") as fh:
                raw_bin = fh.read()
            with open(os.path.join(HERE, "native", f"saved_{version}_{name}.bin"), "wb") as fh:
                fh.write(raw_bin)
            out["models"].append(
                {
                    "name": name,
                    "version": version,
                    "objective": doc["objective"],
                    "n_outputs": doc["n_outputs"],
                    "num_parallel_tree": doc["num_parallel_tree"],
                    "best_iteration": doc["best_iteration"],
                    "tree_weights": doc["tree_weights"],
                    "base_score": doc["base_score"],
                    "trees": trees,
                    "margins_bits": margins,
                }
            )
    dst = os.path.join(HERE, "saved_models.json")
    with open(dst, "w") as fh:
        json.dump(out, fh, separators=(",", ":"))
    print("wrote", dst, "with", len(out["models"]), "models")
    # two native JSON files verbatim: the model writer's byte-level fixtures
    os.makedirs(os.path.join(HERE, "native"), exist_ok=True)
    # and three native binary files (zstd frames of the section container)
    # verbatim: the binary writer's and reader's fixtures
    for name, ext in (("early_stopping", ".json"), ("multiclass_forest", ".json"),
                      ("early_stopping", ".bin"), ("multi_target", ".bin"),
                      ("multiclass_forest", ".bin")):
        src = os.path.join(saved, "0.4.9", name + ext)
        with open(src, "rb") as fh:
            raw = fh.read()
        with open(os.path.join(HERE, "native", name + ext), "wb") as fh:
            fh.write(raw)
        print("copied", src)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/hessboost-checkout")
    main(sys.argv[1])
