"""Native JSON model files (the reference's BoostedModel serde form).

* byte for byte: the oracle's early_stopping forest (which reproduces the
  reference's training known answer bit for bit), written with the
  reference's early-stopping iteration, is the reference's saved file;
* a reference file loads and writes back to the same JSON values;
* on the GPU: a device-trained model survives a save and load with its
  predictions bit for bit.
"""

import json
import os

import numpy as np
import pytest

import hessboost_b200 as H
import oracle_lib as O
from hessboost_b200 import model_io, synth

NATIVE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "native")


def _read(name):
    with open(os.path.join(NATIVE, name + ".json")) as fh:
        return fh.read()


def test_shortest_float_layout():
    cases = [(0.5247525, "0.5247525"), (160.0, "160.0"), (1e-7, "1e-7"), (1.5e-7, "1.5e-7"),
             (3e-5, "0.00003"), (0.0, "0.0"), (-0.11136258, "-0.11136258"), (1e13, "1e13"),
             (123456.0, "123456.0"), (2.5e20, "2.5e20")]
    for v, want in cases:
        assert model_io._shortest(v, True) == want, v
    assert model_io._shortest(1e15, False) == "1000000000000000.0"
    assert model_io._shortest(1e17, False) == "1e17"


def test_oracle_early_stopping_forest_writes_the_reference_file():
    g = O.golden()
    nodes, ptr, base, _ = O.train(g["x"], g["y1"], 4, max_depth=3)
    text = model_io.to_native_json(nodes.view(H.NODE_DTYPE), ptr, base, 4,
                                   objective="reg:squarederror", best_iteration=1)
    assert text == _read("early_stopping")


def test_reference_file_round_trips():
    for name in ("early_stopping", "multiclass_forest"):
        text = _read(name)
        nodes, ptr, base, nf, fields = model_io.from_native_json(text)
        again = model_io.to_native_json(nodes, ptr, base, nf, objective=fields["objective"],
                                        num_class=fields["num_class"],
                                        best_iteration=fields["best_iteration"],
                                        tree_weights=fields["tree_weights"],
                                        num_parallel_tree=fields["num_parallel_tree"])
        a, b = json.loads(text), json.loads(again)
        assert a == b, name


def test_loaded_reference_model_predicts_its_margins():
    g = O.golden()
    nodes, ptr, base, nf, fields = model_io.from_native_json(_read("early_stopping"))
    ref = next(m for m in g["models"] if m["name"] == "early_stopping")
    n = fields["best_iteration"] + 1
    want = np.array(ref["margins_bits"], np.uint32).view(np.float32)
    got = O.predict(nodes[: int(ptr[n])].view(O.NODE_DTYPE), ptr[: n + 1], 1, base, g["x"])[:, 0]
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.gpu
def test_device_model_save_load_predicts_the_same(tmp_path):
    x, y = synth.logistic_c2(5000, 10, seed=21)
    p = H.TrainingParams(objective="binary:logistic", max_depth=4, eta=0.3)
    m = H.train(p, x, y, 3)
    path = tmp_path / "model.json"
    m.save_native(path, p)
    back = H.Model.load_native(path)
    np.testing.assert_array_equal(back.predict_margin(x).view(np.uint32), m.predict_margin(x).view(np.uint32))
    doc = json.loads(path.read_text())
    assert doc["objective"] == "binary:logistic" and doc["n_features"] == 10 and len(doc["trees"]) == 3
