"""The parity checker itself (tests/parity.py), on CPU: the oracle's
fixed-point forest is bit-exact with itself, meets the north-star criteria
against the f64 mode, and the round-by-round comparison from shared margins
keeps counting after a planted structural difference."""

import numpy as np

import oracle_lib as O
import parity as P
from hessboost_b200 import synth


class OracleEngine:
    """Stands in for the GPU engine in forced_f64_rounds: the oracle's
    fixed-point trainer behind the engine's load/train/read calls."""

    def __init__(self, x, y, plant_round=None, **kw):
        self.t = O.Trainer(x, y, fixed_point=True, **kw)
        self.plant_round, self.r = plant_round, 0

    def load_margins(self, m):
        self.t.set_margins(m)

    def train_rounds(self, params, k):
        n, p = self.t.rounds(k)
        if self.r == self.plant_round:  # a different split at the root (not a tie)
            n = n.copy()
            n[0]["split_bin"] += 1
            n[0]["split_gain"] *= 2.0
        self.r += 1
        return n, p

    def read_margins(self):
        return self.t.margins()[:, 0].copy()


KW = dict(objective=1, max_depth=6, eta=0.3)


def test_fixed_point_forest_bit_exact_with_itself_and_not_with_f64():
    x, y = synth.logistic_c2(5000, 8, seed=3)
    a = O.train(x, y, 3, fixed_point=True, **KW)
    b = O.train(x, y, 3, fixed_point=True, **KW)
    assert P.forest_bit_exact(a[0], a[1], b[0], b[1]) == (True, "")
    c = O.train(x, y, 3, fixed_point=False, **KW)
    for ta, tc in zip(P.trees(a[0], a[1]), P.trees(c[0], c[1])):
        r = P.compare_tree_f64(ta, tc)
        assert r["structure_equal"] and r["leaf_ok"], r


def test_forced_rounds_meet_the_criteria():
    x, y = synth.logistic_c2(6000, 8, seed=4)
    eng = OracleEngine(x, y, **KW)
    t64 = O.Trainer(x, y, fixed_point=False, **KW)
    out = P.forced_f64_rounds(eng, None, t64, 4)
    assert out["pass"] and out["rounds"] == 4 and out["trees_structure_equal"] == 4, out


def test_forced_rounds_keep_comparing_after_a_difference():
    x, y = synth.logistic_c2(6000, 8, seed=5)
    eng = OracleEngine(x, y, plant_round=1, **KW)
    t64 = O.Trainer(x, y, fixed_point=False, **KW)
    out = P.forced_f64_rounds(eng, None, t64, 4)
    assert not out["pass"]
    assert [d["round"] for d in out["not_ties"]] == [1]
    # rounds 2 and 3 start from the oracle's margins again and match
    assert out["trees_structure_equal"] == 3 and out["rounds"] == 4
