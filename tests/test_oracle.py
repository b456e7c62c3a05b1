"""The CPU oracle, pinned before it is trusted.

* against the reference's own golden fixture (gbr.{montlok,io}, checked at
  1e-12 relative like the reference's C++ consumer test, tests/cpp/test_core.cpp:32-59);
* against the committed golden fixtures of tests/golden (the reference's
  predictions and leaf indices, bit for bit);
* against restatements of LightGBM's and XGBoost's published decision rules;
* against the reference library itself, compiled from its sources, on fresh
  random ensembles (when oracle/_ref was built here).
"""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest

import oracle
from forests import GRID, NARROWING, edge_inputs, random_model, same_bits
from montlok import export, synth

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("*.npz"))


def load_case(name):
    data = np.load(GOLDEN / f"{name}.npz")
    return data["model"].tobytes(), data["x"], data["out"], data["leaves"]


def test_reference_gbr_fixture():
    model = (GOLDEN / "gbr.montlok").read_bytes()
    io = np.fromfile(GOLDEN / "gbr.io", dtype="<f8")
    spec, _ = export.read(model)
    f, k = spec["inputs"]["features"], spec["outputs"]["size"]
    x, want = io[:3 * f].reshape(3, f), io[3 * f:].reshape(3, k)
    got = oracle.Oracle(model).predict(x)
    np.testing.assert_allclose(got, want, rtol=1e-12, atol=0)
    assert np.isnan(x).any(), "the fixture's NaN row reaches the default branch"


@pytest.mark.parametrize("name", CASES)
def test_golden_cases_bit_exact(name):
    model, x, out, leaves = load_case(name)
    o = oracle.Oracle(model)
    assert same_bits(o.predict(x), out)
    np.testing.assert_array_equal(o.leaves(x), leaves)


def test_float32_inputs_match_widened_float64():
    model, x, _, _ = load_case("edge_lt_f32")
    o = oracle.Oracle(model)
    x32 = x.astype(np.float32)
    assert same_bits(o.predict(x32), o.predict(x32.astype(np.float64)))


# --- published decision rules, restated on the file's node arrays ---------


def lightgbm_rule(spec, t, x):
    """LightGBM's numerical decision (missing types None / Zero / NaN) and
    GBDT sum, one row and tree at a time."""
    zero = float(np.float32(1e-35))
    k = spec["outputs"]["size"]
    raw = np.zeros((len(x), k))
    for tree, root in enumerate(t["trees.root"]):
        for i, row in enumerate(x):
            n = int(root)
            while t["trees.feature"][n] >= 0:
                v = float(row[t["trees.feature"][n]])
                flags = int(t["trees.flags"][n])
                mode, default_left = (flags >> 1) & 3, flags & 1
                if math.isnan(v) and mode != 1 and mode != 2:
                    v = 0.0
                if (mode == 2 and (math.isnan(v) or -zero <= v <= zero)) or (mode == 1 and math.isnan(v)):
                    go_left = bool(default_left)
                else:
                    go_left = v <= t["trees.threshold"][n]
                n = int(t["trees.left"][n] if go_left else t["trees.right"][n])
            raw[i, t["trees.output"][tree]] += t["trees.value"][n]
    return raw


@pytest.mark.parametrize("name", ["lightgbm_regression", "lightgbm_binary", "lightgbm_multiclass"])
def test_lightgbm_decision_rule(name):
    model, x, _, _ = load_case(name)
    spec, t = export.read(model)
    raw = lightgbm_rule(spec, t, x)
    link = spec["config"]["link"]
    if link == "sigmoid":
        expected = 1 / (1 + np.exp(-spec["config"]["sigmoid_scale"] * raw))
    elif link == "softmax":
        e = np.exp(raw - raw.max(axis=1, keepdims=True))
        expected = e / e.sum(axis=1, keepdims=True)
    else:
        expected = raw
    np.testing.assert_allclose(oracle.Oracle(model).predict(x), expected, rtol=1e-12, atol=1e-14)


def test_xgboost_decision_rule():
    """XGBoost: float32 features, `x < split_condition`, missing to the default child."""
    model, x, _, _ = load_case("xgboost_logistic")
    spec, t = export.read(model)
    xf = x.astype(np.float32)
    margin = np.full(len(x), spec["config"]["base_score"][0])
    for root in t["trees.root"]:
        for i, row in enumerate(xf):
            n = int(root)
            while t["trees.feature"][n] >= 0:
                v = row[t["trees.feature"][n]]
                if np.isnan(v):
                    go_left = bool(t["trees.flags"][n] & 1)
                else:
                    go_left = v < np.float32(t["trees.threshold"][n])
                n = int(t["trees.left"][n] if go_left else t["trees.right"][n])
            margin[i] += t["trees.value"][n]
    np.testing.assert_allclose(oracle.Oracle(model).predict(x)[:, 0], 1 / (1 + np.exp(-margin)), rtol=1e-12,
                               atol=1e-14)


def test_exp_against_libm():
    xs = np.concatenate([np.linspace(-708, 708, 2001), [-1e-300, 0.0, -0.0, 1e-300, 0.5, -0.5]])
    for v in xs:
        got, want = oracle.oracle_exp(v), math.exp(v)
        assert abs(got - want) <= 4 * math.ulp(want), v
    assert oracle.oracle_exp(1000.0) == oracle.oracle_exp(708.0)
    assert oracle.oracle_exp(-1000.0) == oracle.oracle_exp(-708.0)
    assert math.isnan(oracle.oracle_exp(float("nan")))


# --- live reference ------------------------------------------------------

needs_reference = pytest.mark.skipif(not oracle.available_reference(),
                                     reason="oracle/_ref (the reference compiled from its sources) not built")


@needs_reference
@pytest.mark.parametrize("seed", range(6))
def test_random_ensembles_against_reference(seed):
    rng = np.random.default_rng(100 + seed)
    decision, cast = ("le", "lt")[seed % 2], ("f64", "f32")[(seed // 2) % 2]
    outputs = (1, 3)[seed % 2]
    link = ("identity", "softmax")[seed % 2] if outputs > 1 else ("identity", "sigmoid", "exp")[seed % 3]
    model = random_model(rng, features=7, decision=decision, cast=cast, trees=150, outputs=outputs, link=link,
                         inf_thresholds=0.05 * (seed % 3), aggregate=("sum", "mean")[seed % 2])
    x = edge_inputs(rng, 500, 7)
    ref = oracle.Reference()
    o = oracle.Oracle(model)
    assert same_bits(o.predict(x), ref.predict(model, x))
    np.testing.assert_array_equal(o.leaves(x), ref.leaves(model, x))


@needs_reference
@pytest.mark.parametrize("decision, outputs", [("le", 1), ("lt", 1), ("le", 3)])
def test_float32_cast_models_see_only_the_float32_value(decision, outputs):
    """The library rounds pageable float64 rows of float32-cast models
    without preprocessing to float32 on the host. That rests on this
    property of the reference: such a model gives the same bits for float64
    rows as for those rows rounded to float32, threshold neighbours,
    subnormal, overflowing and infinite values included."""
    rng = np.random.default_rng([len(decision), outputs])
    model = random_model(rng, features=6, trees=120, max_depth=10, cast="f32", decision=decision, outputs=outputs,
                         link="softmax" if outputs > 1 else "sigmoid", inf_thresholds=0.05)
    x = edge_inputs(rng, 3000, 6, special=0.3)
    near = rng.random(x.shape) < 0.15
    scale = rng.choice([-1.0, 1.0], size=int(near.sum())) * 10.0 ** rng.uniform(-15, -6, size=int(near.sum()))
    x[near] = rng.choice(GRID, size=int(near.sum())) * (1 + scale) + scale
    odd = rng.random(x.shape) < 0.05
    x[odd] = rng.choice(np.array(NARROWING), size=int(odd.sum()))
    with np.errstate(over="ignore"):
        rounded = x.astype(np.float32).astype(np.float64)
    ref = oracle.Reference()
    assert same_bits(ref.predict(model, x), ref.predict(model, rounded))
    np.testing.assert_array_equal(ref.leaves(model, x), ref.leaves(model, rounded))


@needs_reference
def test_shared_nodes_and_infinite_thresholds_against_reference():
    nodes = export.Nodes()
    split = nodes.add(feature=0, threshold=-np.inf, flags=1 | (1 << 1))
    nodes.left[split] = nodes.add(value=1.0)
    nodes.right[split] = nodes.add(value=2.0)
    model = export.tree_ensemble(nodes, [split, split], [0, 0], features=1).to_bytes()
    x = np.array([[-np.inf], [-1e308], [0.0], [np.inf], [np.nan]])
    ref = oracle.Reference().predict(model, x)
    np.testing.assert_array_equal(ref[:, 0], [2.0, 4.0, 4.0, 4.0, 2.0])
    assert same_bits(oracle.Oracle(model).predict(x), ref)


@needs_reference
@pytest.mark.parametrize("name", ["c1", "c2", "c4", "c5"])
def test_recipes_against_reference(name):
    kw = {"c1": {"trees": 50}, "c2": {"trees": 90}, "c4": {"rounds": 6}, "c5": {"trees": 90}}[name]
    model = getattr(synth, f"model_{name}")(**kw).to_bytes()
    x = getattr(synth, f"inputs_{name}")(batch=300 if name != "c5" else 64)
    ref = oracle.Reference()
    o = oracle.Oracle(model)
    assert same_bits(o.predict(x), ref.predict(model, x))
    np.testing.assert_array_equal(o.leaves(x), ref.leaves(model, x))
