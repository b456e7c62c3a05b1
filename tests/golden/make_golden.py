#!/usr/bin/env python3
"""Regenerates the golden fixtures in this directory from the reference.

Needs the montlok.cpp sources (their directory in MONTLOK_REFERENCE) and
the reference library compiled from them (``make -C oracle ref``); it is
run by hand in the development container, never on the GPU box, and its
outputs are committed:

* ``gbr.montlok`` / ``gbr.io`` - copied verbatim from the reference's own
  fixture (tests/data): an sklearn GradientBoostingRegressor of 25 depth-3
  trees on 4 features; ``.io`` holds 3 input rows (one NaN) and then the 3
  outputs the reference produced, little-endian float64.
* ``<case>.npz`` - for each case: the model file bytes, float64 inputs, the
  reference's predictions (``out``) and the node index of the leaf the
  reference reached in every tree (``leaves``, read through the leaf-id
  re-export of oracle/oracle.py). Models are written with the reference's
  own exporter (python/montlok/export.py, imported from the sources) where a
  dump format applies, so the fixtures do not depend on this build's writer.
"""

from __future__ import annotations

import importlib.util
import json
import os
import shutil
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT / "montlok.cpp_b200" / "python"))
sys.path.insert(0, str(ROOT / "tests"))

import oracle  # noqa: E402

REF = oracle.reference_sources()
from forests import edge_inputs, random_model  # noqa: E402
from montlok import synth  # noqa: E402


def reference_export():
    spec = importlib.util.spec_from_file_location("montlok_reference_export", REF / "python/montlok/export.py")
    module = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = module  # dataclasses look their module up
    spec.loader.exec_module(module)
    return module


def lightgbm_tree(rng, depth, features, missing_types=("None", "Zero", "NaN")):
    if depth == 0 or rng.random() < 0.2:
        return {"leaf_value": float(rng.normal())}
    return {"split_feature": int(rng.integers(features)), "threshold": float(rng.normal()), "decision_type": "<=",
            "default_left": bool(rng.random() < 0.5), "missing_type": str(rng.choice(list(missing_types))),
            "left_child": lightgbm_tree(rng, depth - 1, features, missing_types),
            "right_child": lightgbm_tree(rng, depth - 1, features, missing_types)}


def lightgbm_dump(objective, per_round, trees, features, seed):
    rng = np.random.default_rng(seed)
    return {"name": "tree", "version": "v4", "num_class": per_round, "num_tree_per_iteration": per_round,
            "max_feature_idx": features - 1, "objective": objective, "average_output": False,
            "feature_names": [f"x{i}" for i in range(features)],
            "tree_info": [{"tree_index": i, "tree_structure": lightgbm_tree(rng, 6, features)} for i in range(trees)]}


def xgboost_tree(rng, features, depth=5):
    counter = iter(range(10_000))

    def node(level):
        nodeid = next(counter)
        if level == depth or rng.random() < 0.2:
            return {"nodeid": nodeid, "leaf": float(np.float32(rng.normal()))}
        left, right = node(level + 1), node(level + 1)
        return {"nodeid": nodeid, "depth": level, "split": f"f{rng.integers(features)}",
                "split_condition": float(np.float32(rng.normal())), "yes": left["nodeid"], "no": right["nodeid"],
                "missing": left["nodeid"] if rng.random() < 0.5 else right["nodeid"], "children": [left, right]}

    return node(0)


def cases(ref_export):
    rng = np.random.default_rng(2024)
    out = {}
    for objective, k in (("regression", 1), ("binary sigmoid:0.7", 1), ("multiclass num_class:3", 3)):
        name = "lightgbm_" + objective.split()[0]
        dump = lightgbm_dump(objective, k, 24, 5, seed=len(name))
        out[name] = (ref_export.from_lightgbm(json.dumps(dump)).to_bytes(), edge_inputs(rng, 300, 5))
    trees = [json.dumps(xgboost_tree(np.random.default_rng(7 + i), 5)) for i in range(20)]
    out["xgboost_logistic"] = (ref_export.from_xgboost(trees, features=5, objective="binary:logistic",
                                                       base_score=0.3).to_bytes(), edge_inputs(rng, 300, 5))
    out["xgboost_softmax"] = (ref_export.from_xgboost(trees[:18], features=5, objective="multi:softprob",
                                                      base_score=0.5, classes=3).to_bytes(), edge_inputs(rng, 300, 5))
    for decision in ("le", "lt"):
        for cast in ("f64", "f32"):
            name = f"edge_{decision}_{cast}"
            model = random_model(np.random.default_rng([3, len(decision), len(cast)]), features=6, decision=decision,
                                 cast=cast, trees=90, inf_thresholds=0.1)
            out[name] = (model, edge_inputs(rng, 400, 6))
    out["mean_exp"] = (random_model(np.random.default_rng(11), features=6, trees=140, outputs=4, link="exp",
                                    aggregate="mean", base=[0.1, -0.2, 0.3, 0.0]), edge_inputs(rng, 200, 6, 0.2))
    out["softmax_12"] = (random_model(np.random.default_rng(12), features=6, trees=200, outputs=12, link="softmax"),
                         edge_inputs(rng, 200, 6, 0.2))
    pre = {"mean": rng.normal(size=6) * 2, "scale": rng.uniform(0.5, 2, 6), "clip": (-1.5, 1.25)}
    out["preprocess_f64"] = (random_model(np.random.default_rng(13), features=6, trees=80, preprocess=pre),
                             edge_inputs(rng, 300, 6) * 2 + pre["mean"])
    out["preprocess_f32_sigmoid"] = (random_model(np.random.default_rng(14), features=6, trees=80, cast="f32",
                                                  decision="lt", link="sigmoid", sigmoid_scale=0.7, preprocess=pre),
                                     edge_inputs(rng, 300, 6) * 2 + pre["mean"])
    # The benchmark recipes, small.
    out["c1"] = (synth.model_c1(trees=30).to_bytes(), synth.inputs_c1(batch=256))
    out["c2"] = (synth.model_c2(trees=70).to_bytes(), synth.inputs_c2(batch=256))
    out["c3"] = (synth.model_c3(trees=3, samples=3000).to_bytes(), synth.inputs_c3(batch=256))
    out["c4"] = (synth.model_c4(rounds=4).to_bytes(), synth.inputs_c4(batch=256))
    out["c5"] = (synth.model_c5(trees=70).to_bytes(), synth.inputs_c5(batch=64))
    return out


def main() -> None:
    if REF is None:
        raise SystemExit("the reference sources are needed: set MONTLOK_REFERENCE to their directory")
    oracle.build(reference=True)
    ref = oracle.Reference()
    ref_export = reference_export()
    for name in ("gbr.montlok", "gbr.io"):
        shutil.copyfile(REF / "tests" / "data" / name, HERE / name)
    for name, (model, x) in cases(ref_export).items():
        x = np.ascontiguousarray(x, dtype=np.float64)
        out = ref.predict(model, x)
        leaves = ref.leaves(model, x)
        np.savez_compressed(HERE / f"{name}.npz", model=np.frombuffer(model, dtype=np.uint8), x=x, out=out,
                            leaves=leaves)
        print(f"{name}: {len(x)} rows, {leaves.shape[1]} trees, {out.shape[1]} outputs")


if __name__ == "__main__":
    main()
