"""The model-file writer and reader (montlok.export).

The file format has to match the reference's byte for byte (readers of
either build open files of both): these tests write the same models with
both exporters and compare the bytes, when the reference sources are here.
"""

from __future__ import annotations

import importlib.util
import json
import os
import struct
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle
from golden.make_golden import lightgbm_dump, xgboost_tree
from montlok import export, synth

REF = oracle.reference_sources()


@pytest.fixture(scope="module")
def ref_export():
    if REF is None:
        pytest.skip("reference sources absent (set MONTLOK_REFERENCE)")
    path = REF / "python/montlok/export.py"
    spec = importlib.util.spec_from_file_location("montlok_reference_export_t", path)
    module = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = module
    spec.loader.exec_module(module)
    return module


def strip_exporter(data: bytes) -> tuple[dict, dict]:
    spec, tensors = export.read(data)
    spec["metadata"].pop("exporter", None)
    return spec, tensors


def test_round_trip():
    rng = np.random.default_rng(0)
    e = export.tree_ensemble({"feature": [0, -1, -1], "threshold": [0.5, 0, 0], "left": [1, -1, -1],
                              "right": [2, -1, -1], "value": [0, 1.5, -2.0], "flags": [3, 0, 0]}, [0], [0],
                             features=2, preprocess={"mean": rng.normal(size=2), "scale": [1.0, 2.0], "clip": (-3, 3)},
                             feature_names=["a", "b"])
    data = e.to_bytes()
    (length,) = struct.unpack_from("<Q", data)
    assert (8 + length) % 8 == 0
    spec, tensors = export.read(data)
    assert spec == e.spec
    for name, value in e.tensors.items():
        np.testing.assert_array_equal(tensors[name], value)
    header = json.loads(data[8:8 + length])
    for name, entry in header.items():
        if name != "__metadata__":
            width = np.dtype(export._FROM_TAG[entry["dtype"]]).itemsize
            assert entry["data_offsets"][0] % width == 0


def test_lightgbm_matches_reference_bytes(ref_export):
    for objective, k in (("regression", 1), ("binary sigmoid:0.7", 1), ("multiclass num_class:3", 3),
                         ("poisson", 1)):
        dump = lightgbm_dump(objective, k, 12, 5, seed=k)
        mine = export.from_lightgbm(json.dumps(dump)).to_bytes()
        theirs = ref_export.from_lightgbm(json.dumps(dump)).to_bytes()
        assert strip_exporter(mine)[0] == strip_exporter(theirs)[0]
        a, b = strip_exporter(mine)[1], strip_exporter(theirs)[1]
        assert a.keys() == b.keys()
        for name in a:
            np.testing.assert_array_equal(a[name], b[name])


def test_xgboost_matches_reference_bytes(ref_export):
    trees = [json.dumps(xgboost_tree(np.random.default_rng(i), 6)) for i in range(9)]
    for objective, kw in (("binary:logistic", {"base_score": 0.3}), ("reg:squarederror", {"base_score": 0.5}),
                          ("multi:softprob", {"base_score": 0.5, "classes": 3}), ("count:poisson", {"base_score": 2.0})):
        mine = export.from_xgboost(trees, features=6, objective=objective, **kw).to_bytes()
        theirs = ref_export.from_xgboost(trees, features=6, objective=objective, **kw).to_bytes()
        assert strip_exporter(mine)[0] == strip_exporter(theirs)[0]
        a, b = strip_exporter(mine)[1], strip_exporter(theirs)[1]
        for name in a:
            np.testing.assert_array_equal(a[name], b[name])


def test_same_bytes_when_the_exporter_string_matches(ref_export):
    dump = lightgbm_dump("regression", 1, 5, 4, seed=3)
    mine = export.from_lightgbm(json.dumps(dump)).with_metadata(exporter="x")
    theirs = ref_export.from_lightgbm(json.dumps(dump)).with_metadata(exporter="x")
    assert mine.to_bytes() == theirs.to_bytes()


def test_sklearn_trees_match_reference(ref_export):
    from sklearn import ensemble, tree

    rng = np.random.default_rng(0)
    x = rng.normal(size=(300, 5))
    x[rng.random(x.shape) < 0.05] = np.nan
    y = np.sin(np.nan_to_num(x[:, 0])) + np.nan_to_num(x[:, 1])
    for est in (tree.DecisionTreeRegressor(max_depth=6, random_state=0),
                ensemble.RandomForestRegressor(n_estimators=5, max_depth=5, random_state=0),
                ensemble.GradientBoostingRegressor(n_estimators=8, max_depth=3, random_state=0),
                ensemble.HistGradientBoostingRegressor(max_iter=6, random_state=0)):
        xx = np.nan_to_num(x) if type(est).__name__ == "GradientBoostingRegressor" else x
        est.fit(xx, y)
        a = strip_exporter(export.from_sklearn(est).to_bytes())
        b = strip_exporter(ref_export.from_sklearn(est).to_bytes())
        assert a[0] == b[0]
        for name in a[1]:
            np.testing.assert_array_equal(a[1][name], b[1][name])


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4", "c5"])
def test_recipes_are_seeded(name):
    kw = {"c1": {"trees": 5}, "c2": {"trees": 5}, "c3": {"trees": 1, "samples": 500}, "c4": {"rounds": 1},
          "c5": {"trees": 5}}[name]
    a = getattr(synth, f"model_{name}")(**kw).to_bytes()
    b = getattr(synth, f"model_{name}")(**kw).to_bytes()
    assert a == b
    x1 = getattr(synth, f"inputs_{name}")(batch=16)
    x2 = getattr(synth, f"inputs_{name}")(batch=16)
    np.testing.assert_array_equal(x1, x2)
