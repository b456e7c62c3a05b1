"""The reference's own C++ consumer test, run against this library.

oracle/_ref/test_core_consumer is the reference's tests/cpp/test_core.cpp,
compiled unchanged against the reference's headers (its montlok.hpp C++
wrapper over its montlok.h) and linked to this repository's libmontlok.so
(oracle/Makefile, target `consumer`): a C++ program built for the reference
must run on the GPU library with no change. It replays two fixtures from a
data directory through the C ABI at 1e-12 relative, checks that a one-row
stream step equals predict, that latency threads can be set and cleared,
that garbage bytes fail with MONTLOK_ERROR_FORMAT and that a wrong input size
fails with MONTLOK_ERROR_SHAPE.

The directory holds the reference's `gbr` fixture (tests/golden/gbr.*, a
scikit-learn gradient-boosting regressor, with the outputs the reference
produced) and, under the name the test expects for its second fixture, a
tree-ensemble model: the reference's second fixture is a GRU, a family
outside this build. That model (softmax over 3 classes, preprocessing,
missing values) is written with its three input rows and the outputs of the
oracle, the CPU restatement pinned to the reference in test_oracle.py.
"""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle
from forests import edge_inputs, random_model

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_reference_cpp_consumer_runs_unchanged(gpu, tmp_path):
    if not oracle.CONSUMER.exists():
        pytest.skip("the consumer test was not built (it needs the reference sources at build time)")
    for suffix in ("montlok", "io"):
        shutil.copyfile(GOLDEN / f"gbr.{suffix}", tmp_path / f"gbr.{suffix}")
    rng = np.random.default_rng(12)
    pre = {"mean": rng.normal(size=5), "scale": rng.uniform(0.5, 2.0, 5), "clip": (-4.0, 4.0)}
    model = random_model(rng, features=5, trees=60, outputs=3, link="softmax", preprocess=pre,
                         base=[0.1, -0.2, 0.3])
    x = edge_inputs(rng, 3, 5, special=0.2)
    y = oracle.Oracle(model).predict(x)
    (tmp_path / "gru.montlok").write_bytes(model)
    np.concatenate([x.ravel(), y.ravel()]).astype("<f8").tofile(tmp_path / "gru.io")
    r = subprocess.run([str(oracle.CONSUMER), str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all checks passed" in r.stdout
    assert "gbr: predict matches the Python binding" in r.stdout
