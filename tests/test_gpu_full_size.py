"""Parity at the benchmarked model sizes, kernel by kernel.

The benchmark configurations run their kernels at shapes the smaller parity
cases do not reach: the complete-tree kernel combines 64-tree blocks in rounds
of four teams, so only ensembles of more than 256 trees (c2: 500 trees, 8
blocks, 2 rounds; c5: 1000 trees, 4 rounds) exercise its later rounds; the
multi-output kernel streams 300 trees per class for c4; the deep-tree kernel
walks c3's 200 trees grown on 100k samples. Each case builds the recipe at its
configured size, predicts a few thousand of the configuration's own rows with
NaN, exact zeros and values on and beside the model's thresholds mixed in,
checks which kernel ran, and compares every prediction bit for bit and every
(row, tree) leaf index with the oracle (the reference's predict restated in C,
pinned to the reference itself in test_oracle.py and test_full_size_pins.py).
"""

from __future__ import annotations

import numpy as np
import pytest

import montlok
from forests import full_model, near_thresholds, random_model, same_bits
from montlok import synth
from oracle import Oracle

pytestmark = pytest.mark.gpu


def check(model: bytes, x: np.ndarray, kernel: str, leaves: bool = True) -> None:
    m = montlok.load(model)
    assert m.kernel(len(x)) == kernel
    o = Oracle(model)
    want = o.predict(x)
    got = m.predict(x)
    assert same_bits(got.reshape(want.shape), want), "predictions differ from the oracle"
    if leaves:
        np.testing.assert_array_equal(m.predict_leaves(x).reshape(len(x), -1), o.leaves(x))


def edge_rows(model: bytes, x: np.ndarray, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    y = near_thresholds(model, x, rng)
    y[rng.random(y.shape) < 0.02] = np.nan
    y[rng.random(y.shape) < 0.02] = 0.0
    y[rng.random(y.shape) < 0.005] = -0.0
    return y


@pytest.mark.parametrize("rows", [6000, 300])
def test_c2_full_size_heap_kernel(gpu, rows):
    """500 complete depth-8 trees: 8 blocks over 4 teams, 2 rounds."""
    model = full_model("c2")
    check(model, edge_rows(model, synth.inputs_c2(batch=rows), 21), "complete-tree")


# Batches of at least 148 x 128 rows keep 128 rows per CTA: the staged kernel,
# whose producer warps prepare each CTA's next row group in tensor memory.
# 40,000 rows are 313 groups, two or three per CTA, the last one partial.
STAGED_ROWS = 40_000


def test_c2_full_size_staged_kernel(gpu):
    model = full_model("c2")
    check(model, edge_rows(model, synth.inputs_c2(batch=STAGED_ROWS), 23), "complete-tree-staged")


@pytest.mark.parametrize("trees", [257, 777])
@pytest.mark.parametrize("cast, decision", [("f32", "lt"), ("f64", "le")])
def test_staged_kernel_every_missing_mode(gpu, trees, cast, decision):
    """Every missing mode (all four key variants of a feature staged),
    infinite thresholds, float32 and float64 features, partial blocks and
    rounds, float64 and float32 inputs."""
    rng = np.random.default_rng([trees, len(cast), len(decision), 1])
    model = random_model(rng, features=9, trees=trees, max_depth=8, cast=cast, decision=decision,
                         inf_thresholds=0.05, link="sigmoid", base=0.4)
    x = near_thresholds(model, rng.normal(size=(STAGED_ROWS + 77, 9)), rng, frac=0.2)
    x[rng.random(x.shape) < 0.05] = np.nan
    x[rng.random(x.shape) < 0.02] = 0.0
    check(model, x, "complete-tree-staged", leaves=False)
    x32 = x.astype(np.float32)
    assert same_bits(montlok.load(model).predict(x32).reshape(-1, 1), Oracle(model).predict(x32))


def test_c5_full_size_heap_kernel(gpu):
    """1000 trees with preprocessing: 16 blocks, 4 rounds, at a batch above
    the small-batch kernel's."""
    model = full_model("c5")
    x = synth.inputs_c5(batch=4096)
    x[np.random.default_rng(5).random(x.shape) < 0.01] = np.nan
    check(model, x, "complete-tree")


def test_c5_full_size_small_batch_kernel(gpu):
    model = full_model("c5")
    check(model, synth.inputs_c5(batch=64), "small-batch")


def test_c1_full_size_heap_kernel(gpu):
    model = full_model("c1")
    check(model, edge_rows(model, synth.inputs_c1(batch=4096), 11), "complete-tree")


@pytest.mark.parametrize("trees", [257, 300, 520, 777])
@pytest.mark.parametrize("cast, decision", [("f32", "lt"), ("f64", "le")])
def test_heap_kernel_later_rounds(gpu, trees, cast, decision):
    """Random one-output forests of depth <= 8 (every missing mode, infinite
    thresholds, float32 and float64 features) past four blocks: partial last
    blocks, partial last rounds, teams with no block in the last round."""
    rng = np.random.default_rng([trees, len(cast), len(decision)])
    model = random_model(rng, features=9, trees=trees, max_depth=8, cast=cast, decision=decision,
                         inf_thresholds=0.05, link="sigmoid", base=0.4)
    x = near_thresholds(model, rng.normal(size=(3000, 9)), rng, frac=0.2)
    x[rng.random(x.shape) < 0.05] = np.nan
    check(model, x, "complete-tree")


def test_c4_full_size_multi_output_kernel(gpu):
    """5 classes x 300 rounds of leaf-wise trees up to depth 12, Zero and NaN
    missing types, softmax."""
    model = full_model("c4")
    check(model, edge_rows(model, synth.inputs_c4(batch=3000), 41), "multi-output")


def test_c3_full_size_deep_tree_kernel(gpu):
    """200 random-split trees grown to depth 20 on the 100k-row sample, mean."""
    model = full_model("c3")
    check(model, edge_rows(model, synth.inputs_c3(batch=3000), 31), "deep-tree")
