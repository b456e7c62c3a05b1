"""Seeded synthetic tree models and inputs for the five benchmark configurations.

No public dataset or trained model is involved: models come from seed 0 and
inputs from seed 1 (``numpy.random.default_rng``), with the shapes, split
rules, missing-value modes and value distributions of each configuration.
Split thresholds are drawn from the empirical quantiles of a 100k-sample
N(0, 1), like the split points a GBDT library picks from its histogram bins.

    c1  LightGBM-style regression: 100 trees of <= 31 leaves (depth <= 6), 40
        features, ``<=`` splits, NaN missing type, random default side,
        leaves N(0, 0.01), identity; 4096 rows N(0, 1) with 1% NaN.
    c2  XGBoost-style binary classifier: 500 complete depth-8 trees, 128
        features, ``<`` on float32 features, thresholds stored as float32,
        random default side, leaves float32 N(0, 0.05), base_score 0.5
        (margin 0), sigmoid; 1M rows N(0, 1) with 5% NaN.
    c3  scikit-learn RandomForest-style regressor: 200 trees grown by random
        feature / quantile splits on a 100k x 64 N(0, 1) sample to depth <= 20
        with >= 2 samples per leaf, ``<=`` on float32 features, mean of trees;
        1M rows N(0, 1), no missing values.
    c4  LightGBM multiclass: 5 classes x 300 rounds, <= 255 leaves, depth <=
        12, 256 features; features 0-127 use the Zero missing type (inputs have
        10% exact zeros), 128-255 the NaN type (2% NaN); leaves N(0, 0.02);
        softmax; 4M rows.
    c5  low-latency XGBoost-style: 1000 depth-8 trees, 200 features, 1% NaN,
        sigmoid, preprocess mean ~ N(0, 1), scale ~ U(0.5, 2), clip (-8, 8);
        calls of 1, 8 and 64 rows.

Every generator takes size overrides so tests can build the same recipe small.
Nodes are numbered in creation order (breadth-first for grown trees), which
keeps every child after its parent as the file format requires.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Callable

import numpy as np

from . import export

MODEL_SEED, DATA_SEED = 0, 1
_DEFAULT = export.MISSING_DEFAULT
_ZERO_OR_NAN = export.MISSING_ZERO_OR_NAN


def quantile_pool(rng: np.random.Generator, size: int = 100_000) -> np.ndarray:
    return np.sort(rng.standard_normal(size))


def _complete(rng: np.random.Generator, trees: int, depth: int, features: int, pool: np.ndarray,
              leaf_scale: float, f32: bool) -> tuple[dict, np.ndarray]:
    """``trees`` complete trees of ``depth``, each in heap order (children of i
    at 2i+1 and 2i+2), XGBoost-style: thresholds and leaves rounded to float32
    when ``f32``; every split a random default side with the NaN missing mode."""
    internal, per_tree = 2 ** depth - 1, 2 ** (depth + 1) - 1
    n = trees * per_tree
    local = np.tile(np.arange(per_tree, dtype=np.int64), trees)
    base = np.repeat(np.arange(trees, dtype=np.int64) * per_tree, per_tree)
    is_split = local < internal
    feature = np.where(is_split, rng.integers(0, features, size=n), -1).astype(np.int32)
    threshold = pool[rng.integers(0, len(pool), size=n)]
    leaves = rng.normal(0.0, leaf_scale, size=n)
    if f32:
        threshold = threshold.astype(np.float32).astype(np.float64)
        leaves = leaves.astype(np.float32).astype(np.float64)
    default_left = rng.random(n) < 0.5
    nodes = {
        "feature": feature,
        "threshold": np.where(is_split, threshold, 0.0),
        "left": np.where(is_split, base + 2 * local + 1, -1).astype(np.int32),
        "right": np.where(is_split, base + 2 * local + 2, -1).astype(np.int32),
        "value": np.where(is_split, 0.0, leaves),
        "flags": np.where(is_split, default_left.astype(np.uint8) | (_DEFAULT << 1), 0).astype(np.uint8),
    }
    return nodes, (np.arange(trees, dtype=np.int64) * per_tree).astype(np.int32)


def _leafwise(rng: np.random.Generator, trees: int, leaves: int, max_depth: int, features: int, pool: np.ndarray,
              leaf_scale: float, missing_of: Callable[[np.ndarray], np.ndarray]) -> tuple[dict, np.ndarray]:
    """LightGBM-style leaf-wise growth: each tree splits a random leaf shallower
    than ``max_depth`` until it has ``leaves`` leaves. ``missing_of(feature)``
    gives each split's missing mode."""
    feature, left, right, roots = [], [], [], []
    for _ in range(trees):
        root = len(feature)
        roots.append(root)
        feature.append(-1)
        left.append(-1)
        right.append(-1)
        open_leaves, depth = [root], {root: 0}
        picks = rng.random(leaves)
        for k in range(leaves - 1):
            splittable = [i for i in open_leaves if depth[i] < max_depth]
            if not splittable:
                break
            node = splittable[int(picks[k] * len(splittable))]
            open_leaves.remove(node)
            a, b = len(feature), len(feature) + 1
            feature[node] = 0  # marked as a split; the feature is drawn below
            left[node], right[node] = a, b
            for child in (a, b):
                feature.append(-1)
                left.append(-1)
                right.append(-1)
                depth[child] = depth[node] + 1
                open_leaves.append(child)
    feature = np.asarray(feature, dtype=np.int64)
    n = len(feature)
    is_split = feature >= 0
    feat = np.where(is_split, rng.integers(0, features, size=n), -1)
    default_left = (rng.random(n) < 0.5).astype(np.uint8)
    flags = np.where(is_split, default_left | (missing_of(feat).astype(np.uint8) << 1), 0).astype(np.uint8)
    nodes = {
        "feature": feat.astype(np.int32),
        "threshold": np.where(is_split, pool[rng.integers(0, len(pool), size=n)], 0.0),
        "left": np.asarray(left, dtype=np.int32),
        "right": np.asarray(right, dtype=np.int32),
        "value": np.where(is_split, 0.0, rng.normal(0.0, leaf_scale, size=n)),
        "flags": flags,
    }
    return nodes, np.asarray(roots, dtype=np.int32)


_SAMPLE: tuple | None = None  # (x, y) of the forest being grown, set once per worker process


def _set_sample(x: np.ndarray, y: np.ndarray) -> None:
    global _SAMPLE
    _SAMPLE = (x, y)


def _grow(seed: list, features: int, max_depth: int, min_leaf: int) -> tuple:
    """One random-split tree on the sample set by _set_sample, from its own
    seed: (feature, threshold, child, value) arrays in breadth-first order."""
    x, y = _SAMPLE
    rng = np.random.default_rng(seed)
    samples = len(x)
    cap = 4 * samples
    feat = np.full(cap, -1, dtype=np.int64)
    thr = np.zeros(cap)
    kid = np.full(cap, -1, dtype=np.int64)
    val = np.zeros(cap)
    count = 1
    live = np.arange(samples)
    at = np.zeros(samples, dtype=np.int64)
    first, width = 0, 1
    for level in range(max_depth + 1):
        local = at[live] - first
        n_at = np.bincount(local, minlength=width)
        y_at = np.bincount(local, weights=y[live], minlength=width)
        val[first:first + width] = y_at / np.maximum(n_at, 1)
        can = (n_at >= 2 * min_leaf) & (level < max_depth)
        if not can.any():
            break
        choice = rng.integers(0, features, size=width)
        keep = can[local]
        live, local = live[keep], local[keep]
        v = x[live, choice[local]]
        order = np.lexsort((v, local))
        live, local, v = live[order], local[order], v[order]
        split = np.flatnonzero(can)
        n = n_at[split]
        starts = np.concatenate([[0], np.cumsum(n)])[:-1]
        k = min_leaf + np.floor(rng.random(len(split)) * (n - 2 * min_leaf + 1)).astype(np.int64)
        lo = v[starts + k - 1].astype(np.float64)
        hi = v[starts + k].astype(np.float64)
        ok = hi > lo  # equal neighbours cannot be separated: that node stays a leaf
        good = split[ok]
        if len(good) == 0:
            break
        mid = (lo + (hi - lo) / 2.0)[ok]
        children = count + 2 * np.arange(len(good))
        feat[first + good] = choice[good]
        thr[first + good] = mid
        kid[first + good] = children
        child_of = np.full(width, -1, dtype=np.int64)
        child_of[good] = children
        thr_of = np.full(width, np.inf)
        thr_of[good] = mid
        c = child_of[local]
        moving = c >= 0
        at[live[moving]] = c[moving] + (v[moving] > thr_of[local[moving]])
        live = live[moving]
        first, width = count, 2 * len(good)
        count += width
    return feat[:count], thr[:count], kid[:count], val[:count]


def _forest(rng: np.random.Generator, trees: int, samples: int, features: int, max_depth: int,
            min_leaf: int = 2, seed: int = MODEL_SEED) -> tuple[dict, np.ndarray]:
    """Random-split regression trees grown breadth-first on a N(0, 1) sample:
    each node of >= 2 * min_leaf samples above the depth limit splits a random
    feature between two adjacent sorted sample values (their midpoint, in
    float64 of float32 features, as scikit-learn does), with a random number of
    samples in [min_leaf, n - min_leaf] on the left. Leaves hold the mean target
    of their samples. Tree t draws from its own seed (seed, 3, t), so large
    forests grow in parallel worker processes (started with spawn, which is
    safe after CUDA was initialised) with the same result."""
    x = rng.standard_normal((samples, features)).astype(np.float32)
    y = np.sin(x[:, 0]) + 0.5 * x[:, 1] * x[:, 2] + 0.1 * rng.standard_normal(samples)
    seeds = [[seed, 3, t] for t in range(trees)]
    workers = min(trees, os.cpu_count() or 1)
    if workers > 1 and trees * samples >= 4_000_000:
        import multiprocessing
        from concurrent.futures import ProcessPoolExecutor

        with ProcessPoolExecutor(workers, mp_context=multiprocessing.get_context("spawn"), initializer=_set_sample,
                                 initargs=(x, y)) as pool:
            grown = list(pool.map(_grow, seeds, [features] * trees, [max_depth] * trees, [min_leaf] * trees))
    else:
        _set_sample(x, y)
        grown = [_grow(sd, features, max_depth, min_leaf) for sd in seeds]
    parts: dict[str, list] = {k: [] for k in ("feature", "threshold", "left", "right", "value", "flags")}
    roots, total = [], 0
    for feat, thr, kid, val in grown:
        count = len(feat)
        roots.append(total)
        is_split = feat >= 0
        parts["feature"].append(feat.astype(np.int32))
        parts["threshold"].append(thr)
        parts["left"].append(np.where(is_split, kid + total, -1).astype(np.int32))
        parts["right"].append(np.where(is_split, kid + 1 + total, -1).astype(np.int32))
        parts["value"].append(np.where(is_split, 0.0, val))
        parts["flags"].append(np.where(is_split, 1 | (_DEFAULT << 1), 0).astype(np.uint8))
        total += count
    nodes = {k: np.concatenate(v) for k, v in parts.items()}
    return nodes, np.asarray(roots, dtype=np.int32)


# ---------------------------------------------------------------------------
# The five configurations
# ---------------------------------------------------------------------------


@dataclass
class Config:
    name: str
    batch: int
    model: Callable[..., export.Exported]
    inputs: Callable[..., np.ndarray]
    describe: str


def model_c1(trees: int = 100, features: int = 40) -> export.Exported:
    rng = np.random.default_rng(MODEL_SEED)
    pool = quantile_pool(rng)
    nodes, roots = _leafwise(rng, trees, 31, 6, features, pool, 0.01, lambda f: np.full(f.shape, _DEFAULT))
    return export.tree_ensemble(nodes, roots, np.zeros(len(roots), np.int32), features=features,
                                metadata={"synthetic": "c1"})


def inputs_c1(batch: int = 4096, features: int = 40) -> np.ndarray:
    rng = np.random.default_rng(DATA_SEED)
    x = rng.standard_normal((batch, features))
    x[rng.random(x.shape) < 0.01] = np.nan
    return x


def model_c2(trees: int = 500, depth: int = 8, features: int = 128) -> export.Exported:
    rng = np.random.default_rng(MODEL_SEED)
    pool = quantile_pool(rng)
    nodes, roots = _complete(rng, trees, depth, features, pool, 0.05, f32=True)
    # base_score 0.5 under binary:logistic is margin log(0.5 / 0.5) = 0.
    return export.tree_ensemble(nodes, roots, np.zeros(trees, np.int32), features=features, decision="lt",
                                feature_cast="f32", link="sigmoid", base_score=0.0, metadata={"synthetic": "c2"})


def inputs_c2(batch: int = 1_000_000, features: int = 128, nan: float = 0.05) -> np.ndarray:
    rng = np.random.default_rng(DATA_SEED)
    x = rng.standard_normal((batch, features))
    x[rng.random(x.shape) < nan] = np.nan
    return x


def model_c3(trees: int = 200, samples: int = 100_000, features: int = 64, max_depth: int = 20) -> export.Exported:
    rng = np.random.default_rng(MODEL_SEED)
    nodes, roots = _forest(rng, trees, samples, features, max_depth)
    return export.tree_ensemble(nodes, roots, np.zeros(len(roots), np.int32), features=features, decision="le",
                                feature_cast="f32", aggregate="mean", metadata={"synthetic": "c3"})


def inputs_c3(batch: int = 1_000_000, features: int = 64) -> np.ndarray:
    return np.random.default_rng(DATA_SEED).standard_normal((batch, features))


def model_c4(rounds: int = 300, classes: int = 5, leaves: int = 255, max_depth: int = 12,
             features: int = 256) -> export.Exported:
    rng = np.random.default_rng(MODEL_SEED)
    pool = quantile_pool(rng)
    half = features // 2
    nodes, roots = _leafwise(rng, rounds * classes, leaves, max_depth, features, pool, 0.02,
                             lambda f: np.where(f < half, _ZERO_OR_NAN, _DEFAULT))
    outputs = np.arange(len(roots), dtype=np.int32) % classes
    return export.tree_ensemble(nodes, roots, outputs, features=features, outputs=classes, link="softmax",
                                metadata={"synthetic": "c4"})


def inputs_c4(batch: int = 4_000_000, features: int = 256) -> np.ndarray:
    rng = np.random.default_rng(DATA_SEED)
    x = rng.standard_normal((batch, features))
    half = features // 2
    x[:, :half][rng.random((batch, half)) < 0.10] = 0.0
    x[:, half:][rng.random((batch, features - half)) < 0.02] = np.nan
    return x


def c5_preprocess(features: int = 200) -> tuple[np.ndarray, np.ndarray]:
    """c5's standardisation: mean ~ N(0, 1), scale ~ U(0.5, 2) per feature."""
    rng = np.random.default_rng([MODEL_SEED, 5])
    return rng.standard_normal(features), rng.uniform(0.5, 2.0, features)


def model_c5(trees: int = 1000, depth: int = 8, features: int = 200) -> export.Exported:
    rng = np.random.default_rng(MODEL_SEED)
    pool = quantile_pool(rng)
    nodes, roots = _complete(rng, trees, depth, features, pool, 0.05, f32=True)
    mean, scale = c5_preprocess(features)
    return export.tree_ensemble(nodes, roots, np.zeros(trees, np.int32), features=features, decision="lt",
                                feature_cast="f32", link="sigmoid", base_score=0.0,
                                preprocess={"mean": mean, "scale": scale, "clip": (-8.0, 8.0)},
                                metadata={"synthetic": "c5"})


def inputs_c5(batch: int = 64, features: int = 200) -> np.ndarray:
    """Raw inputs around the preprocess mean, so (x - mean) / scale is about
    N(0, 1), with 1% NaN."""
    mean, scale = c5_preprocess(features)
    rng = np.random.default_rng(DATA_SEED)
    z = rng.standard_normal((batch, features))
    z[rng.random(z.shape) < 0.01] = np.nan
    return mean + scale * z


CONFIGS = {
    "c1": Config("c1", 4096, model_c1, inputs_c1, "LightGBM regression, 100 trees <=31 leaves, F=40, 4096 rows"),
    "c2": Config("c2", 1_000_000, model_c2, inputs_c2, "XGBoost binary, 500 depth-8 trees, F=128, 1M rows"),
    "c3": Config("c3", 1_000_000, model_c3, inputs_c3, "RandomForest regressor, 200 trees depth<=20, F=64, 1M rows"),
    "c4": Config("c4", 4_000_000, model_c4, inputs_c4, "LightGBM multiclass 5x300, <=255 leaves, F=256, 4M rows"),
    "c5": Config("c5", 64, model_c5, inputs_c5, "low-latency XGBoost, 1000 depth-8 trees, F=200, preprocess"),
}
