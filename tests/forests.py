"""Test models: random ensembles over every missing-value mode, and inputs
full of the values that sit exactly on split rules (NaN, signed zeros,
LightGBM's zero band, infinities, thresholds themselves)."""

from __future__ import annotations

import functools

import numpy as np

from montlok import export

GRID = np.array([-1.5, -0.25, 0.0, 0.5, 2.0])
SPECIALS = [np.nan, 0.0, -0.0, 1e-35, -1e-36, 1e-36, np.inf, -np.inf, 1e-300, -1e-300, *GRID]
# Doubles whose float32 rounding is subnormal, zero, the largest float or
# infinite.
NARROWING = [1e-40, -1e-40, 1e-46, -1e-46, 8e-46, 3.5e38, -3.5e38, 3.4028235677973366e38, 3.4028235e38 * (1 + 1e-9)]


def random_model(rng: np.random.Generator, features: int = 5, decision: str = "le", cast: str = "f64",
                 trees: int = 40, outputs: int = 1, link: str = "identity", aggregate: str = "sum",
                 max_depth: int = 8, inf_thresholds: float = 0.0, base=0.25, sigmoid_scale: float = 1.0,
                 preprocess=None, share: bool = False, tree_outputs=None) -> bytes:
    """Trees of random depth; every split a random feature, threshold (grid or
    normal, optionally infinite), default side and missing mode."""
    nodes = export.Nodes()
    roots = []
    for _ in range(trees):
        depth = int(rng.integers(1, max_depth + 1))

        def grow(level: int) -> int:
            if level == depth or (level > 0 and rng.random() < 0.2):
                return nodes.add(value=float(rng.normal()))
            flags = int(rng.integers(2)) | (int(rng.integers(3)) << 1)
            if rng.random() < inf_thresholds:
                threshold = float(rng.choice([np.inf, -np.inf]))
            elif rng.random() < 0.5:
                threshold = float(rng.choice(GRID))
            else:
                threshold = float(rng.normal())
            i = nodes.add(feature=int(rng.integers(features)), threshold=threshold, flags=flags)
            nodes.left[i] = grow(level + 1)
            nodes.right[i] = grow(level + 1)
            return i

        roots.append(grow(0))
    if share and len(roots) > 1:
        roots[-1] = roots[0]
    if tree_outputs is None:
        tree_outputs = [t % outputs for t in range(trees)]
    return export.tree_ensemble(nodes, roots, tree_outputs, features=features, outputs=outputs, decision=decision,
                                feature_cast=cast, aggregate=aggregate, link=link, base_score=base,
                                sigmoid_scale=sigmoid_scale, preprocess=preprocess).to_bytes()


def edge_inputs(rng: np.random.Generator, rows: int, features: int, special: float = 0.4) -> np.ndarray:
    x = rng.normal(size=(rows, features))
    pick = rng.random((rows, features)) < special
    x[pick] = rng.choice(np.array(SPECIALS), size=int(pick.sum()))
    return x


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    """Equal as float64 bit patterns, every NaN counting as equal to any NaN."""
    a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
    if a.shape != b.shape:
        return False
    nan = np.isnan(a)
    return bool(np.array_equal(nan, np.isnan(b)) and np.array_equal(a[~nan].view(np.int64), b[~nan].view(np.int64)))


@functools.lru_cache(maxsize=None)
def full_model(name: str) -> bytes:
    """The benchmark recipe `name` at its configured size (built once per process)."""
    from montlok import synth

    return synth.CONFIGS[name].model().to_bytes()


def near_thresholds(model: bytes, x: np.ndarray, rng: np.random.Generator, frac: float = 0.08) -> np.ndarray:
    """A copy of `x` with a fraction of its values moved onto the split rules of
    the model's own trees: each picked (row, feature) takes a threshold of a
    random split on that feature, exactly, one double ulp either side, its
    float32 rounding, the float32 neighbours of that, or the midpoints between
    them (doubles that round to the float32 value from above or below)."""
    spec, t = export.read(model)
    p = (spec.get("config") or {}).get("tensors", "trees")
    feature, threshold = t[p + ".feature"], t[p + ".threshold"]
    split = feature >= 0
    by_feature: dict[int, np.ndarray] = {}
    for f in np.unique(feature[split]):
        values = threshold[split & (feature == f)]
        by_feature[int(f)] = values[np.isfinite(values)]
    y = np.array(x, dtype=np.float64, copy=True)
    rows, cols = np.nonzero(rng.random(y.shape) < frac)
    for r, c in zip(rows, cols):
        pool = by_feature.get(int(c))
        if pool is None or len(pool) == 0:
            continue
        th = float(pool[rng.integers(len(pool))])
        f32 = np.float32(th)
        up32, down32 = np.nextafter(f32, np.float32(np.inf)), np.nextafter(f32, np.float32(-np.inf))
        choices = [th, np.nextafter(th, np.inf), np.nextafter(th, -np.inf), float(f32), float(up32), float(down32),
                   (float(f32) + float(up32)) / 2, (float(f32) + float(down32)) / 2]
        y[r, c] = choices[int(rng.integers(len(choices)))]
    return y
