"""Write and read montlok model files, and build ``tree_ensemble`` models.

A model file is a safetensors file: an 8-byte little-endian header length, a
JSON header naming every tensor (dtype, shape, byte range), the tensor bytes,
and the model spec as the JSON string ``__metadata__["montlok"]`` with schema
``montlok.model/1``.  The layout matches the reference writer
(python/montlok/export.py:75-96 in montlok.cpp) byte for byte: tensors sorted by
descending element size and then name, so each one starts at a multiple of its
element size, and the header padded with spaces to a multiple of 8 bytes.

Tree models are flat node tables (reference src/core/trees.cpp:5-14):

    trees.root i32[T], trees.output i32[T]
    trees.feature i32[N] (-1 = leaf), trees.threshold f64[N],
    trees.left i32[N], trees.right i32[N], trees.value f64[N],
    trees.flags u8[N]: bit 0 missing goes left; bits 1-2 missing mode
                       (0: NaN reads as 0.0, 1: NaN takes the default branch,
                        2: NaN and |x| <= 1e-35 take it, LightGBM "Zero")

``from_lightgbm`` reads LightGBM ``dump_model()`` dicts and ``from_xgboost``
XGBoost JSON tree dumps, the way the reference converters do
(export.py:542-593 and :608-682): neither library is needed.
"""

from __future__ import annotations

import json
import math
import os
import re
import struct
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Mapping, Sequence

import numpy as np

SCHEMA = "montlok.model/1"

__all__ = ["SCHEMA", "Exported", "Nodes", "encode", "from_lightgbm", "from_sklearn", "from_xgboost", "make",
           "read", "tree_ensemble"]

_TAG = {np.dtype(np.float64): "F64", np.dtype(np.float32): "F32", np.dtype(np.int64): "I64",
        np.dtype(np.int32): "I32", np.dtype(np.uint8): "U8", np.dtype(np.bool_): "BOOL"}
_FROM_TAG = {tag: dtype for dtype, tag in _TAG.items()}

# Missing-value modes of the flags byte (bits 1-2).
MISSING_AS_ZERO, MISSING_DEFAULT, MISSING_ZERO_OR_NAN = 0, 1, 2


def encode(spec: Mapping[str, Any], tensors: Mapping[str, Any]) -> bytes:
    """The bytes of a model file holding ``spec`` and ``tensors``."""
    arrays = {}
    for name, value in tensors.items():
        a = np.asarray(value)
        if a.dtype not in _TAG:
            raise TypeError(f"tensor {name!r}: dtype {a.dtype} cannot be stored")
        arrays[name] = np.ascontiguousarray(a.astype(a.dtype.newbyteorder("<"), copy=False))
    names = sorted(arrays, key=lambda n: (-arrays[n].dtype.itemsize, n))
    header: dict[str, Any] = {}
    at = 0
    for name in names:
        a = arrays[name]
        header[name] = {"dtype": _TAG[a.dtype.newbyteorder("=")], "shape": list(a.shape),
                        "data_offsets": [at, at + a.nbytes]}
        at += a.nbytes
    header["__metadata__"] = {"montlok": json.dumps(spec, separators=(",", ":"), allow_nan=False,
                                                    ensure_ascii=False)}
    text = json.dumps(header, separators=(",", ":"), ensure_ascii=False).encode()
    text += b" " * ((8 - (8 + len(text)) % 8) % 8)
    return struct.pack("<Q", len(text)) + text + b"".join(arrays[n].tobytes() for n in names)


def read(source: str | os.PathLike | bytes) -> tuple[dict, dict[str, np.ndarray]]:
    """``(spec, tensors)`` of a model file (path or bytes); tensors as NumPy arrays."""
    data = bytes(source) if isinstance(source, (bytes, bytearray, memoryview)) else Path(source).read_bytes()
    (length,) = struct.unpack_from("<Q", data, 0)
    header = json.loads(data[8:8 + length])
    meta = header.pop("__metadata__", {})
    if "montlok" not in meta:
        raise ValueError("not a montlok model: __metadata__.montlok is missing")
    start = 8 + length
    tensors = {}
    for name, entry in header.items():
        dtype = np.dtype(_FROM_TAG[entry["dtype"]]).newbyteorder("<")
        lo, hi = entry["data_offsets"]
        flat = np.frombuffer(data, dtype=dtype, count=(hi - lo) // dtype.itemsize, offset=start + lo)
        tensors[name] = flat.reshape(entry["shape"]).astype(dtype.newbyteorder("="))
    return json.loads(meta["montlok"]), tensors


@dataclass
class Exported:
    """A spec and its tensors, ready to write or to open."""

    spec: dict
    tensors: dict = field(default_factory=dict)

    def to_bytes(self) -> bytes:
        return encode(self.spec, self.tensors)

    def save(self, path: str | os.PathLike) -> Path:
        """Writes through a temporary file and a rename, so readers never see half a file."""
        path = Path(path)
        part = path.with_name(path.name + ".tmp")
        part.write_bytes(self.to_bytes())
        os.replace(part, path)
        return path

    def load(self):
        """Opens the model in memory (``montlok.load`` of the bytes)."""
        from . import load

        return load(self.to_bytes())

    def with_metadata(self, **items: Any) -> "Exported":
        spec = dict(self.spec)
        spec["metadata"] = {**spec.get("metadata", {}), **items}
        return Exported(spec, dict(self.tensors))


def _exporter() -> str:
    try:
        from . import __version__
    except ImportError:  # pragma: no cover - module used on its own
        return "montlok unknown"
    return f"montlok {__version__}"


def make(family: str, config: Mapping[str, Any], tensors: Mapping[str, Any], *, features: int, outputs: int,
         sequence: int = 0, preprocess: Mapping[str, Any] | None = None,
         feature_names: Sequence[str] | None = None, output_names: Sequence[str] | None = None,
         metadata: Mapping[str, Any] | None = None) -> Exported:
    """A model of ``family``.  ``preprocess`` may hold ``mean`` and ``scale`` (one
    value per feature) and ``clip=(low, high)``: inputs become
    ``clip((x - mean) / scale)`` in float64 before the family reads them."""
    tensors = dict(tensors)
    spec: dict[str, Any] = {"schema": SCHEMA, "family": family,
                            "inputs": {"features": int(features), "sequence": int(sequence)},
                            "outputs": {"size": int(outputs)}, "config": dict(config)}
    if feature_names is not None:
        names = [str(n) for n in feature_names]
        if len(names) != features:
            raise ValueError(f"{len(names)} feature names for {features} features")
        spec["inputs"]["names"] = names
    if output_names is not None:
        names = [str(n) for n in output_names]
        if len(names) != outputs:
            raise ValueError(f"{len(names)} output names for {outputs} outputs")
        spec["outputs"]["names"] = names
    if preprocess:
        block: dict[str, Any] = {}
        mean, scale = preprocess.get("mean"), preprocess.get("scale")
        if (mean is None) != (scale is None):
            raise ValueError("preprocess needs both mean and scale")
        if mean is not None:
            mean = np.asarray(mean, dtype=np.float64).reshape(-1)
            scale = np.asarray(scale, dtype=np.float64).reshape(-1)
            if mean.shape != (features,) or scale.shape != (features,):
                raise ValueError("preprocess mean/scale need one value per feature")
            if not (np.isfinite(mean).all() and np.isfinite(scale).all() and (scale > 0).all()):
                raise ValueError("preprocess mean must be finite and scale finite and positive")
            tensors["preprocess.mean"], tensors["preprocess.scale"] = mean, scale
            block.update(mean="preprocess.mean", scale="preprocess.scale")
        clip = preprocess.get("clip")
        if clip is not None:
            low, high = (float(v) for v in clip)
            if not low < high:
                raise ValueError("preprocess clip needs low < high")
            block["clip"] = [low, high]
        spec["preprocess"] = block
    spec["metadata"] = {"exporter": _exporter(), **(metadata or {})}
    return Exported(spec, tensors)


# ---------------------------------------------------------------------------
# Tree ensembles
# ---------------------------------------------------------------------------


class Nodes:
    """A growing flat node table (the ``trees.*`` tensors)."""

    def __init__(self) -> None:
        self.feature: list[int] = []
        self.threshold: list[float] = []
        self.left: list[int] = []
        self.right: list[int] = []
        self.value: list[float] = []
        self.flags: list[int] = []

    def add(self, feature: int = -1, threshold: float = 0.0, value: float = 0.0, flags: int = 0) -> int:
        """Appends a node (a leaf when ``feature`` is -1) and returns its index."""
        self.feature.append(int(feature))
        self.threshold.append(float(threshold))
        self.left.append(-1)
        self.right.append(-1)
        self.value.append(float(value))
        self.flags.append(int(flags))
        return len(self.feature) - 1

    def tensors(self, prefix: str = "trees") -> dict[str, np.ndarray]:
        return {f"{prefix}.feature": np.asarray(self.feature, dtype=np.int32),
                f"{prefix}.threshold": np.asarray(self.threshold, dtype=np.float64),
                f"{prefix}.left": np.asarray(self.left, dtype=np.int32),
                f"{prefix}.right": np.asarray(self.right, dtype=np.int32),
                f"{prefix}.value": np.asarray(self.value, dtype=np.float64),
                f"{prefix}.flags": np.asarray(self.flags, dtype=np.uint8)}


_Nodes = Nodes  # the reference's name for the same builder


def tree_ensemble(nodes: Nodes | Mapping[str, Any], roots: Sequence[int], tree_outputs: Sequence[int], *,
                  features: int, outputs: int = 1, decision: str = "le", feature_cast: str = "f64",
                  aggregate: str = "sum", link: str = "identity", base_score: float | Sequence[float] = 0.0,
                  sigmoid_scale: float = 1.0, **kwargs: Any) -> Exported:
    """A ``tree_ensemble`` model.  ``nodes`` is a :class:`Nodes` or a mapping with
    the arrays feature/threshold/left/right/value/flags."""
    if isinstance(nodes, Nodes):
        tensors = nodes.tensors()
    else:
        kinds = {"feature": np.int32, "threshold": np.float64, "left": np.int32, "right": np.int32,
                 "value": np.float64, "flags": np.uint8}
        tensors = {f"trees.{k}": np.asarray(nodes[k], dtype=t) for k, t in kinds.items()}
    tensors["trees.root"] = np.asarray(roots, dtype=np.int32)
    tensors["trees.output"] = np.asarray(tree_outputs, dtype=np.int32)
    if np.ndim(base_score) == 0:
        base = [float(base_score)] * outputs
    else:
        base = [float(v) for v in base_score]
    config = {"decision": decision, "feature_cast": feature_cast, "aggregate": aggregate, "link": link,
              "base_score": base, "sigmoid_scale": float(sigmoid_scale)}
    return make("tree_ensemble", config, tensors, features=features, outputs=outputs, **kwargs)


def _lightgbm_dump(model: Any) -> dict:
    if isinstance(model, Mapping):
        return dict(model)
    if isinstance(model, (str, bytes)):
        return json.loads(model)
    booster = getattr(model, "booster_", model)
    if hasattr(booster, "dump_model"):
        return booster.dump_model()
    raise TypeError("expected a LightGBM Booster/LGBMModel, its dump_model() dict, or that dict as JSON")


_LGB_MISSING = {"None": MISSING_AS_ZERO, "NaN": MISSING_DEFAULT, "Zero": MISSING_ZERO_OR_NAN}


def _append_dump_tree(nodes: Nodes, root: Any, split_of, leaf_of) -> None:
    """Numbers one dumped tree into ``nodes`` in pre-order, left subtree first.

    ``split_of(node)`` returns None for a leaf, else (feature, threshold, flags,
    left child, right child); ``leaf_of(node)`` returns a leaf's value."""
    stack = [(root, -1, False)]
    while stack:
        node, parent, is_right = stack.pop()
        split = split_of(node)
        if split is None:
            index = nodes.add(value=leaf_of(node))
        else:
            feature, threshold, flags, left, right = split
            index = nodes.add(feature=feature, threshold=threshold, flags=flags)
            stack.append((right, index, True))
            stack.append((left, index, False))
        if parent >= 0:
            (nodes.right if is_right else nodes.left)[parent] = index


def from_lightgbm(model: Any, *, feature_names: Sequence[str] | None = None,
                  metadata: Mapping[str, Any] | None = None) -> Exported:
    """A LightGBM model with numerical splits (dump_model() dict, its JSON, or a
    Booster).  Binary and multiclass objectives predict probabilities."""
    dump = _lightgbm_dump(model)
    if dump.get("is_linear"):
        raise ValueError("linear trees are not supported")
    features = int(dump["max_feature_idx"]) + 1
    per_round = int(dump.get("num_tree_per_iteration", 1))
    objective = str(dump.get("objective", "regression"))
    link, scale = _lightgbm_link(objective)

    def split_of(node):
        if "split_feature" not in node:
            if "leaf_coeff" in node:
                raise ValueError("linear trees are not supported")
            return None
        if node.get("decision_type", "<=") != "<=":
            raise ValueError("categorical LightGBM splits are not supported")
        flags = (1 if node.get("default_left", True) else 0) | (_LGB_MISSING[node.get("missing_type", "None")] << 1)
        return node["split_feature"], float(node["threshold"]), flags, node["left_child"], node["right_child"]

    nodes = Nodes()
    roots, tree_outputs = [], []
    for t, info in enumerate(dump["tree_info"]):
        roots.append(len(nodes.feature))
        tree_outputs.append(t % per_round)
        _append_dump_tree(nodes, info["tree_structure"], split_of, lambda n: float(n["leaf_value"]))
    names = feature_names if feature_names is not None else dump.get("feature_names")
    return tree_ensemble(nodes, roots, tree_outputs, features=features, outputs=per_round, link=link,
                         sigmoid_scale=scale, aggregate="mean" if dump.get("average_output") else "sum",
                         feature_names=names,
                         metadata={"source": "lightgbm", "objective": " ".join(objective.split()), **(metadata or {})})


# The link LightGBM's predict() applies to the raw sum, by objective family
# (the first word of the dump's "objective"; "sigmoid:<k>" scales the
# logistic). One-vs-all multiclass has a per-class sigmoid: not representable.
_LGB_LINKS = {"binary": "sigmoid", "cross_entropy": "sigmoid", "xentropy": "sigmoid", "multiclass": "softmax",
              "softmax": "softmax", "poisson": "exp", "gamma": "exp", "tweedie": "exp"}
_LGB_ONE_VS_ALL = {"multiclassova", "multiclass_ova", "ova", "ovr"}


def _lightgbm_link(objective: str) -> tuple[str, float]:
    family, *options = objective.split() or ["regression"]
    if family in _LGB_ONE_VS_ALL:
        raise ValueError("one-vs-all multiclass objectives are not supported")
    link = _LGB_LINKS.get(family, "identity")
    settings = {key: value for key, sep, value in (o.partition(":") for o in options) if sep}
    return link, float(settings.get("sigmoid", 1.0)) if link == "sigmoid" else 1.0


# XGBoost objectives whose prediction is not the raw margin: the link on the
# summed margin, and how base_score (a prediction) turns into a margin.
_XGB_OBJECTIVES = {
    "binary:logistic": ("sigmoid", lambda p: math.log(p / (1.0 - p))),
    "reg:logistic": ("sigmoid", lambda p: math.log(p / (1.0 - p))),
    "count:poisson": ("exp", math.log),
    "reg:gamma": ("exp", math.log),
    "reg:tweedie": ("exp", math.log),
    "survival:cox": ("exp", math.log),
}


def _xgboost_link(objective: str) -> tuple[str, Any]:
    if objective in _XGB_OBJECTIVES:
        return _XGB_OBJECTIVES[objective]
    return ("softmax" if objective.startswith("multi:") else "identity"), float


def from_xgboost(model: Any, *, features: int | None = None, objective: str | None = None,
                 base_score: float | None = None, base_margin: float | None = None, classes: int | None = None,
                 parallel_trees: int = 1, feature_names: Sequence[str] | None = None,
                 metadata: Mapping[str, Any] | None = None) -> Exported:
    """An XGBoost gbtree model: a Booster, or its JSON tree dumps with
    ``features``, ``objective`` and ``base_score`` (or ``base_margin``).
    Splits are ``x < split_condition`` on float32 features; thresholds are
    stored as float32 values, as XGBoost keeps them."""
    if hasattr(model, "get_booster"):
        model = model.get_booster()
    if hasattr(model, "get_dump"):
        learner = json.loads(model.save_config())["learner"]
        objective = objective or learner["objective"]["name"]
        params = learner["learner_model_param"]
        if base_score is None:
            base_score = float(str(params["base_score"]).strip("[]"))
        features = features or int(params["num_feature"])
        classes = classes or int(params.get("num_class", 0))
        tree_params = learner.get("gradient_booster", {}).get("gbtree_model_param", {})
        parallel_trees = int(tree_params.get("num_parallel_tree", parallel_trees))
        feature_names = feature_names or model.feature_names
        dumps = model.get_dump(dump_format="json")
    else:
        dumps = list(model)
    if features is None or objective is None or (base_score is None and base_margin is None):
        raise ValueError("tree dumps need features=, objective= and base_score= or base_margin=")
    link, to_margin = _xgboost_link(objective)
    margin = base_margin if base_margin is not None else to_margin(float(base_score))
    outputs = classes if classes and classes > 1 else 1
    by_name = {str(n): i for i, n in enumerate(feature_names)} if feature_names else {}

    def feature_index(split: str) -> int:
        if split in by_name:
            return by_name[split]
        match = re.fullmatch(r"f(\d+)", split)
        if not match:
            raise ValueError(f"unknown feature {split!r}; pass feature_names=")
        return int(match.group(1))

    def split_of(node):
        if "children" not in node:
            return None
        kids = {child["nodeid"]: child for child in node["children"]}
        flags = (1 if node["missing"] == node["yes"] else 0) | (MISSING_DEFAULT << 1)
        return (feature_index(str(node["split"])), float(np.float32(node["split_condition"])), flags,
                kids[node["yes"]], kids[node["no"]])

    nodes = Nodes()
    roots, tree_outputs = [], []
    for t, dumped in enumerate(dumps):
        tree = json.loads(dumped) if isinstance(dumped, (str, bytes)) else dumped
        roots.append(len(nodes.feature))
        tree_outputs.append((t // parallel_trees) % outputs)
        _append_dump_tree(nodes, tree, split_of, lambda n: float(n["leaf"]))
    return tree_ensemble(nodes, roots, tree_outputs, features=int(features), outputs=outputs, decision="lt",
                         feature_cast="f32", link=link, base_score=margin, feature_names=feature_names,
                         metadata={"source": "xgboost", "objective": objective, **(metadata or {})})


def _sklearn_tree(nodes: Nodes, tree: Any, scale: float = 1.0) -> int:
    """Appends a fitted sklearn ``Tree`` (NaN goes where it was trained to, left
    when the tree never saw one); returns its root index."""
    if tree.n_outputs != 1:
        raise ValueError("multi-output trees are not supported")
    base = len(nodes.feature)
    nan_left = getattr(tree, "missing_go_to_left", None)
    values = tree.value[:, 0, 0]
    for i in range(tree.node_count):
        if tree.children_left[i] == -1:
            nodes.add(value=scale * values[i] if scale != 1.0 else values[i])
        else:
            default_left = int(nan_left[i]) if nan_left is not None else 1
            j = nodes.add(feature=tree.feature[i], threshold=tree.threshold[i],
                          flags=default_left | (MISSING_DEFAULT << 1))
            nodes.left[j] = base + int(tree.children_left[i])
            nodes.right[j] = base + int(tree.children_right[i])
    return base


def _hist_predictor(nodes: Nodes, predictor: Any) -> int:
    table = predictor.nodes
    if table["is_categorical"].any():
        raise ValueError("categorical HistGradientBoosting splits are not supported")
    base = len(nodes.feature)
    for row in table:
        if row["is_leaf"]:
            nodes.add(value=float(row["value"]))
        else:
            j = nodes.add(feature=int(row["feature_idx"]), threshold=float(row["num_threshold"]),
                          flags=int(row["missing_go_to_left"]) | (MISSING_DEFAULT << 1))
            nodes.left[j] = base + int(row["left"])
            nodes.right[j] = base + int(row["right"])
    return base


def from_sklearn(estimator: Any, *, feature_names: Sequence[str] | None = None,
                 metadata: Mapping[str, Any] | None = None) -> Exported:
    """A fitted scikit-learn tree model: DecisionTree/ExtraTree, RandomForest/
    ExtraTrees, GradientBoosting or HistGradientBoosting regressors (optionally
    behind a StandardScaler in a Pipeline, which becomes the float64
    preprocess).  Other estimator kinds belong to families this build does not
    run on the GPU."""
    preprocess = None
    if type(estimator).__name__ == "Pipeline":
        steps = [s for _, s in estimator.steps if s not in (None, "passthrough")]
        if len(steps) == 2 and type(steps[0]).__name__ == "StandardScaler":
            scaler = steps[0]
            n = scaler.n_features_in_
            preprocess = {"mean": scaler.mean_ if scaler.with_mean else np.zeros(n),
                          "scale": scaler.scale_ if scaler.with_std else np.ones(n)}
            estimator = steps[1]
        elif len(steps) != 1:
            raise TypeError("only Pipeline([StandardScaler, model]) or a single estimator are supported")
        else:
            estimator = steps[0]
    name = type(estimator).__name__
    features = int(estimator.n_features_in_)
    if feature_names is None and hasattr(estimator, "feature_names_in_"):
        feature_names = [str(f) for f in estimator.feature_names_in_]
    common = dict(feature_names=feature_names, preprocess=preprocess,
                  metadata={"source": f"sklearn.{name}", **(metadata or {})})
    nodes = Nodes()
    if name in ("DecisionTreeRegressor", "ExtraTreeRegressor"):
        root = _sklearn_tree(nodes, estimator.tree_)
        return tree_ensemble(nodes, [root], [0], features=features, feature_cast="f32", **common)
    if name in ("RandomForestRegressor", "ExtraTreesRegressor"):
        roots = [_sklearn_tree(nodes, est.tree_) for est in estimator.estimators_]
        return tree_ensemble(nodes, roots, [0] * len(roots), features=features, feature_cast="f32",
                             aggregate="mean", **common)
    if name == "GradientBoostingRegressor":
        init = estimator.init_
        if isinstance(init, str) and init == "zero":
            base = 0.0
        elif type(init).__name__ == "DummyRegressor":
            base = float(np.asarray(init.constant_).reshape(-1)[0])
        else:
            raise TypeError("GradientBoostingRegressor with a non-constant init estimator is not supported")
        rate = float(estimator.learning_rate)
        roots = [_sklearn_tree(nodes, stage[0].tree_, scale=rate) for stage in estimator.estimators_]
        return tree_ensemble(nodes, roots, [0] * len(roots), features=features, feature_cast="f32",
                             base_score=base, **common)
    if name == "HistGradientBoostingRegressor":
        loss = getattr(estimator, "loss", "squared_error")
        roots = [_hist_predictor(nodes, p[0]) for p in estimator._predictors]
        base = float(np.asarray(estimator._baseline_prediction).reshape(-1)[0])
        return tree_ensemble(nodes, roots, [0] * len(roots), features=features, base_score=base,
                             link="exp" if loss in ("poisson", "gamma") else "identity", **common)
    raise TypeError(f"cannot export {name}: only tree models run on this build")
