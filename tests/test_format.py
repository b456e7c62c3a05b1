"""Loading and validation through the C ABI (no GPU needed): damaged files,
invalid specs and invalid trees are clean errors with the reference's
statuses (src/core/archive.cpp:105-188, runtime.cpp:443-520, trees.cpp:70-156),
and input validation happens before any device work."""

from __future__ import annotations

import struct

import numpy as np
import pytest

import montlok
from montlok import export


def tiny() -> export.Exported:
    nodes = export.Nodes()
    root = nodes.add(feature=0, threshold=0.5, flags=1 | (1 << 1))
    nodes.left[root] = nodes.add(value=1.0)
    right = nodes.add(feature=2, threshold=-1.0, flags=2 << 1)
    nodes.right[root] = right
    nodes.left[right] = nodes.add(value=2.0)
    nodes.right[right] = nodes.add(value=3.0)
    return export.tree_ensemble(nodes, [root, right], [0, 1], features=3, outputs=2, link="softmax",
                                base_score=[0.1, 0.2], feature_names=["a", "b", "c"],
                                preprocess={"mean": [1.0, 2.0, 3.0], "scale": [2.0, 4.0, 8.0], "clip": (-3, 3)},
                                metadata={"release": "unit"})


def reencode(data: bytes, mutate) -> bytes:
    spec, tensors = export.read(data)
    mutate(spec, tensors)
    return export.encode(spec, tensors)


def test_round_trip_and_spec():
    e = tiny()
    model = montlok.load(e.to_bytes())
    assert (model.family, model.features, model.sequence, model.outputs, model.trees) == ("tree_ensemble", 3, 0, 2, 2)
    assert model.preprocess and model.streamable
    assert model.spec["inputs"]["names"] == ["a", "b", "c"]
    assert model.spec["metadata"]["release"] == "unit"


def test_path_bytes_and_file_object(tmp_path):
    path = tiny().save(tmp_path / "m.montlok")
    for source in (path, str(path), path.read_bytes()):
        assert montlok.load(source).features == 3
    with path.open("rb") as handle:
        assert montlok.load(handle).outputs == 2


def test_missing_file():
    with pytest.raises(OSError):
        montlok.load("/nonexistent/model.montlok")


@pytest.mark.parametrize("mutate, error", [
    (lambda s, t: s.update(schema="montlok.model/9"), NotImplementedError),
    (lambda s, t: s.update(family="sequential"), NotImplementedError),
    (lambda s, t: s.update(family="no_such_family"), NotImplementedError),
    (lambda s, t: s.pop("family"), ValueError),
    (lambda s, t: s["inputs"].update(features=0), ValueError),
    (lambda s, t: s["inputs"].update(features=2), ValueError),       # a split reads feature 2
    (lambda s, t: s["inputs"].update(sequence=4), ValueError),
    (lambda s, t: s["outputs"].update(size=1), ValueError),          # softmax needs two; tree 1 adds to output 1
    (lambda s, t: s["preprocess"].update(clip=[3, -3]), ValueError),
    (lambda s, t: s["preprocess"].update(mean=None), ValueError),
    (lambda s, t: s["inputs"].update(names=["a"]), ValueError),
    (lambda s, t: s["config"].update(decision="ge"), ValueError),
    (lambda s, t: s["config"].update(feature_cast="f16"), ValueError),
    (lambda s, t: s["config"].update(aggregate="max"), ValueError),
    (lambda s, t: s["config"].update(link="tanh"), NotImplementedError),
    (lambda s, t: s["config"].update(base_score=[1.0]), ValueError),
    (lambda s, t: s["config"].update(tensors="nope"), ValueError),
    (lambda s, t: t.__setitem__("trees.threshold", np.array([np.nan, 0, -1.0, 0, 0])), ValueError),
    (lambda s, t: t.__setitem__("trees.flags", np.array([7, 0, 4, 0, 0], dtype=np.uint8)), ValueError),
    (lambda s, t: t.__setitem__("trees.left", np.array([0, -1, 3, -1, -1], dtype=np.int32)), ValueError),
    (lambda s, t: t.__setitem__("trees.right", np.array([9, -1, 4, -1, -1], dtype=np.int32)), ValueError),
    (lambda s, t: t.__setitem__("trees.value", np.array([0, np.inf, 0, 2, 3])), ValueError),
    (lambda s, t: t.__setitem__("trees.root", np.array([0, 7], dtype=np.int32)), ValueError),
    (lambda s, t: t.__setitem__("trees.output", np.array([0, 2], dtype=np.int32)), ValueError),
    (lambda s, t: t.__setitem__("trees.output", np.array([0], dtype=np.int32)), ValueError),
    (lambda s, t: t.__setitem__("trees.root", np.zeros(0, dtype=np.int32)), ValueError),
    (lambda s, t: t.__setitem__("trees.feature", np.array([0, -1, 2, -1], dtype=np.int32)), ValueError),
    (lambda s, t: t.__setitem__("trees.threshold", np.array([0.5, 0, -1.0, 0, 0], dtype=np.int32)), ValueError),
    (lambda s, t: t.__setitem__("preprocess.scale", np.array([1.0, 0.0, 1.0])), ValueError),
])
def test_invalid_specs_and_trees_are_rejected(mutate, error):
    with pytest.raises(error):
        montlok.load(reencode(tiny().to_bytes(), mutate))


def test_wide_integer_tensors_are_accepted_and_range_checked():
    ok = reencode(tiny().to_bytes(), lambda s, t: t.__setitem__("trees.left", t["trees.left"].astype(np.int64)))
    assert montlok.load(ok).trees == 2
    bad = reencode(tiny().to_bytes(),
                   lambda s, t: t.__setitem__("trees.left", np.array([1 << 40, -1, 3, -1, -1], dtype=np.int64)))
    with pytest.raises(ValueError):
        montlok.load(bad)


@pytest.mark.parametrize("data", [
    b"",
    b"\x01",
    struct.pack("<Q", 1 << 40) + b"{}",
    struct.pack("<Q", 2) + b"{}",
    struct.pack("<Q", 2) + b"[]",
    struct.pack("<Q", 5) + b'{"a":',
    struct.pack("<Q", 47) + b'{"t":{"dtype":"F64","shape":[2],"data_offsets":[0,16]}}',
    struct.pack("<Q", 56) + b'{"__metadata__":{"montlok":"{\\"schema\\":1}"},"x":1,"y":2}',
    struct.pack("<Q", 11) + b'{"a":1,"a":2}',
])
def test_garbage_is_a_clean_error(data):
    with pytest.raises((ValueError, NotImplementedError)):
        montlok.load(data)


def test_random_corruption_is_a_clean_error():
    data = bytearray(tiny().to_bytes())
    rng = np.random.default_rng(1)
    for _ in range(600):
        mutated = bytearray(data)
        for at in rng.integers(0, len(mutated), size=rng.integers(1, 4)):
            mutated[at] = int(rng.integers(0, 256))
        try:
            montlok.load(bytes(mutated))
        except (ValueError, NotImplementedError, OSError, RuntimeError):
            pass
    for cut in range(0, len(data), 7):
        with pytest.raises((ValueError, NotImplementedError)):
            montlok.load(bytes(data[:cut]))


def test_input_validation_before_device_work():
    model = tiny().load()
    with pytest.raises(ValueError):
        model.predict(np.zeros((2, 4)))
    with pytest.raises(ValueError):
        model.predict(np.zeros((2, 3, 1)))
    with pytest.raises(TypeError):
        model.predict(np.zeros((2, 3)), out=[0.0] * 4)
    with pytest.raises(ValueError):
        model.predict(np.zeros((2, 3)), out=np.zeros(3))
    with pytest.raises(ValueError):
        model.predict(np.zeros((2, 3)), out=np.zeros(4, dtype=np.float32))
    assert model.predict(np.zeros((0, 3))).shape == (0, 2)
    with pytest.raises(ValueError):
        model.stream(0)


def test_no_cpu_fallback_without_a_gpu():
    if montlok.device_count() > 0:
        pytest.skip("a GPU is visible")
    model = tiny().load()
    with pytest.raises(RuntimeError, match="CUDA"):
        model.predict(np.zeros((4, 3)))


# JSON edge cases placed inside a model spec (as the value of a metadata
# field), so the spec parser meets them; each must be accepted or rejected
# exactly as the reference runtime (compiled from its sources) does.
JSON_EDGES = [
    "1", "-0", "0.5e1", "1E+2", "1e-2", "123456789012345678901234567890", "1e308", "1e309", "-1e309", "1e-400",
    "01", "1.", ".5", "1e", "-", "+1", "0x10", "NaN", "Infinity",
    '"plain"', '"\\u00e9\\u4e2d"', '"\\ud83d\\ude00"', '"\\ud800"', '"\\udc00"', '"\\ud800x"', '"\\ud800\\u0041"',
    '"tab\\there"', '"\\x41"', '"\\U0041"', '"raw\x01control"', '"raw\x7fdel"', '"\xc3\xa9"',
    "true", "false", "null", "True", "nul", "[]", "{}", "[1,2,]", "[,1]", "[1 2]", '{"a":1,}', '{"a" 1}',
    '{"a":1,"a":2}', '{"a":{"b":1,"b":2}}', '{"":1}', '[[[[]]]]', "\f1", " 1 ", "[1]]", "{1:2}",
    "[" * 126 + "]" * 126, "[" * 127 + "]" * 127, "[" * 128 + "]" * 128, "[" * 127 + "1" + "]" * 127,
    "[" * 126 + "1" + "]" * 126, "[" * 400 + "]" * 400,
]


def spec_with_edge(text: str) -> bytes:
    import json as _json

    data = tiny().to_bytes()
    n = struct.unpack("<Q", data[:8])[0]
    header = _json.loads(data[8:8 + n])
    spec_text = header["__metadata__"]["montlok"]
    assert spec_text.endswith("}")
    edited = spec_text[:-1] + ',"x-edge":' + text + "}"
    header["__metadata__"]["montlok"] = edited
    raw = _json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * (-len(raw) % 8)
    return struct.pack("<Q", len(raw)) + raw + data[8 + n:]


@pytest.mark.parametrize("edge", JSON_EDGES, ids=range(len(JSON_EDGES)))
def test_spec_json_is_read_like_the_reference(edge):
    import oracle

    if not oracle.available_reference():
        pytest.skip("the reference library (oracle/_ref) was not built here")
    model = spec_with_edge(edge)
    try:
        oracle.Reference().close(oracle.Reference().open(model))
        reference_accepts = True
    except ValueError:
        reference_accepts = False
    try:
        montlok.load(model)
        ours = True
    except (ValueError, NotImplementedError):
        ours = False
    assert ours == reference_accepts
