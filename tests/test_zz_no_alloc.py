"""montlok_model_predict_device_noalloc, the entry point that allocates nothing.

It is for callers that cannot allocate GPU memory while they predict: serving
loops whose device memory belongs to another allocator (a framework's caching
pool that has already reserved the GPU), and latency-critical paths that must
not pay for cudaMalloc/cudaFree or the device-wide synchronisation cudaFree
implies. Its scratch is a fixed 16 MiB device array inside the library.

These tests call it through the C ABI and compare it bit for bit with
montlok_model_predict_device and with the CPU oracle, on two calls in a row
(the second call finds the array holding the first call's tables). The file sorts last,
so a run that stops at its first failure has run every other test; it also
passes alone in a fresh process, because each test first makes its model
resident with the regular entry point.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import montlok
from forests import edge_inputs, random_model, same_bits
from montlok import _core, export, synth
from oracle import Oracle

pytestmark = pytest.mark.gpu

lib = _core.lib
lib.montlok_model_predict_device_noalloc.restype = ctypes.c_int
lib.montlok_model_predict_device_noalloc.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
                                                     ctypes.c_void_p, ctypes.c_void_p]


def noalloc(model, x_ptr: int, batch: int, out_ptr: int) -> int:
    return lib.montlok_model_predict_device_noalloc(model._h, _core.FLOAT64, x_ptr, batch, out_ptr, None)


def case(i: int):
    rng = np.random.default_rng(77 + i)
    if i == 0:  # wide: key tables past shared memory, the generic kernel on the static array
        return random_model(rng, features=1200, trees=300, max_depth=10), edge_inputs(rng, 700, 1200, 0.3)
    if i == 1:  # the benchmark recipe, small: the complete-tree kernel
        return synth.model_c2(trees=96).to_bytes(), synth.inputs_c2(batch=5000)
    if i == 2:  # 12 outputs: the generic kernel, key tables in shared memory
        return random_model(rng, features=7, trees=150, outputs=12, link="softmax"), edge_inputs(rng, 999, 7)
    if i == 3:  # 5 classes: the multi-output kernel
        return synth.model_c4(rounds=20).to_bytes(), synth.inputs_c4(batch=3000)
    # one output, depth 14: the deep-tree kernel
    return random_model(rng, features=6, trees=100, max_depth=14), edge_inputs(rng, 2000, 6, 0.3)


@pytest.mark.parametrize("i", range(5))
def test_matches_predict_device_on_two_calls(gpu, i):
    torch = pytest.importorskip("torch")
    model_bytes, x = case(i)
    m = montlok.load(model_bytes)
    n = len(x)
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    want = torch.empty((n, m.outputs), dtype=torch.float64, device="cuda")
    m.predict_device(xd.data_ptr(), n, want.data_ptr(), _core.FLOAT64, 0)
    torch.cuda.synchronize()
    oracle = Oracle(model_bytes).predict(x)
    assert same_bits(want.cpu().numpy(), oracle)
    for _ in range(2):
        got = torch.full((n, m.outputs), float("nan"), dtype=torch.float64, device="cuda")
        status = noalloc(m, xd.data_ptr(), n, got.data_ptr())
        assert status == 0, lib.montlok_last_error()
        torch.cuda.synchronize()
        assert same_bits(got.cpu().numpy(), want.cpu().numpy())
        assert same_bits(got.cpu().numpy(), oracle)


def test_needs_a_resident_model(gpu):
    torch = pytest.importorskip("torch")
    m = montlok.load(random_model(np.random.default_rng(5), features=4, trees=10))
    x = torch.zeros((8, 4), dtype=torch.float64, device="cuda")
    out = torch.zeros((8, 1), dtype=torch.float64, device="cuda")
    assert noalloc(m, x.data_ptr(), 8, out.data_ptr()) == 6
    assert b"resident" in lib.montlok_last_error()


def test_rejects_models_beyond_the_scratch(gpu):
    torch = pytest.importorskip("torch")
    # A chain of splits reading 65601 features with both NaN directions:
    # 131202 slots, one 32-row key table of 16.8 MB > 16 MiB. Rejected before
    # any kernel runs (the model is made resident without predicting).
    features = 65601
    nodes = export.Nodes()
    root = prev = -1
    for i in range(2 * features):
        split = nodes.add(feature=i % features, threshold=0.0, flags=(i // features) | (1 << 1))
        nodes.left[split] = nodes.add(value=1.0)
        if prev >= 0:
            nodes.right[prev] = split
        else:
            root = split
        prev = split
    nodes.right[prev] = nodes.add(value=2.0)
    m = montlok.load(export.tree_ensemble(nodes, [root], [0], features=features).to_bytes())
    assert m.kernel(1) == "generic-global-keys"
    x = torch.zeros((1, features), dtype=torch.float64, device="cuda")
    out = torch.zeros((1, 1), dtype=torch.float64, device="cuda")
    assert noalloc(m, x.data_ptr(), 1, out.data_ptr()) == 4
    assert b"no-allocation" in lib.montlok_last_error()
