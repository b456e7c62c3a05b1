"""Parity of the CUDA path with the CPU oracle, through the C ABI.

Every case compares, bit for bit, the predictions and the leaf index of every
(row, tree) that libmontlok.so computes on the GPU with the oracle's (the
plain-C restatement of the reference, itself pinned to the reference in
test_oracle.py): the five benchmark recipes at test sizes, random ensembles
over every missing-value mode with inputs on the split rules, every link,
mean aggregation, float32 inputs, preprocess, multi-pass outputs, the
global-memory key path, shared nodes and infinite thresholds.
"""

from __future__ import annotations

import os
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import montlok
from forests import GRID, NARROWING, edge_inputs, random_model, same_bits
from montlok import export, synth
from oracle import Oracle

pytestmark = pytest.mark.gpu


def check(model: bytes, x: np.ndarray, leaves: bool = True) -> None:
    m = montlok.load(model)
    o = Oracle(model)
    got = m.predict(x)
    want = o.predict(x)
    assert same_bits(got.reshape(want.shape), want), "predictions differ from the oracle"
    if leaves:
        np.testing.assert_array_equal(m.predict_leaves(x).reshape(len(want), -1), o.leaves(x))


RECIPES = {
    "c1": (lambda: synth.model_c1().to_bytes(), lambda: synth.inputs_c1(batch=2000)),
    "c2": (lambda: synth.model_c2(trees=120).to_bytes(), lambda: synth.inputs_c2(batch=3000)),
    "c3": (lambda: synth.model_c3(trees=6, samples=20_000).to_bytes(), lambda: synth.inputs_c3(batch=1500)),
    "c4": (lambda: synth.model_c4(rounds=14).to_bytes(), lambda: synth.inputs_c4(batch=1500)),
    "c5": (lambda: synth.model_c5(trees=150).to_bytes(), lambda: synth.inputs_c5(batch=64)),
}


@pytest.mark.parametrize("name", sorted(RECIPES))
def test_benchmark_recipes(gpu, name):
    make_model, make_x = RECIPES[name]
    check(make_model(), make_x())


@pytest.mark.parametrize("decision", ["le", "lt"])
@pytest.mark.parametrize("cast", ["f64", "f32"])
@pytest.mark.parametrize("inf", [0.0, 0.15])
def test_edge_values_every_missing_mode(gpu, decision, cast, inf):
    rng = np.random.default_rng([len(decision), len(cast), int(inf * 100)])
    model = random_model(rng, features=7, decision=decision, cast=cast, trees=150, inf_thresholds=inf)
    check(model, edge_inputs(rng, 700, 7))


@pytest.mark.parametrize("link, outputs, aggregate", [
    ("sigmoid", 1, "sum"), ("exp", 1, "sum"), ("softmax", 3, "sum"), ("softmax", 12, "sum"),
    ("identity", 5, "mean"), ("exp", 4, "mean"), ("identity", 11, "sum"), ("sigmoid", 9, "mean"),
])
def test_links_outputs_and_aggregates(gpu, link, outputs, aggregate):
    rng = np.random.default_rng(outputs * 7 + len(link))
    model = random_model(rng, features=6, trees=200, outputs=outputs, link=link, aggregate=aggregate,
                         base=list(rng.normal(size=outputs)), sigmoid_scale=0.7)
    check(model, edge_inputs(rng, 400, 6, special=0.2))


@pytest.mark.parametrize("outputs", [2, 5, 8])
@pytest.mark.parametrize("cast, decision", [("f64", "le"), ("f32", "lt")])
def test_multi_output_kernel(gpu, outputs, cast, decision):
    """2..8 outputs take the per-output team kernel. Outputs are assigned to
    trees at random, so some 64-tree blocks hold no tree of an output (whose
    sum then adds a 0.0 partial, turning -0.0 into +0.0 as the reference
    does); every missing mode, infinite thresholds, deep trees."""
    rng = np.random.default_rng([outputs, len(cast), len(decision)])
    trees = 300
    tree_outputs = list(rng.integers(0, outputs, size=trees))
    tree_outputs[:outputs] = range(outputs)
    for link, aggregate in (("softmax", "sum"), ("identity", "mean")):
        model = random_model(rng, features=9, trees=trees, outputs=outputs, link=link, aggregate=aggregate,
                             decision=decision, cast=cast, max_depth=12, inf_thresholds=0.05,
                             base=list(rng.normal(size=outputs)), tree_outputs=tree_outputs)
        check(model, edge_inputs(rng, 700, 9, special=0.3))
    # An output whose trees all sit in block 0, followed by blocks without it.
    tree_outputs = [0] * 10 + [1] * 150
    model = random_model(rng, features=5, trees=160, outputs=2, base=[-0.0, 0.5], tree_outputs=tree_outputs)
    check(model, edge_inputs(rng, 300, 5))


@pytest.mark.parametrize("cast, decision", [("f64", "le"), ("f32", "lt"), ("f32", "le")])
@pytest.mark.parametrize("inf", [0.0, 0.1])
def test_deep_tree_kernel(gpu, cast, decision, inf):
    """One output, trees deeper than 8 levels: the deep-tree kernel (node
    array in L2, 8 trees per lane, leaf words naming their values), every
    missing mode, infinite thresholds, mean and sum, float32 inputs."""
    rng = np.random.default_rng([len(cast), len(decision), int(inf * 10)])
    for aggregate, link in (("sum", "sigmoid"), ("mean", "identity")):
        model = random_model(rng, features=8, trees=150, max_depth=16, cast=cast, decision=decision,
                             inf_thresholds=inf, aggregate=aggregate, link=link, base=0.3)
        x = edge_inputs(rng, 900, 8, special=0.3)
        check(model, x)
        assert same_bits(montlok.load(model).predict(x.astype(np.float32)).reshape(-1, 1),
                         Oracle(model).predict(x.astype(np.float32)))


@pytest.mark.parametrize("cast", ["f64", "f32"])
def test_preprocess_then_cast(gpu, cast):
    rng = np.random.default_rng(5)
    pre = {"mean": rng.normal(size=6) * 3, "scale": rng.uniform(0.5, 2.0, 6), "clip": (-1.2, 1.7)}
    model = random_model(rng, features=6, cast=cast, trees=90, preprocess=pre)
    x = edge_inputs(rng, 500, 6) * 2 + pre["mean"]
    check(model, x)


def test_float32_inputs(gpu):
    rng = np.random.default_rng(11)
    for cast in ("f64", "f32"):
        model = random_model(rng, features=9, cast=cast, trees=80)
        check(model, edge_inputs(rng, 600, 9).astype(np.float32))


@pytest.mark.parametrize("rows", [1, 2, 31, 32, 33, 63, 65, 4099])
def test_ragged_batches(gpu, rows):
    rng = np.random.default_rng(rows)
    model = random_model(rng, features=4, trees=70)
    check(model, edge_inputs(rng, rows, 4))


SMALL_MODELS = {
    # complete depth-8 trees, float32 leaves, preprocess: the latency recipe
    "c5": lambda: synth.model_c5(trees=1000).to_bytes(),
    # float64 features (ties decided on the doubles), every missing mode, 70 trees: a partial last block
    "f64_edges": lambda: random_model(np.random.default_rng(31), features=7, trees=70, inf_thresholds=0.1),
    # float32 features, `lt`, 33 trees: the second CTA of the only block has one tree
    "f32_lt_33": lambda: random_model(np.random.default_rng(32), features=6, trees=33, decision="lt", cast="f32"),
    # mean of 130 trees, float64 leaves
    "mean_130": lambda: random_model(np.random.default_rng(33), features=5, trees=130, aggregate="mean", base=0.5),
    # fewer trees than a CTA takes
    "tiny_5": lambda: random_model(np.random.default_rng(34), features=4, trees=5, link="sigmoid"),
}


@pytest.mark.parametrize("name", sorted(SMALL_MODELS))
@pytest.mark.parametrize("rows", [1, 3, 4, 5, 8, 9, 31, 33, 64])
def test_small_batches_tree_parallel(gpu, name, rows):
    """Batches of at most 64 rows on complete-tree models take the
    tree-parallel kernel (one CTA per 64-tree block and group of 8 rows, each
    thread one tree for two rows, block sums in tree order, the link by the
    last CTA of each row group); partial groups and partial blocks."""
    model = SMALL_MODELS[name]()
    m = montlok.load(model)
    rng = np.random.default_rng(rows)
    x = synth.inputs_c5(batch=rows) if name == "c5" else edge_inputs(rng, rows, m.features, 0.2)
    check(model, x, leaves=rows <= 8)
    x32 = np.ascontiguousarray(x, dtype=np.float32)
    assert same_bits(m.predict(x32).reshape(rows, -1), Oracle(model).predict(x32))
    # The same rows twice in a row: the per-launch counters start from zero again.
    assert same_bits(m.predict(x).reshape(rows, -1), Oracle(model).predict(x))


def test_small_calls_from_pinned_and_pageable_inputs(gpu):
    """Small host-buffer calls replay a cached graph whose input copy reads
    the caller's buffer in place when it is pinned: alternate pinned and
    pageable inputs of the same shape and check every call's bits."""
    torch = pytest.importorskip("torch")
    model = synth.model_c2(trees=130).to_bytes()
    m, o = montlok.load(model), Oracle(model)
    for rows in (1, 64, 3000):
        xs = [synth.inputs_c2(batch=rows + k)[k:] for k in range(3)]
        pinned = [torch.from_numpy(np.ascontiguousarray(x)).pin_memory() for x in xs]
        for x, xp in zip(xs, pinned):
            want = o.predict(x)
            assert same_bits(m.predict(x).reshape(want.shape), want)
            assert same_bits(m.predict(xp.numpy()).reshape(want.shape), want)
        assert same_bits(m.predict(xs[0]).reshape(rows, 1), o.predict(xs[0]))


@pytest.mark.parametrize("decision", ["le", "lt"])
def test_float32_cast_models_narrow_host_rows(gpu, decision):
    """Pageable host batches above the small-call size of float32-cast models
    without preprocessing are rounded to float32 while they are staged.
    Doubles just beside the thresholds, subnormal, overflowing and infinite
    values, on complete, deep and shallow forests, must give the reference's
    bits, as must the same rows from a pinned buffer (sent as float64) and a
    model with preprocessing (which keeps float64 rows)."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(len(decision) * 7)
    pre = {"mean": rng.normal(size=6), "scale": rng.uniform(0.5, 2.0, 6), "clip": (-1.2, 1.7)}
    for depth, trees, preprocess in ((8, 70, None), (14, 90, None), (5, 40, None), (8, 50, pre)):
        model = random_model(rng, features=6, trees=trees, max_depth=depth, cast="f32", decision=decision,
                             inf_thresholds=0.05, preprocess=preprocess)
        x = edge_inputs(rng, 9000, 6, special=0.3)
        near = rng.random(x.shape) < 0.1
        scale = rng.choice([-1.0, 1.0], size=int(near.sum())) * 10.0 ** rng.uniform(-15, -6, size=int(near.sum()))
        x[near] = rng.choice(GRID, size=int(near.sum())) * (1 + scale) + scale
        odd = rng.random(x.shape) < 0.05
        x[odd] = rng.choice(np.array(NARROWING), size=int(odd.sum()))
        check(model, x, leaves=preprocess is None)
        want = Oracle(model).predict(x)
        got = montlok.load(model).predict(torch.from_numpy(x).pin_memory().numpy())
        assert same_bits(got.reshape(want.shape), want)


def test_small_calls_after_a_model_that_dirties_the_scratch(gpu):
    """A thread's workspace scratch is shared by the models it runs: a wide
    model's global key tables fill it, then small calls on a complete-tree
    model (whose kernel counts finished CTAs) must still be exact."""
    rng = np.random.default_rng(21)
    wide = random_model(rng, features=1200, trees=40, max_depth=10)
    xw = edge_inputs(rng, 4000, 1200, 0.3)
    small = synth.model_c5(trees=200).to_bytes()
    m_wide, m_small, o_small = montlok.load(wide), montlok.load(small), Oracle(small)
    for rows in (1, 64, 33, 1):
        m_wide.predict(xw)
        x = synth.inputs_c5(batch=rows)
        assert same_bits(m_small.predict(x).reshape(rows, 1), o_small.predict(x))


def test_single_row_and_empty_batch(gpu):
    rng = np.random.default_rng(2)
    model = random_model(rng, features=5, trees=30)
    m = montlok.load(model)
    x = edge_inputs(rng, 10, 5)
    block = m.predict(x)
    rows = np.stack([m.predict(r) for r in x])
    assert same_bits(block, rows)
    assert m.predict(np.zeros((0, 5))).shape == (0, 1)


def test_shared_nodes_and_infinite_thresholds(gpu):
    """Mirrors the reference test of the same name (tests/python/test_trees.py:275-283)."""
    nodes = export.Nodes()
    split = nodes.add(feature=0, threshold=-np.inf, flags=1 | (1 << 1))
    nodes.left[split] = nodes.add(value=1.0)
    nodes.right[split] = nodes.add(value=2.0)
    model = export.tree_ensemble(nodes, [split, split], [0, 0], features=1).to_bytes()
    x = np.array([[-np.inf], [-1e308], [0.0], [np.inf], [np.nan]])
    np.testing.assert_array_equal(montlok.load(model).predict(x)[:, 0], [2.0, 4.0, 4.0, 4.0, 2.0])
    check(model, x)


def test_many_features_use_global_key_tables(gpu):
    """Over ~1750 (feature, rule) slots the key tables move to global memory."""
    rng = np.random.default_rng(3)
    model = random_model(rng, features=1200, trees=400, max_depth=10)
    check(model, edge_inputs(rng, 300, 1200, special=0.3))


def test_wide_rows_over_several_pipelined_chunks(gpu):
    """A host call is cut into 64 MB chunks that alternate between two
    streams; with 3000 float64 features a chunk is 2796 rows, so 5597 rows
    run three chunks, two of them at once, each with its own global key
    tables."""
    rng = np.random.default_rng(31)
    model = random_model(rng, features=3000, trees=40, max_depth=10)
    x = edge_inputs(rng, 2 * 2796 + 5, 3000, special=0.3)
    o, m = Oracle(model), montlok.load(model)
    want = o.predict(x)
    assert m.kernel(len(x)) == "generic-global-keys"
    for _ in range(2):
        assert same_bits(m.predict(x).reshape(want.shape), want)
    np.testing.assert_array_equal(m.predict_leaves(x), o.leaves(x))


def test_device_buffers_match_host_buffers(gpu):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(4)
    model = random_model(rng, features=8, trees=100, outputs=3, link="softmax")
    m = montlok.load(model)
    x = edge_inputs(rng, 1000, 8)
    host = m.predict(x)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty((1000, 3), dtype=torch.float64, device="cuda")
    m.predict(xd, out=out)
    torch.cuda.synchronize()
    assert same_bits(out.cpu().numpy(), host)


def test_concurrent_callers_get_the_same_bits(gpu):
    rng = np.random.default_rng(6)
    model = random_model(rng, features=6, trees=120, cast="f32", decision="lt")
    m = montlok.load(model)
    rows = edge_inputs(rng, 64, 6)
    expected = m.predict(rows)
    with ThreadPoolExecutor(6) as pool:
        got = list(pool.map(lambda r: m.predict(r), rows))
    assert same_bits(np.stack(got), expected)


def test_concurrent_large_host_calls_share_the_staging_pool(gpu):
    """Threads predict batches of several 64 MB chunks from pageable and
    pinned host buffers at once, on a float32-cast model (pageable rows
    narrowed while staged) and a float64 one: the staging jobs share one
    pool of host threads, and every result equals the same call made alone
    (and the oracle on a slice)."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(41)
    models = [synth.model_c2(trees=40).to_bytes(),
              random_model(rng, features=128, trees=60, max_depth=10, cast="f64")]
    x = synth.inputs_c2(batch=150_000)
    pinned = torch.from_numpy(x).pin_memory().numpy()
    for model in models:
        m = montlok.load(model)
        alone = m.predict(x)
        want = Oracle(model).predict(x[:2000])
        assert same_bits(alone[:2000].reshape(want.shape), want)
        with ThreadPoolExecutor(4) as pool:
            got = list(pool.map(lambda i: m.predict(x if i % 2 == 0 else pinned), range(8)))
        for g in got:
            assert same_bits(g, alone)


def test_concurrent_mixed_calls_on_several_models(gpu):
    """Threads interleave calls of many shapes on several models (each thread
    its own workspace and graph cache, evicting shapes past its capacity):
    every result is the oracle's."""
    rng = np.random.default_rng(16)
    models = [synth.model_c2(trees=70).to_bytes(), synth.model_c4(rounds=6).to_bytes(),
              random_model(rng, features=6, trees=90, max_depth=13)]
    loaded = [montlok.load(b) for b in models]
    oracles = [Oracle(b) for b in models]
    inputs = [synth.inputs_c2(batch=3000), synth.inputs_c4(batch=3000), edge_inputs(rng, 3000, 6)]
    sizes = [1, 3, 8, 33, 64, 65, 200, 1000, 3000, 7, 2, 129]

    def job(i: int) -> bool:
        k = i % 3
        n = sizes[i % len(sizes)]
        x = inputs[k][(i * 37) % 100:][:n]
        return same_bits(loaded[k].predict(x).reshape(len(x), -1), oracles[k].predict(x))

    with ThreadPoolExecutor(8) as pool:
        assert all(pool.map(job, range(96)))


def test_stream_is_stateless_predict(gpu):
    rng = np.random.default_rng(8)
    m = montlok.load(random_model(rng, features=4, trees=20))
    live = m.stream()
    x = edge_inputs(rng, 20, 4)
    for row in x:
        assert same_bits(live.step(row), m.predict(row))


@pytest.mark.parametrize("fault", ["alloc", "copy", "launch"])
def test_injected_cuda_failures_are_clean_errors(gpu, fault):
    # 100 rows: past the small-batch kernel, whose cluster form reads small
    # calls' rows from pinned memory with no copy for "copy" to fail
    rng = np.random.default_rng(9)
    m = montlok.load(random_model(rng, features=4, trees=10))
    x = edge_inputs(rng, 100, 4)
    expected = m.predict(x)
    errors = []

    def call():  # a fresh thread has no workspace yet, so "alloc" bites
        try:
            m.predict(x)
        except RuntimeError as e:
            errors.append(str(e))

    os.environ["MONTLOK_FAULT_INJECT"] = fault
    try:
        t = threading.Thread(target=call)
        t.start()
        t.join()
    finally:
        del os.environ["MONTLOK_FAULT_INJECT"]
    assert errors and "injected fault" in errors[0]
    assert same_bits(m.predict(x), expected)
