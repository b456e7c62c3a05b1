"""The latency engine: small host calls answered by a resident kernel.

With latency threads on (montlok_set_latency_threads(n > 0), the setting the
reference uses for its spinning single-row workers), host-buffer predicts of
at most 8 rows on complete-tree models go to a kernel that stays resident per
calling thread, holds each 64-tree block in one CTA's shared memory and
answers requests posted in pinned host memory. Engines of at most 16 blocks
run as one thread-block cluster (rows pushed into every CTA's shared memory
for requests of 1 or 2 c5 rows, relayed through device memory for larger
ones; block sums gathered in CTA 0's shared memory); larger ones meet through
device memory (the 1100-tree model, 18 blocks). Every answer must carry the
oracle's bits: preprocessing, float32 and float64 models (ties decided on the
double), every missing-value rule, mean aggregation, float32 inputs, every
row count up to 8, several threads each with their own engine, an engine that
left after its idle limit and was started again, and the way back to the
graph path when latency threads are turned off.
"""

from __future__ import annotations

import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import montlok
from forests import edge_inputs, full_model, near_thresholds, random_model, same_bits
from montlok import synth
from oracle import Oracle

pytestmark = pytest.mark.gpu


@pytest.fixture
def engine(gpu):
    montlok.set_latency_threads(1)
    yield
    montlok.set_latency_threads(0)


def models():
    rng = np.random.default_rng(17)
    return {
        "c5": full_model("c5"),
        "f64_every_rule": random_model(rng, features=7, trees=150, max_depth=8, inf_thresholds=0.1, link="sigmoid"),
        "f32_lt_mean": random_model(rng, features=6, trees=70, max_depth=6, cast="f32", decision="lt",
                                    aggregate="mean", base=0.5),
        "blocks_18": random_model(rng, features=10, trees=1100, max_depth=6, inf_thresholds=0.05, link="sigmoid"),
        "one_block": random_model(rng, features=5, trees=40, max_depth=7, link="exp"),  # a cluster of one CTA
    }


@pytest.mark.parametrize("name", ["c5", "f64_every_rule", "f32_lt_mean", "blocks_18", "one_block"])
def test_engine_answers_small_calls_exactly(engine, name):
    model = models()[name]
    m, o = montlok.load(model), Oracle(model)
    rng = np.random.default_rng(len(name))
    for rows in (1, 2, 3, 4, 5, 7, 8, 1, 8):
        x = synth.inputs_c5(batch=rows) if name == "c5" else edge_inputs(rng, rows, m.features, 0.3)
        if name != "c5":
            x = near_thresholds(model, x, rng, frac=0.3)
        for _ in range(3):
            assert same_bits(m.predict(x).reshape(rows, 1), o.predict(x))
        x32 = np.ascontiguousarray(x, dtype=np.float32)
        assert same_bits(m.predict(x32).reshape(rows, 1), o.predict(x32))


def test_each_thread_has_its_own_engine(engine):
    all_models = models()
    loaded = {k: montlok.load(v) for k, v in all_models.items()}
    oracles = {k: Oracle(v) for k, v in all_models.items()}
    rng = np.random.default_rng(5)
    inputs = {k: edge_inputs(rng, 64, loaded[k].features, 0.2) for k in all_models}
    names = sorted(all_models)

    def job(i: int) -> bool:
        k = names[i % len(names)]
        x = inputs[k][i % 60:][: 1 + i % 8]
        return same_bits(loaded[k].predict(x).reshape(len(x), 1), oracles[k].predict(x))

    with ThreadPoolExecutor(4) as pool:
        assert all(pool.map(job, range(200)))


def test_engine_restarts_after_its_idle_limit(engine):
    model = models()["f32_lt_mean"]
    m, o = montlok.load(model), Oracle(model)
    x = edge_inputs(np.random.default_rng(9), 3, m.features)
    assert same_bits(m.predict(x).reshape(3, 1), o.predict(x))
    time.sleep(0.6)  # past the engine's idle limit: it has left
    for _ in range(3):
        assert same_bits(m.predict(x).reshape(3, 1), o.predict(x))


def test_turning_latency_threads_off_returns_to_the_graph_path(engine):
    model = models()["c5"]
    m, o = montlok.load(model), Oracle(model)
    x = synth.inputs_c5(batch=4)
    assert same_bits(m.predict(x).reshape(4, 1), o.predict(x))
    montlok.set_latency_threads(0)
    assert montlok.latency_threads() == 0
    for _ in range(2):
        assert same_bits(m.predict(x).reshape(4, 1), o.predict(x))
