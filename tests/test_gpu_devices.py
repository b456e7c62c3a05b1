"""Host-buffer predicts split over several GPUs (montlok_set_devices).

A call with set_devices(n) cuts the rows into n contiguous slices, each
predicted on its own GPU by that device's long-lived worker thread, which
writes its slice of `out`. The results must be the one-GPU results bit for
bit (and the oracle's), across repeated calls of several shapes from several
threads (each device's worker keeps its buffers between calls), and a shard
that fails must fail the whole call cleanly. Needs two or more GPUs.
"""

from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import montlok
from forests import same_bits
from montlok import synth
from oracle import Oracle

pytestmark = pytest.mark.gpu


@pytest.fixture
def devices(gpu):
    if montlok.device_count() < 2:
        pytest.skip("needs two or more GPUs")
    yield montlok.device_count()
    montlok.set_devices(0)


def test_split_calls_match_one_gpu(devices):
    cases = [(synth.model_c2(trees=200).to_bytes(), synth.inputs_c2(batch=20_011)),
             (synth.model_c4(rounds=20).to_bytes(), synth.inputs_c4(batch=9_001))]
    for model, x in cases:
        m = montlok.load(model)
        alone = m.predict(x)
        assert same_bits(alone[:500].reshape(500, -1), Oracle(model).predict(x[:500]))
        for n in sorted({2, devices}):
            montlok.set_devices(n)
            for rows in (len(x), 4097, 3, 1):
                assert same_bits(m.predict(x[:rows]).reshape(rows, -1), alone[:rows].reshape(rows, -1))
            with ThreadPoolExecutor(3) as pool:
                got = list(pool.map(lambda _: m.predict(x), range(6)))
            assert all(same_bits(g, alone) for g in got)
        montlok.set_devices(0)


def test_a_failing_shard_fails_the_call(devices):
    m = montlok.load(synth.model_c2(trees=64).to_bytes())
    x = synth.inputs_c2(batch=10_000)
    want = m.predict(x)
    montlok.set_devices(2)
    os.environ["MONTLOK_FAULT_INJECT"] = "shard"
    try:
        with pytest.raises(RuntimeError, match="shard"):
            m.predict(x)
    finally:
        del os.environ["MONTLOK_FAULT_INJECT"]
    assert same_bits(m.predict(x), want)
