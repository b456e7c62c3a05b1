"""Failure detection without a GPU fault: bounded waits that run out.

The complete-tree and multi-output kernels stream tree data into shared
memory with bulk copies and wait on them with a time limit. Under
MONTLOK_FAULT_INJECT=wait the host launches them with their copies switched
off and a 2 ms limit: every wait runs out, no copy is in flight, each CTA
gives up cleanly and sets the call's status word. A host-buffer call must then
fail with MONTLOK_ERROR_INTERNAL (RuntimeError here) naming the wait; a
device-buffer call (which returns before its kernel runs) reports it through
montlok_model_device_status. The next call on the same model, with the
injection off, must give the oracle's bits: the status is per call.
"""

from __future__ import annotations

import os
import threading

import numpy as np
import pytest

import montlok
from forests import edge_inputs, random_model, same_bits
from montlok import synth
from oracle import Oracle

pytestmark = pytest.mark.gpu

CASES = {
    "complete-tree": (lambda: synth.model_c2(trees=300).to_bytes(), lambda: synth.inputs_c2(batch=5000)),
    # 128 rows per CTA: the producer warps' TMEM stage beside the walkers
    "complete-tree-staged": (lambda: synth.model_c2(trees=300).to_bytes(), lambda: synth.inputs_c2(batch=40000)),
    "multi-output": (lambda: synth.model_c4(rounds=12).to_bytes(), lambda: synth.inputs_c4(batch=3000)),
}


def injected(fn):
    """Runs fn() on a fresh thread with MONTLOK_FAULT_INJECT=wait; returns the
    exception it raised (or None)."""
    raised = []

    def run():
        try:
            fn()
        except Exception as e:  # noqa: BLE001
            raised.append(e)

    os.environ["MONTLOK_FAULT_INJECT"] = "wait"
    try:
        t = threading.Thread(target=run)
        t.start()
        t.join()
    finally:
        del os.environ["MONTLOK_FAULT_INJECT"]
    return raised[0] if raised else None


@pytest.mark.parametrize("kernel", sorted(CASES))
def test_host_call_reports_a_wait_that_ran_out(gpu, kernel):
    make_model, make_x = CASES[kernel]
    model, x = make_model(), make_x()
    m = montlok.load(model)
    assert m.kernel(len(x)) == kernel
    want = Oracle(model).predict(x)
    assert same_bits(m.predict(x).reshape(want.shape), want)
    error = injected(lambda: m.predict(x))
    assert isinstance(error, RuntimeError) and "bounded wait ran out" in str(error)
    for _ in range(2):  # the same thread's workspace and a fresh call: both clean
        assert same_bits(m.predict(x).reshape(want.shape), want)


@pytest.mark.parametrize("kernel", sorted(CASES))
def test_device_call_reports_a_wait_that_ran_out(gpu, kernel):
    torch = pytest.importorskip("torch")
    make_model, make_x = CASES[kernel]
    model, x = make_model(), make_x()
    m = montlok.load(model)
    want = Oracle(model).predict(x)
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    out = torch.empty((len(x), m.outputs), dtype=torch.float64, device="cuda")

    def call():
        m.predict(xd, out=out)
        torch.cuda.synchronize()

    call()
    m.check_device_status()
    assert injected(call) is None  # the call itself returns before the kernel runs
    with pytest.raises(RuntimeError, match="gave up waiting"):
        m.check_device_status()
    m.check_device_status()  # the record was cleared
    call()
    m.check_device_status()
    assert same_bits(out.cpu().numpy(), want)


def test_kernels_without_waits_ignore_the_injection(gpu):
    """The small-batch, deep-tree and generic kernels read tree data straight
    from global memory: nothing to wait for, so the injected call succeeds
    (and the small-batch kernel's arrival counters stay consistent)."""
    rng = np.random.default_rng(3)
    for model, rows in ((random_model(rng, features=6, trees=60, max_depth=14), 500),
                        (random_model(rng, features=6, trees=60, outputs=11), 500),
                        (random_model(rng, features=6, trees=300, max_depth=8), 40)):
        m = montlok.load(model)
        x = edge_inputs(rng, rows, 6)
        want = Oracle(model).predict(x)
        got = []
        assert injected(lambda: got.append(m.predict(x))) is None
        assert same_bits(got[0].reshape(want.shape), want)
