"""The oracle against the reference itself at the benchmarked model sizes.

The GPU parity tests of the full-size recipes (test_gpu_full_size.py) compare
the kernels with the oracle; this file closes the chain on the CPU: for each
recipe at its configured size (c1 100 trees, c2 500, c3 200 deep trees grown
on 100k samples, c4 1500, c5 1000 with preprocessing), a few hundred of the
configuration's rows, with values on and beside the thresholds mixed in, get
the same prediction bits and the same leaf in every tree from the oracle and
from the reference runtime compiled from its own sources (oracle/_ref). The
reference's leaf choice is read through its own predict on a re-export of the
model whose leaves carry their node indices (oracle.Reference.leaves).
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from forests import full_model, near_thresholds, same_bits
from montlok import synth

pytestmark = pytest.mark.skipif(not oracle.available_reference(),
                                reason="the reference library (oracle/_ref) was not built here")

ROWS = {"c1": 300, "c2": 200, "c3": 200, "c4": 150, "c5": 200}


@pytest.mark.parametrize("name", sorted(ROWS))
def test_full_size_recipe_matches_the_reference(name):
    model = full_model(name)
    rng = np.random.default_rng([7, ROWS[name]])
    x = near_thresholds(model, synth.CONFIGS[name].inputs(batch=ROWS[name]), rng, frac=0.1)
    x[rng.random(x.shape) < 0.02] = np.nan
    ref = oracle.Reference()
    o = oracle.Oracle(model)
    assert same_bits(o.predict(x), ref.predict(model, x))
    np.testing.assert_array_equal(o.leaves(x), ref.leaves(model, x))
