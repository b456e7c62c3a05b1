"""scikit-learn tree models exported to .montlok and predicted on the GPU.

The families the reference's exporter produces (python/montlok/export.py:
decision trees and extra trees, random-forest mean, gradient boosting with
the learning rate folded into the leaves, histogram gradient boosting with
the exp link of the Poisson loss, a StandardScaler as the float64
preprocess): every prediction bit-identical to the oracle (the reference's
arithmetic), and within 1e-12 relative of scikit-learn's own predict, whose
float summation order differs from the reference's 64-tree blocks.
"""

from __future__ import annotations

import numpy as np
import pytest

import montlok
from forests import same_bits
from montlok import export
from oracle import Oracle

pytestmark = pytest.mark.gpu

sklearn = pytest.importorskip("sklearn")
from sklearn import ensemble, pipeline, preprocessing, tree  # noqa: E402


def data(n: int = 3000, features: int = 7, nan: bool = False, seed: int = 0):
    rng = np.random.default_rng(seed)
    x = rng.normal(size=(n, features))
    y = np.sin(x[:, 0]) + 0.5 * x[:, 1] * x[:, 2] + 0.1 * rng.normal(size=n)
    if nan:
        x[rng.random(x.shape) < 0.05] = np.nan
    return x, y


ESTIMATORS = {
    "decision_tree": lambda: tree.DecisionTreeRegressor(max_depth=12, random_state=0),
    "extra_tree": lambda: tree.ExtraTreeRegressor(max_depth=10, random_state=0),
    "random_forest": lambda: ensemble.RandomForestRegressor(n_estimators=90, max_depth=14, random_state=0),
    "extra_trees": lambda: ensemble.ExtraTreesRegressor(n_estimators=70, max_depth=9, random_state=0),
    "gradient_boosting": lambda: ensemble.GradientBoostingRegressor(n_estimators=150, max_depth=4, learning_rate=0.07,
                                                                    random_state=0),
    "hist_gradient_boosting": lambda: ensemble.HistGradientBoostingRegressor(max_iter=120, random_state=0),
    "scaled_forest": lambda: pipeline.make_pipeline(preprocessing.StandardScaler(),
                                                    ensemble.RandomForestRegressor(n_estimators=40, max_depth=10,
                                                                                   random_state=0)),
}


@pytest.mark.parametrize("name", sorted(ESTIMATORS))
def test_sklearn_regressors(gpu, name):
    nan = name == "hist_gradient_boosting"
    x, y = data(nan=nan)
    est = ESTIMATORS[name]().fit(x, y)
    model = export.from_sklearn(est).to_bytes()
    m = montlok.load(model)
    xt, _ = data(2000, nan=nan, seed=1)
    got = m.predict(xt).reshape(-1)
    assert same_bits(got, Oracle(model).predict(xt).reshape(-1))
    want = est.predict(xt)
    np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-12)


def test_poisson_histogram_boosting_uses_the_exp_link(gpu):
    x, _ = data()
    y = np.random.default_rng(2).poisson(np.exp(0.3 * x[:, 0] + 0.2 * x[:, 1]))
    est = ensemble.HistGradientBoostingRegressor(loss="poisson", max_iter=80, random_state=0).fit(x, y)
    model = export.from_sklearn(est).to_bytes()
    assert export.read(model)[0]["config"]["link"] == "exp"
    xt, _ = data(1500, seed=3)
    got = montlok.load(model).predict(xt).reshape(-1)
    assert same_bits(got, Oracle(model).predict(xt).reshape(-1))
    np.testing.assert_allclose(got, est.predict(xt), rtol=1e-12)
