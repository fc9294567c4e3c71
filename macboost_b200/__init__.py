"""macboost_b200 -- B200 batch inference for MacBoost tree ensembles.

Scores models saved by MacBoost (its JSON model file) on NVIDIA B200 GPUs
through libmacboostc.so, a C ABI compatible with MacBoost's own
(Sources/MacBoostC/CAPI.swift).  The estimator classes mirror the predict side
of MacBoost's scikit-learn wrappers (python/macboost/__init__.py):

    from macboost_b200 import MacBoostClassifier
    model = MacBoostClassifier.load_model("model.json")
    p = model.predict_proba(X)          # sigmoid / softmax fused on the GPU

Training is not part of this package (it is an inference engine).
"""

import numpy as np

from . import _core
from ._core import MacBoostError

__all__ = ["MacBoostRegressor", "MacBoostClassifier", "MacBoostError", "load_model"]
__version__ = "0.1.0"


class _BaseBooster:
    """Predict-side surface of MacBoost's _BaseBooster (__init__.py:109-390)."""

    def __init__(self, devices=None):
        self.devices = list(devices) if devices else None
        self._handle = None
        self.classes_ = None

    def fit(self, *args, **kwargs):
        raise MacBoostError("training requires MacBoost's Metal core; this package is the "
                            "B200 inference engine -- use load_model() on a saved model")

    @classmethod
    def load_model(cls, path, devices=None):
        model = cls(devices=devices)
        model._handle = _core.load(path)
        return model

    def _need(self):
        if self._handle is None:
            raise MacBoostError("model is not loaded; call load_model()")
        return self._handle

    def _run(self, X, kind):
        out = _core.predict_ex(self._need(), X, kind=kind, layout="row", devices=self.devices)
        return out

    def _raw_predict(self, X):
        raw = self._run(X, _core.KIND_RAW)
        return raw[:, 0] if raw.shape[1] == 1 else raw

    predict_raw = _raw_predict

    def predict_leaf(self, X):
        """Heap index of the leaf reached in every tree, (rows, n_trees) int32."""
        return self._run(X, _core.KIND_LEAF)

    def predict_contrib(self, X):
        """SHAP contributions (MacBoost's predict_contrib, __init__.py:338-348):
        rows x (n_features + 1) per class, the expected value last; each row
        (per class) sums to the raw prediction.  Computed on the GPU."""
        return _core.predict_contrib_ex(self._need(), X, layout="row", devices=self.devices)

    def feature_importance(self, importance_type="gain"):
        return _core.feature_importance(self._need(), importance_type)

    @property
    def feature_importances_(self):
        return self.feature_importance()

    def save_model(self, path):
        _core.save(self._need(), path)

    @property
    def n_trees_(self):
        return _core.num_trees(self._handle) if self._handle else 0

    @property
    def n_features_in_(self):
        return _core.num_features(self._handle) if self._handle else 0

    n_features_ = n_features_in_

    @property
    def best_iteration_(self):
        best = _core.best_iteration(self._handle) if self._handle else 0
        return best or None

    def describe(self):
        """JSON description of the device layout and launch plan."""
        return _core.describe(self._need())


class MacBoostRegressor(_BaseBooster):
    _estimator_type = "regressor"

    def predict(self, X):
        """MacBooster.predict: raw margins, exp() for poisson / tweedie."""
        out = self._run(X, _core.KIND_PREDICT)
        return out[:, 0] if out.shape[1] == 1 else out

    def score(self, X, y):
        y = np.asarray(y, dtype=np.float64).ravel()
        pred = self.predict(X).astype(np.float64)
        ss_res = float(np.sum((y - pred) ** 2))
        ss_tot = float(np.sum((y - y.mean()) ** 2))
        return 1.0 - ss_res / ss_tot if ss_tot > 0 else 0.0


class MacBoostClassifier(_BaseBooster):
    _estimator_type = "classifier"

    def predict_proba(self, X):
        """MacBoostClassifier.predict_proba (__init__.py:433-445): [1-p, p] for
        one class, softmax over classes otherwise; computed in float64 on the
        GPU and returned as float64 of the float32-rounded values."""
        return self._run(X, _core.KIND_PROBA).astype(np.float64)

    def predict(self, X):
        idx = np.argmax(self.predict_proba(X), axis=1)
        classes = self.classes_
        if classes is None:
            k = max(_core.num_classes(self._need()), 2)
            classes = np.arange(k)
        return classes[idx]

    def score(self, X, y):
        return float(np.mean(self.predict(X) == np.asarray(y).ravel()))


def load_model(path, devices=None):
    """Load a model as a regressor (predict returns MacBooster.predict values)."""
    return MacBoostRegressor.load_model(path, devices=devices)
