"""Client SDK surface (reference ``libs/synthefy/src/synthefy/nori_client.py``).

``SynthefyNoriClient(mode="local", model=...)`` runs predictions in-process on this
framework (the reference's local mode calls ``synthefy_nori.predict`` /
``NoriRegressor``, nori_client.py:2011, 2241-2305). The hosted modes (``"remote"``
HTTPS to the Synthefy API, ``"sagemaker"``) need network access and credentials and are
rejected with a clear error here.
"""

from __future__ import annotations

import numpy as np

from synthefy_nori_b200.api import NoriRegressor


class SynthefyNoriClient:
    def __init__(self, mode: str = "local", model: str = "nori-6m", *, model_path: str | None = None,
                 weights: str | None = None, device=None, **regressor_kwargs):
        if mode not in ("local", "remote", "sagemaker"):
            raise ValueError(f"unknown mode {mode!r}")
        if mode != "local":
            raise RuntimeError(f"mode={mode!r} needs the hosted Synthefy service; use mode='local'")
        self.mode, self.model = mode, model
        self._kw = dict(model=model, model_path=model_path, weights=weights, device=device, **regressor_kwargs)

    def predict(self, X_train, y_train, X_test, *, output_type: str = "mean", quantiles=None):
        """Fit on (X_train, y_train) and predict X_test; ``y_train`` may be 2-D (one model
        per target column, the reference's independent multi-target strategy)."""
        y = np.asarray(y_train)
        if y.ndim == 2 and y.shape[1] > 1:
            outs = [self.predict(X_train, y[:, j], X_test, output_type=output_type, quantiles=quantiles)
                    for j in range(y.shape[1])]
            return np.stack(outs, -1)
        reg = NoriRegressor(**self._kw).fit(X_train, y.reshape(-1))
        return reg.predict(X_test, output_type=output_type, quantiles=quantiles)


__all__ = ["SynthefyNoriClient"]
