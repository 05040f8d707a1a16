"""Handle lifetimes: a garbage collector may free a dataset handle before the booster
built on it (for example when both sit in a reference cycle kept by a traceback)."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dataset():
    import lightgbm_rs_b200 as lgb

    rng = np.random.default_rng(3)
    X = rng.normal(0, 1, (50_000, 12))
    y = (X[:, 0] + rng.normal(0, 1, len(X)) > 0).astype(np.float32)
    p = {"objective": "binary", "num_leaves": 31, "use_quantized_grad": True,
         "num_grad_quant_bins": 4}
    return lgb.Dataset(X, y, p), p


def test_booster_destroyed_after_its_dataset():
    """Destroying the booster after its dataset touches only the booster's own state, and
    no stale CUDA error reaches the next call."""
    import lightgbm_rs_b200 as lgb
    from lightgbm_rs_b200 import _lib as C

    ds, p = _dataset()
    b = lgb.Booster(p, ds)
    b.update(1)
    L = C.lib()
    assert L.lgbm_b200_dataset_destroy(ds._handle) == C.OK
    ds._handle = None
    assert L.lgbm_b200_booster_destroy(b._handle) == C.OK
    b._handle = None
    ds2, _ = _dataset()
    b2 = lgb.Booster(p, ds2)
    assert b2.update(1) == 1
