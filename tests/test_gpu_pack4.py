"""4-bit bin matrix: when every feature has at most 16 bins (max_bin <= 15), the device
keeps two bins per byte. Binning, histograms, partitions, score updates and whole trees
must be exactly those of the one-byte matrix and of the oracle."""

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TREE_EXACT = ["split_feature", "threshold_bin", "decision_type", "left_child", "right_child",
              "leaf_count", "internal_count"]
TREE_BITS = ["leaf_value", "leaf_weight", "internal_value", "split_gain"]


def _dataset(F=28, n=40_000, max_bin=15, cats=(), seed=3, pack=True):
    import lightgbm_rs_b200 as lgb
    from lightgbm_rs_b200 import synthetic

    X, y = synthetic.binary_c0(num_data=n, num_features=F, seed=seed)
    X = X.astype(np.float64)
    for c in cats:
        X[:, c] = np.minimum(np.abs(X[:, c]) * 5, 13).astype(np.int64)
    saved = os.environ.get("LGBM_B200_PACK4")
    os.environ["LGBM_B200_PACK4"] = "1" if pack else "0"
    try:
        ds = lgb.Dataset(X, y, {"max_bin": max_bin, "min_data_in_leaf": 20},
                         categorical_feature=list(cats))
        ds.construct()
    finally:
        if saved is None:
            os.environ.pop("LGBM_B200_PACK4", None)
        else:
            os.environ["LGBM_B200_PACK4"] = saved
    return X, y, ds


def _metas(ds):
    return [{k: m[k] for k in ("num_bin", "default_bin", "most_freq_bin", "missing_type",
                               "bin_type")} for m in ds.mappers]


def _equal(a, b, tag):
    assert a["num_leaves"] == b["num_leaves"], tag
    for k in TREE_EXACT:
        assert np.asarray(a[k]).tolist() == np.asarray(b[k]).tolist(), (tag, k)
    for k in TREE_BITS:
        x = np.asarray(a[k])
        assert x.tobytes() == np.asarray(b[k]).astype(x.dtype).tobytes(), (tag, k)


@pytest.mark.parametrize("F", [7, 28, 45])
def test_packed_device_bins_equal_host_bins(F):
    X, y, ds = _dataset(F=F, n=5_003)
    assert max(m["num_bin"] for m in ds.mappers) <= 16
    assert np.array_equal(ds.device_bins(), ds.bins.astype(np.uint8))


@pytest.mark.parametrize("leaves,quant_bins", [(31, 4), (255, 4), (63, 16)])
def test_packed_quantized_trees_bit_exact(leaves, quant_bins):
    """4 quant bins: the fused partition and root build on 4-bit rows; 16: the separate
    partition and k_build on 4-bit rows."""
    import lightgbm_rs_b200 as lgb
    import oracle

    X, y, ds = _dataset()
    p = {"objective": "binary", "num_leaves": leaves, "min_data_in_leaf": 20,
         "learning_rate": 0.1, "use_quantized_grad": True, "num_grad_quant_bins": quant_bins}
    b = lgb.train(p, ds, num_boost_round=4)
    ref = oracle.train(ds.bins, _metas(ds), y, objective="binary", num_iterations=4,
                       learning_rate=0.1, num_leaves=leaves, use_quantized_grad=True,
                       stochastic_rounding=True, num_grad_quant_bins=quant_bins,
                       min_data_in_leaf=20)
    for i, (a, w) in enumerate(zip(b.trees(), ref["trees"])):
        _equal(a, w, f"tree {i}")
    assert b.train_scores().tobytes() == ref["scores"].tobytes()


def test_packed_equals_unpacked_f32_and_categorical():
    """f32 gradients (the fused f32 partition on 4-bit rows) and two categorical features:
    the 4-bit and the one-byte matrix grow the same trees and scores."""
    import lightgbm_rs_b200 as lgb

    p = {"objective": "binary", "num_leaves": 63, "min_data_in_leaf": 20, "learning_rate": 0.1}
    out = []
    for pack in (True, False):
        X, y, ds = _dataset(F=20, cats=(3, 11), pack=pack)
        b = lgb.train(p, ds, num_boost_round=3)
        out.append((b.trees(), b.train_scores()))
    for i, (a, w) in enumerate(zip(out[0][0], out[1][0])):
        _equal(a, w, f"tree {i}")
    assert out[0][1].tobytes() == out[1][1].tobytes()
