"""Whole-tree and whole-training parity of the device learner against the oracle.

Quantized gradients (the reference's use_quantized_grad path, gbdt.rs:931-959):
trees, leaf values, split gains and leaf row sets must be bit-identical.
f32 gradients: histograms accumulate in 64-bit fixed point, so the tree structure
must match and leaf values agree to 1e-9 relative (near-tie splits are reported).
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TREE_EXACT = ["split_feature", "threshold_bin", "decision_type", "left_child", "right_child",
              "leaf_count", "internal_count"]
TREE_BITS = ["leaf_value", "leaf_weight", "internal_value", "split_gain"]


@pytest.fixture(scope="module")
def data():
    import lightgbm_rs_b200 as lgb
    from lightgbm_rs_b200 import synthetic

    X, y = synthetic.binary_c0(num_data=60_000, seed=1)
    params = {"max_bin": 255, "min_data_in_leaf": 20}
    ds = lgb.Dataset(X, y, params)
    metas = [{"num_bin": m["num_bin"], "default_bin": m["default_bin"],
              "most_freq_bin": m["most_freq_bin"], "missing_type": m["missing_type"]}
             for m in ds.mappers]
    return X, y, ds, metas


def _assert_trees_bit_equal(got, want, tag):
    assert got["num_leaves"] == want["num_leaves"], tag
    for k in TREE_EXACT:
        assert got[k].tolist() == want[k].tolist(), (tag, k)
    for k in TREE_BITS:
        a = np.asarray(got[k])
        b = np.asarray(want[k]).astype(a.dtype)
        assert a.tobytes() == b.tobytes(), (tag, k)


def _leaf_sets(part, nl):
    out = []
    for l in range(nl):
        b, c = part["leaf_begin"][l], part["leaf_count"][l]
        out.append(np.sort(part["indices"][b:b + c]))
    return out


@pytest.mark.parametrize("num_quant_bins,num_leaves", [(4, 31), (4, 255), (16, 63)])
def test_quantized_tree_bit_exact(data, num_quant_bins, num_leaves):
    import lightgbm_rs_b200 as lgb
    import oracle

    X, y, ds, metas = data
    init = oracle.boost_from_score("binary", y)
    rng = np.random.default_rng(num_leaves)
    score = init + rng.normal(0, 0.3, len(y))  # a mid-training score
    g, h = oracle.binary_gradients(score, y)
    gq, hq, q, scales = oracle.quantize(g, h, num_quant_bins)
    want, wpart, _ = oracle.grow_tree(ds.bins, metas, gq, hq, num_leaves=num_leaves,
                                      min_data_in_leaf=20, min_sum_hessian_in_leaf=1e-3)
    learner = lgb.Learner(ds, {"num_leaves": num_leaves, "min_data_in_leaf": 20})
    sc = [scales[0], scales[1], scales[2], num_quant_bins]
    got, gpart = learner.grow(quantized=q, scales=sc)
    _assert_trees_bit_equal(got, want, f"q{num_quant_bins}/L{num_leaves}")
    assert gpart["leaf_count"].tolist() == wpart["leaf_count"].tolist()
    for a, b in zip(_leaf_sets(gpart, got["num_leaves"]), _leaf_sets(wpart, want["num_leaves"])):
        assert np.array_equal(a, b)


def test_quantized_tree_with_regularisation(data):
    import lightgbm_rs_b200 as lgb
    import oracle

    X, y, ds, metas = data
    g, h = oracle.binary_gradients(np.zeros(len(y)), y)
    gq, hq, q, scales = oracle.quantize(g, h, 4)
    kw = dict(min_data_in_leaf=50, min_sum_hessian_in_leaf=1.0, lambda_l1=0.5, lambda_l2=2.0,
              min_gain_to_split=0.1, max_delta_step=0.7, path_smooth=3.0)
    want, _, _ = oracle.grow_tree(ds.bins, metas, gq, hq, num_leaves=63, max_depth=7, **kw)
    learner = lgb.Learner(ds, {"num_leaves": 63, "max_depth": 7, **kw})
    got, _ = learner.grow(quantized=q, scales=[scales[0], scales[1], scales[2], 4])
    _assert_trees_bit_equal(got, want, "regularised")


def test_float_tree_matches_within_tolerance(data):
    import lightgbm_rs_b200 as lgb
    import oracle

    X, y, ds, metas = data
    g, h = oracle.binary_gradients(np.zeros(len(y)), y)
    want, _, _ = oracle.grow_tree(ds.bins, metas, g, h, num_leaves=31, min_data_in_leaf=20)
    learner = lgb.Learner(ds, {"num_leaves": 31, "min_data_in_leaf": 20})
    got, _ = learner.grow(g=g, h=h)
    assert got["num_leaves"] == want["num_leaves"]
    for k in TREE_EXACT:
        assert got[k].tolist() == want[k].tolist(), k
    np.testing.assert_allclose(got["leaf_value"], want["leaf_value"], rtol=1e-9, atol=1e-12)


def test_booster_quantized_bit_exact_vs_oracle(data):
    """Gbdt loop on device (gradients, quantization, trees, shrinkage, score update)
    vs the oracle loop, 10 iterations, use_quantized_grad with 4 bins."""
    import lightgbm_rs_b200 as lgb
    import oracle

    X, y, ds, metas = data
    params = {"objective": "binary", "num_leaves": 31, "min_data_in_leaf": 20,
              "learning_rate": 0.1, "use_quantized_grad": True, "num_grad_quant_bins": 4}
    booster = lgb.train(params, ds, num_boost_round=10)
    ref = oracle.train(ds.bins, metas, y, objective="binary", num_iterations=10,
                       learning_rate=0.1, num_leaves=31, use_quantized_grad=True,
                       stochastic_rounding=True,
                       num_grad_quant_bins=4, min_data_in_leaf=20)
    trees = booster.trees()
    assert len(trees) == len(ref["trees"])
    for i, (a, b) in enumerate(zip(trees, ref["trees"])):
        _assert_trees_bit_equal(a, b, f"tree {i}")
    s = booster.train_scores()
    assert s.view(np.uint64).tolist() == ref["scores"].view(np.uint64).tolist()


@pytest.mark.parametrize("stochastic", [False, True])
def test_booster_quantized_rounding_modes(data, stochastic):
    """Deterministic rounding (the reference's bit-exact gate) and stochastic rounding
    (its default: the seeded xorshift64 stream of gradient_discretizer.rs:252-262, seed
    per iteration gbdt.rs:950), 5 iterations of 63 leaves, bit-exact vs the oracle."""
    import lightgbm_rs_b200 as lgb
    import oracle

    X, y, ds, metas = data
    params = {"objective": "binary", "num_leaves": 63, "min_data_in_leaf": 20,
              "learning_rate": 0.1, "use_quantized_grad": True, "num_grad_quant_bins": 4,
              "stochastic_rounding": stochastic}
    booster = lgb.train(params, ds, num_boost_round=5)
    ref = oracle.train(ds.bins, metas, y, objective="binary", num_iterations=5,
                       learning_rate=0.1, num_leaves=63, use_quantized_grad=True,
                       stochastic_rounding=stochastic, num_grad_quant_bins=4,
                       min_data_in_leaf=20)
    for i, (a, b) in enumerate(zip(booster.trees(), ref["trees"])):
        _assert_trees_bit_equal(a, b, f"tree {i}")
    assert booster.train_scores().tobytes() == ref["scores"].tobytes()


def test_booster_stochastic_rounding_many_segments():
    """2.1M rows: the device jumps each 1024-row segment to its place in the xorshift
    stream (up to 2^22 steps); trees and scores bit-exact vs the oracle's sequential
    stream, L2 objective (constant hessian: the hessian draw is still consumed)."""
    import lightgbm_rs_b200 as lgb
    import oracle

    rng = np.random.default_rng(17)
    n, F = 2_100_000, 6
    bins = rng.integers(0, 64, (F, n)).astype(np.uint8)
    y = (bins[0].astype(np.float32) * 0.05 - bins[1] * 0.02 +
         rng.normal(0, 0.5, n).astype(np.float32)).astype(np.float32)
    mappers = [{"num_bin": 64, "default_bin": 0, "most_freq_bin": 0, "missing_type": 0,
                "bin_type": 0, "upper": np.arange(64, dtype=np.float64) + 0.5,
                "is_trivial": False} for _ in range(F)]
    params = {"objective": "regression", "num_leaves": 15, "min_data_in_leaf": 20,
              "learning_rate": 0.1, "use_quantized_grad": True, "num_grad_quant_bins": 4,
              "stochastic_rounding": True}
    ds = lgb.Dataset(bins=bins, mappers=mappers, label=y, params=params)
    booster = lgb.train(params, ds, num_boost_round=3)
    metas = [{k: m[k] for k in ("num_bin", "default_bin", "most_freq_bin", "missing_type")}
             for m in mappers]
    ref = oracle.train(bins, metas, y, objective="regression", num_iterations=3,
                       learning_rate=0.1, num_leaves=15, use_quantized_grad=True,
                       stochastic_rounding=True, num_grad_quant_bins=4, min_data_in_leaf=20,
                       nthreads=oracle.max_threads())
    for i, (a, b) in enumerate(zip(booster.trees(), ref["trees"])):
        _assert_trees_bit_equal(a, b, f"tree {i}")
    assert booster.train_scores().tobytes() == ref["scores"].tobytes()


def test_booster_float_predictions_close(data):
    import lightgbm_rs_b200 as lgb
    import oracle

    X, y, ds, metas = data
    params = {"objective": "binary", "num_leaves": 31, "min_data_in_leaf": 20,
              "learning_rate": 0.1}
    booster = lgb.train(params, ds, num_boost_round=10)
    ref = oracle.train(ds.bins, metas, y, objective="binary", num_iterations=10,
                       learning_rate=0.1, num_leaves=31, min_data_in_leaf=20)
    s = booster.train_scores()
    np.testing.assert_allclose(s, ref["scores"], rtol=0, atol=1e-5)
    p = booster.predict(X[:1000], raw_score=True)
    np.testing.assert_allclose(p, s[:1000], rtol=0, atol=1e-9)


def test_booster_l2_quantized_constant_hessian(data):
    import lightgbm_rs_b200 as lgb
    import oracle

    X, y, ds, metas = data
    yr = (X[:, 2] * 2.0 + X[:, 9]).astype(np.float32)
    ds2 = lgb.Dataset(bins=ds.bins, mappers=ds.mappers, label=yr,
                      params={"min_data_in_leaf": 20})
    params = {"objective": "regression", "num_leaves": 15, "min_data_in_leaf": 20,
              "use_quantized_grad": True, "num_grad_quant_bins": 4}
    booster = lgb.train(params, ds2, num_boost_round=5)
    ref = oracle.train(ds.bins, metas, yr, objective="l2", num_iterations=5, learning_rate=0.1,
                       num_leaves=15, use_quantized_grad=True,
                       stochastic_rounding=True, num_grad_quant_bins=4,
                       min_data_in_leaf=20)
    for i, (a, b) in enumerate(zip(booster.trees(), ref["trees"])):
        _assert_trees_bit_equal(a, b, f"l2 tree {i}")


@pytest.mark.parametrize("num_features,num_quant_bins", [(72, 4), (72, 16), (40, 4)])
def test_wide_quantized_tree_bit_exact(num_features, num_quant_bins):
    """More features than one shared-memory group: the partition and the build run as
    separate kernels (and the build spans several feature groups)."""
    import lightgbm_rs_b200 as lgb
    import oracle
    from lightgbm_rs_b200 import synthetic

    X, y = synthetic.binary_c0(num_data=30_000, num_features=num_features, seed=3)
    ds = lgb.Dataset(X, y, {"max_bin": 255, "min_data_in_leaf": 20})
    metas = [{k: m[k] for k in ("num_bin", "default_bin", "most_freq_bin", "missing_type")}
             for m in ds.mappers]
    g, h = oracle.binary_gradients(np.zeros(len(y)), y)
    gq, hq, q, scales = oracle.quantize(g, h, num_quant_bins)
    want, wpart, _ = oracle.grow_tree(ds.bins, metas, gq, hq, num_leaves=63, min_data_in_leaf=20)
    learner = lgb.Learner(ds, {"num_leaves": 63, "min_data_in_leaf": 20})
    got, gpart = learner.grow(quantized=q, scales=[scales[0], scales[1], scales[2],
                                                   num_quant_bins])
    _assert_trees_bit_equal(got, want, f"wide F{num_features} q{num_quant_bins}")
    for a, b in zip(_leaf_sets(gpart, got["num_leaves"]), _leaf_sets(wpart, want["num_leaves"])):
        assert np.array_equal(a, b)


def test_tree_that_stops_early(data):
    """A large min_data_in_leaf ends the tree before num_leaves: the remaining split
    steps run with nothing to do and must leave the next tree a clean state."""
    import lightgbm_rs_b200 as lgb
    import oracle

    X, y, ds, metas = data
    g, h = oracle.binary_gradients(np.zeros(len(y)), y)
    gq, hq, q, scales = oracle.quantize(g, h, 4)
    learner = lgb.Learner(ds, {"num_leaves": 255, "min_data_in_leaf": 4000})
    want, _, _ = oracle.grow_tree(ds.bins, metas, gq, hq, num_leaves=255, min_data_in_leaf=4000)
    assert want["num_leaves"] < 255
    for _ in range(2):
        got, _ = learner.grow(quantized=q, scales=[scales[0], scales[1], scales[2], 4])
        _assert_trees_bit_equal(got, want, "early stop")


def _missing_data(n=40_000, seed=11):
    """Numeric features with NaN (missing_type NaN), one zero-as-missing feature and a
    feature with many exact zeros, in the spirit of the reference's na_missing corpus."""
    from lightgbm_rs_b200 import synthetic

    X, y = synthetic.binary_c0(num_data=n, num_features=12, seed=seed)
    rng = np.random.default_rng(seed)
    X = X.astype(np.float64)
    for j in (0, 3, 5, 8):
        X[rng.random(n) < 0.1, j] = np.nan
    X[rng.random(n) < 0.3, 9] = 0.0
    return X, y


@pytest.mark.parametrize("zero_as_missing", [False, True])
def test_missing_values_tree_bit_exact(zero_as_missing):
    """NaN rows go to the NaN bin and are routed by default_left; zero-as-missing
    features skip the default bin in the scan (learner.rs:167-193)."""
    import lightgbm_rs_b200 as lgb
    import oracle

    X, y = _missing_data()
    params = {"max_bin": 255, "min_data_in_leaf": 20, "zero_as_missing": zero_as_missing}
    ds = lgb.Dataset(X, y, params)
    kinds = {m["missing_type"] for m in ds.mappers}
    assert kinds & {1, 2}, kinds
    metas = [{k: m[k] for k in ("num_bin", "default_bin", "most_freq_bin", "missing_type")}
             for m in ds.mappers]
    g, h = oracle.binary_gradients(np.zeros(len(y)), y)
    gq, hq, q, scales = oracle.quantize(g, h, 4)
    want, wpart, _ = oracle.grow_tree(ds.bins, metas, gq, hq, num_leaves=63, min_data_in_leaf=20)
    learner = lgb.Learner(ds, {"num_leaves": 63, "min_data_in_leaf": 20})
    got, gpart = learner.grow(quantized=q, scales=[scales[0], scales[1], scales[2], 4])
    _assert_trees_bit_equal(got, want, f"missing zero_as_missing={zero_as_missing}")
    for a, b in zip(_leaf_sets(gpart, got["num_leaves"]), _leaf_sets(wpart, want["num_leaves"])):
        assert np.array_equal(a, b)


def test_missing_values_booster_bit_exact():
    import lightgbm_rs_b200 as lgb
    import oracle

    X, y = _missing_data(seed=12)
    ds = lgb.Dataset(X, y, {"max_bin": 255, "min_data_in_leaf": 20})
    metas = [{k: m[k] for k in ("num_bin", "default_bin", "most_freq_bin", "missing_type")}
             for m in ds.mappers]
    params = {"objective": "binary", "num_leaves": 31, "min_data_in_leaf": 20,
              "learning_rate": 0.1, "use_quantized_grad": True, "num_grad_quant_bins": 4}
    booster = lgb.train(params, ds, num_boost_round=6)
    ref = oracle.train(ds.bins, metas, y, objective="binary", num_iterations=6,
                       learning_rate=0.1, num_leaves=31, use_quantized_grad=True,
                       stochastic_rounding=True,
                       num_grad_quant_bins=4, min_data_in_leaf=20)
    for i, (a, b) in enumerate(zip(booster.trees(), ref["trees"])):
        _assert_trees_bit_equal(a, b, f"missing tree {i}")
    s = booster.train_scores()
    assert s.view(np.uint64).tolist() == ref["scores"].view(np.uint64).tolist()


def test_trivial_features_left_out():
    """feature_pre_filter (the reference default, true): a constant column and a column
    with too few non-zero rows for any split of min_data_in_leaf rows on both sides are
    trivial, so the reference leaves them out of the dataset
    (lgbm-dataset/src/dataset.rs:106-126). Here they become one-bin features that never
    split; trees and scores stay bit-exact vs the oracle."""
    import lightgbm_rs_b200 as lgb
    import oracle
    from lightgbm_rs_b200 import synthetic

    X, y = synthetic.binary_c0(num_data=40_000, num_features=6, seed=9)
    X = np.concatenate([X, np.full((len(y), 1), 3.0, np.float32),
                        np.zeros((len(y), 1), np.float32)], axis=1)
    X[:10, -1] = np.arange(1, 11)  # 10 non-zero rows: no split leaves 20 on both sides
    params = {"objective": "binary", "num_leaves": 31, "min_data_in_leaf": 20,
              "use_quantized_grad": True, "num_grad_quant_bins": 4}
    ds = lgb.Dataset(X, y, params)
    assert [m["num_bin"] for m in ds.mappers[-2:]] == [1, 1]
    assert all(m["is_trivial"] for m in ds.mappers[-2:])
    assert not any(m["is_trivial"] for m in ds.mappers[:-2])
    booster = lgb.train(params, ds, num_boost_round=3)
    metas = [{k: m[k] for k in ("num_bin", "default_bin", "most_freq_bin", "missing_type")}
             for m in ds.mappers]
    ref = oracle.train(ds.bins, metas, y, objective="binary", num_iterations=3,
                       learning_rate=0.1, num_leaves=31, use_quantized_grad=True,
                       stochastic_rounding=True, num_grad_quant_bins=4, min_data_in_leaf=20)
    for i, (a, b) in enumerate(zip(booster.trees(), ref["trees"])):
        _assert_trees_bit_equal(a, b, f"tree {i}")
        assert not set(a["split_feature"].tolist()) & {6, 7}
    assert booster.train_scores().tobytes() == ref["scores"].tobytes()
    # without the pre-filter neither is trivial: the constant column keeps the zero bin
    # and its value's bin, as the reference's BinMapper does
    ds2 = lgb.Dataset(X, y, dict(params, feature_pre_filter=False))
    assert [m["num_bin"] for m in ds2.mappers[-2:]] == [2, 5]
    assert not any(m["is_trivial"] for m in ds2.mappers)


def test_wide_c2_shape_bit_exact():
    """The C2 shape at test size: 1,200 features ~ U(-1,1), max_bin 63, 127 leaves
    (several feature groups, the non-fused partition + build, one control-step CTA per
    feature), 3 boosting iterations bit-exact vs the oracle."""
    import lightgbm_rs_b200 as lgb
    import oracle
    from lightgbm_rs_b200 import synthetic

    X, y = synthetic.wide_c2(num_data=24_000, num_features=1200, seed=4)
    params = {"objective": "binary", "num_leaves": 127, "min_data_in_leaf": 20,
              "max_bin": 63, "learning_rate": 0.1, "use_quantized_grad": True,
              "num_grad_quant_bins": 4}
    ds = lgb.Dataset(X, y, params)
    assert max(m["num_bin"] for m in ds.mappers) <= 64
    booster = lgb.train(params, ds, num_boost_round=3)
    metas = [{k: m[k] for k in ("num_bin", "default_bin", "most_freq_bin", "missing_type")}
             for m in ds.mappers]
    ref = oracle.train(ds.bins, metas, y, objective="binary", num_iterations=3,
                       learning_rate=0.1, num_leaves=127, use_quantized_grad=True,
                       stochastic_rounding=True, num_grad_quant_bins=4, min_data_in_leaf=20,
                       nthreads=oracle.max_threads())
    trees = booster.trees()
    assert len(trees) == 3
    for i, (a, b) in enumerate(zip(trees, ref["trees"])):
        _assert_trees_bit_equal(a, b, f"tree {i}")
    assert booster.train_scores().tobytes() == ref["scores"].tobytes()


def test_warp_aggregated_build_same_trees():
    """The measured-only warp-aggregated histogram build (LGBM_B200_WARP_AGG=1, the
    255-bin, 28-feature layout) grows the same trees and scores as the default build, on
    data with a heavily skewed feature (most lanes of a warp share a bin)."""
    import os

    import lightgbm_rs_b200 as lgb
    from lightgbm_rs_b200 import synthetic

    X, y = synthetic.binary_c0(num_data=60_000, num_features=28, seed=11)
    X[np.random.default_rng(2).random(len(y)) < 0.8, 3] = 0.0
    ds = lgb.Dataset(X, y, {"max_bin": 255})
    p = {"objective": "binary", "num_leaves": 63, "use_quantized_grad": True,
         "num_grad_quant_bins": 4}
    out = []
    for agg in ("0", "1"):
        os.environ["LGBM_B200_WARP_AGG"] = agg
        try:
            b = lgb.train(p, ds, num_boost_round=3)
        finally:
            os.environ.pop("LGBM_B200_WARP_AGG", None)
        out.append((b.trees(), b.train_scores()))
    for a, w in zip(out[0][0], out[1][0]):
        for k in ("split_feature", "threshold_bin", "left_child", "right_child", "leaf_count"):
            assert np.asarray(a[k]).tolist() == np.asarray(w[k]).tolist(), k
        assert np.asarray(a["leaf_value"]).tobytes() == np.asarray(w["leaf_value"]).tobytes()
    assert out[0][1].tobytes() == out[1][1].tobytes()
