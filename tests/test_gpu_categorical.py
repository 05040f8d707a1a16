"""Categorical features on the device learner.

Pinned to lib_lightgbm 4.6 through the reference's two categorical golden cells
(oracle-harness learner_parity.rs:1486-1535: one-hot and many-vs-many), and to the oracle
on larger random data mixing numeric and categorical features: quantized trees, their
categorical node sets, leaf row sets and boosting scores bit-exact.
"""

import json

import numpy as np
import pytest

import _golden as G

pytestmark = pytest.mark.gpu

TREE_EXACT = ["split_feature", "threshold_bin", "decision_type", "left_child", "right_child",
              "leaf_count", "internal_count"]
TREE_BITS = ["leaf_value", "leaf_weight", "internal_value", "split_gain"]


def _assert_trees_bit_equal(got, want, tag):
    assert got["num_leaves"] == want["num_leaves"], tag
    for k in TREE_EXACT:
        assert got[k].tolist() == want[k].tolist(), (tag, k)
    for k in TREE_BITS:
        a = np.asarray(got[k])
        b = np.asarray(want[k]).astype(a.dtype)
        assert a.tobytes() == b.tobytes(), (tag, k)
    assert got["cat_bins"].tolist() == want["cat_bins"].tolist(), (tag, "cat_bins")


@pytest.mark.parametrize("name", ["cat_onehot", "cat_manyvsmany"])
def test_device_categorical_golden_tree(name):
    import lightgbm_rs_b200 as lgb

    side = json.loads(G.read_text(f"{name}.bins.json"))
    gold_text = G.read_text(f"{name}.txt")
    gold = G.parse_model_text(gold_text)[0]
    raw = dict(l.split("=", 1) for l in gold_text.splitlines()
               if "=" in l and l.split("=", 1)[0] in ("cat_boundaries", "cat_threshold"))
    nb, mfb = int(side["num_bin"]), int(side["most_freq_bin"])
    bins = np.array(side["bins"], dtype=np.uint8).reshape(1, -1)
    mapper = {"num_bin": nb, "default_bin": nb - 1, "most_freq_bin": mfb, "missing_type": 0,
              "bin_type": 1, "bin_to_category": np.array(side["bin_2_categorical"])}
    # the learner reads default_bin only for numerical features; keep it in range here
    ds = lgb.Dataset(bins=bins, mappers=[mapper], label=np.zeros(bins.shape[1], np.float32),
                     params={"min_data_in_leaf": 1})
    params = {"num_leaves": int(side["num_leaves"]), "min_data_in_leaf": 1,
              "min_sum_hessian_in_leaf": 1e-3, "cat_l2": side["cat_l2"],
              "cat_smooth": side["cat_smooth"],
              "min_data_per_group": int(side["min_data_per_group"]),
              "max_cat_threshold": int(side["max_cat_threshold"]),
              "max_cat_to_onehot": int(side["max_cat_to_onehot"])}
    g = np.array(side["grad"], dtype=np.float32)
    tree, _ = lgb.Learner(ds, params).grow(g=g, h=np.ones_like(g))
    assert tree["num_leaves"] == gold["num_leaves"]
    for k in ("split_feature", "decision_type", "left_child", "right_child", "leaf_count",
              "internal_count"):
        assert tree[k].tolist() == gold[k].tolist(), k
    assert [G.g17(float(t)) for t in tree["threshold_bin"]] == \
        [G.g17(t) for t in gold["threshold"]]
    bounds, words = lgb.categorical_bitsets(tree, [mapper])
    assert bounds == [int(x) for x in raw["cat_boundaries"].split()]
    assert words == [int(x) for x in raw["cat_threshold"].split()]
    lv = [0.0 if abs(v * 0.1) <= 1e-35 else v * 0.1 for v in tree["leaf_value"]]
    assert [G.g17(v) for v in lv] == [G.g17(v) for v in gold["leaf_value"]]


def _mixed_data(n=30_000, seed=5):
    """4 numeric features and 4 categorical ones (cardinality 3 -> one-hot, 12, 60, 200;
    Zipf-like codes), label from both."""
    rng = np.random.default_rng(seed)
    Xn = rng.standard_normal((n, 4))
    cards = [3, 12, 60, 200]
    Xc = np.stack([np.minimum(rng.zipf(1.3, n) - 1, c - 1) for c in cards], axis=1)
    eff = [rng.normal(0, 1, c) for c in cards]
    z = Xn @ rng.normal(0, 1, 4) + sum(eff[j][Xc[:, j]] for j in range(4))
    y = (rng.random(n) < 1 / (1 + np.exp(-z))).astype(np.float32)
    X = np.concatenate([Xn, Xc.astype(np.float64)], axis=1)
    X[rng.random(n) < 0.05, 6] = np.nan  # missing categories -> bin 0
    return X, y, [4, 5, 6, 7]


@pytest.mark.parametrize("quant_bins,max_cat_to_onehot,cat_smooth",
                         [(4, 4, 5.0), (16, 4, 5.0), (4, 16, 5.0), (4, 4, 0.0)])
def test_categorical_tree_bit_exact_vs_oracle(quant_bins, max_cat_to_onehot, cat_smooth):
    """cat_smooth 0 keeps categories without rows in a leaf, whose ratio is 0/0 (NaN):
    they keep their place in the sort and split it into runs sorted apart."""
    import lightgbm_rs_b200 as lgb
    import oracle

    X, y, cats = _mixed_data()
    params = {"max_bin": 255, "min_data_in_leaf": 20, "min_data_per_group": 50,
              "cat_smooth": cat_smooth, "max_cat_to_onehot": max_cat_to_onehot}
    ds = lgb.Dataset(X, y, params, categorical_feature=cats)
    assert [m["bin_type"] for m in ds.mappers] == [0, 0, 0, 0, 1, 1, 1, 1]
    metas = [{k: m[k] for k in ("num_bin", "default_bin", "most_freq_bin", "missing_type",
                                "bin_type")} for m in ds.mappers]
    g, h = oracle.binary_gradients(np.zeros(len(y)), y)
    gq, hq, q, scales = oracle.quantize(g, h, quant_bins)
    kw = dict(min_data_in_leaf=20, min_data_per_group=50, cat_smooth=cat_smooth,
              max_cat_to_onehot=max_cat_to_onehot)
    want, wpart, _ = oracle.grow_tree(ds.bins, metas, gq, hq, num_leaves=63, **kw)
    assert (want["decision_type"] & 1).sum() > 0, "the data should grow categorical nodes"
    learner = lgb.Learner(ds, {"num_leaves": 63, **kw})
    got, gpart = learner.grow(quantized=q, scales=[scales[0], scales[1], scales[2], quant_bins])
    _assert_trees_bit_equal(got, want,
                            f"cat q{quant_bins} onehot<={max_cat_to_onehot} smooth {cat_smooth}")
    for l in range(got["num_leaves"]):
        a = np.sort(gpart["indices"][gpart["leaf_begin"][l]:][:gpart["leaf_count"][l]])
        b = np.sort(wpart["indices"][wpart["leaf_begin"][l]:][:wpart["leaf_count"][l]])
        assert np.array_equal(a, b), l


def test_categorical_booster_bit_exact_and_predict():
    import lightgbm_rs_b200 as lgb
    import oracle

    X, y, cats = _mixed_data(seed=9)
    params = {"objective": "binary", "num_leaves": 31, "min_data_in_leaf": 20,
              "learning_rate": 0.1, "use_quantized_grad": True, "num_grad_quant_bins": 4,
              "min_data_per_group": 50, "cat_smooth": 5.0}
    ds = lgb.Dataset(X, y, params, categorical_feature=cats)
    metas = [{k: m[k] for k in ("num_bin", "default_bin", "most_freq_bin", "missing_type",
                                "bin_type")} for m in ds.mappers]
    booster = lgb.train(params, ds, num_boost_round=6)
    ref = oracle.train(ds.bins, metas, y, objective="binary", num_iterations=6,
                       learning_rate=0.1, num_leaves=31, use_quantized_grad=True,
                       stochastic_rounding=True,
                       num_grad_quant_bins=4, min_data_in_leaf=20, min_data_per_group=50,
                       cat_smooth=5.0)
    for i, (a, b) in enumerate(zip(booster.trees(), ref["trees"])):
        _assert_trees_bit_equal(a, b, f"cat booster tree {i}")
    s = booster.train_scores()
    assert s.view(np.uint64).tolist() == ref["scores"].view(np.uint64).tolist()
    p = booster.predict(X[:2000], raw_score=True)
    np.testing.assert_allclose(p, s[:2000], rtol=0, atol=1e-9)
