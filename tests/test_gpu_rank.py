"""Lambdarank on the device (k_lambdarank + the usual tree path).

Pinned to lib_lightgbm 4.6 through the reference's rank fixtures (iteration-1 gradients,
the 10-tree model, the final raw scores; oracle-harness rank/), and to the oracle on
random ranking corpora: gradients every iteration bit-exact, quantized trees and scores
bit-exact. Query shapes cover empty queries, single-row queries, queries longer than a
warp, equal labels, truncation levels below and above the query size, and norm off.
"""

import numpy as np
import pytest

import _golden as G

pytestmark = pytest.mark.gpu

RANK_BIN = dict(max_bin=255, min_data_in_bin=1, min_data_in_leaf=1, pre_filter=False,
                bin_construct_sample_cnt=1_000_000)


def _golden_dataset():
    import lightgbm_rs_b200 as lgb

    X, labels, qb, G1, H1, final = G.rank_case()
    mappers, cols = [], []
    for j in range(X.shape[1]):
        m, b = lgb.bin_column(X[:, j], **RANK_BIN)
        mappers.append(m)
        cols.append(b.astype(np.uint8))
    ds = lgb.Dataset(bins=np.stack(cols), mappers=mappers, label=labels,
                     params={"min_data_in_leaf": 1}, group=np.diff(qb))
    return ds, labels, qb, G1, H1, final


GOLDEN_PARAMS = {"objective": "lambdarank", "num_leaves": 7, "learning_rate": 0.1,
                 "min_data_in_leaf": 1, "min_sum_hessian_in_leaf": 1e-3,
                 "lambdarank_truncation_level": 5, "lambdarank_norm": True}


def test_lambdarank_golden_gradients_and_model():
    import lightgbm_rs_b200 as lgb

    ds, labels, qb, G1, H1, final = _golden_dataset()
    b = lgb.Booster(GOLDEN_PARAMS, ds)
    assert b.init_score() == 0.0  # ranking objectives have no boost-from-average score
    b.update(1)
    g, h = b.last_gradients()
    assert g.view(np.uint32).tolist() == G1.view(np.uint32).tolist()
    assert h.view(np.uint32).tolist() == H1.view(np.uint32).tolist()
    b.update(9)
    model = G.parse_model_text(G.read_text("rank_lambdarank_byq0_es0_model.txt"))
    trees = b.trees()
    assert len(trees) == len(model) == 10
    for i, (t, m) in enumerate(zip(trees, model)):
        for k in ("split_feature", "left_child", "right_child", "leaf_count",
                  "internal_count"):
            assert t[k].tolist() == m[k].tolist(), (i, k)
        assert [G.g17(x) for x in t["leaf_value"]] == [G.g17(x) for x in m["leaf_value"]], i
    assert b.train_scores().view(np.uint64).tolist() == final.view(np.uint64).tolist()


def _corpus(num_queries, mean, max_size, num_features, seed, with_empty=True):
    rng = np.random.default_rng(seed)
    sizes = np.clip(rng.poisson(mean, num_queries), 1, max_size)
    if with_empty:
        sizes[::97] = 0     # empty queries
        sizes[1::89] = 1    # single-row queries
    n = int(sizes.sum())
    X = np.where(rng.random((n, num_features)) < 0.8, 0.0,
                 rng.exponential(1.0, (n, num_features)))
    w = rng.normal(0, 1, num_features)
    z = X @ w + rng.normal(0, 0.5, n)
    cuts = np.quantile(z, [0.5, 0.75, 0.9, 0.97])
    y = np.searchsorted(cuts, z).astype(np.float32)
    qb = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    for q in range(0, num_queries, 53):  # some queries with one label only
        y[qb[q]:qb[q + 1]] = 2.0
    return X, y, sizes, qb


def _dataset(X, y, sizes):
    import lightgbm_rs_b200 as lgb

    ds = lgb.Dataset(X, y, {"max_bin": 255, "min_data_in_leaf": 20}, group=sizes)
    metas = [{k: m[k] for k in ("num_bin", "default_bin", "most_freq_bin", "missing_type")}
             for m in ds.mappers]
    return ds, metas


@pytest.mark.parametrize("trunc,norm,mean,max_size", [(30, True, 23, 200), (1, True, 10, 40),
                                                      (500, False, 60, 300),
                                                      (20, True, 150, 1000)])
def test_lambdarank_gradients_every_iteration_bit_exact(trunc, norm, mean, max_size):
    import lightgbm_rs_b200 as lgb
    import oracle

    X, y, sizes, qb = _corpus(400, mean, max_size, 12, seed=trunc + max_size)
    ds, _ = _dataset(X, y, sizes)
    p = {"objective": "lambdarank", "num_leaves": 31, "min_data_in_leaf": 20,
         "lambdarank_truncation_level": trunc, "lambdarank_norm": norm,
         "use_quantized_grad": True, "num_grad_quant_bins": 4}
    b = lgb.Booster(p, ds)
    for it in range(4):
        s = b.train_scores()
        b.update(1)
        g, h = b.last_gradients()
        og, oh = oracle.lambdarank_gradients(s, y, qb, 1.0, norm, trunc)
        assert g.view(np.uint32).tolist() == og.view(np.uint32).tolist(), it
        assert h.view(np.uint32).tolist() == oh.view(np.uint32).tolist(), it


def test_lambdarank_quantized_booster_bit_exact_vs_oracle():
    import lightgbm_rs_b200 as lgb
    import oracle

    X, y, sizes, qb = _corpus(1500, 23, 200, 20, seed=3)
    ds, metas = _dataset(X, y, sizes)
    p = {"objective": "lambdarank", "num_leaves": 63, "min_data_in_leaf": 20,
         "use_quantized_grad": True, "num_grad_quant_bins": 4, "learning_rate": 0.1}
    b = lgb.train(p, ds, num_boost_round=8)
    ref = oracle.train(ds.bins, metas, y, objective="lambdarank", num_iterations=8,
                       learning_rate=0.1, num_leaves=63, use_quantized_grad=True,
                       stochastic_rounding=True,
                       num_grad_quant_bins=4, query_boundaries=qb, min_data_in_leaf=20)
    assert len(b.trees()) == len(ref["trees"])
    for i, (a, r) in enumerate(zip(b.trees(), ref["trees"])):
        assert a["num_leaves"] == r["num_leaves"], i
        for k in ("split_feature", "threshold_bin", "decision_type", "left_child",
                  "right_child", "leaf_count"):
            assert a[k].tolist() == r[k].tolist(), (i, k)
        assert a["leaf_value"].tobytes() == r["leaf_value"].tobytes(), i
    assert b.train_scores().view(np.uint64).tolist() == ref["scores"].view(np.uint64).tolist()


def test_lambdarank_rejects_bad_queries():
    import lightgbm_rs_b200 as lgb

    X, y, sizes, qb = _corpus(50, 10, 30, 4, seed=1, with_empty=False)
    ds, _ = _dataset(X, y, sizes[:-1])  # sizes no longer cover every row
    with pytest.raises(lgb.LightGBMError):
        lgb.Booster({"objective": "lambdarank"}, ds)
    y2 = y.copy()
    y2[3] = 0.5  # not an integer label
    ds2, _ = _dataset(X, y2, sizes)
    with pytest.raises(lgb.LightGBMError):
        lgb.Booster({"objective": "lambdarank"}, ds2)
    ds3, _ = _dataset(X, y, None)
    with pytest.raises(lgb.LightGBMError):
        lgb.Booster({"objective": "lambdarank"}, ds3)
