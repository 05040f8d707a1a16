"""Look-ahead partitions: the runner-up leaf of each pick is partitioned, with its child
histogram, on a second stream while the next control step runs, and that step takes the
finished partition when it picks the same leaf.

The look-ahead changes when work runs, never its result: trees and scores with the
look-ahead on must be bit-identical to the look-ahead off (LGBM_B200_LOOKAHEAD=0, read
when a booster is created) and, for quantized gradients, to the oracle. The counters of
a profiled iteration show that look-aheads ran and were used.
"""

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TREE_EXACT = ["split_feature", "threshold_bin", "decision_type", "left_child", "right_child",
              "leaf_count", "internal_count"]
TREE_BITS = ["leaf_value", "leaf_weight", "internal_value", "split_gain"]


def _assert_trees_bit_equal(got, want, tag):
    assert got["num_leaves"] == want["num_leaves"], tag
    for k in TREE_EXACT:
        assert np.asarray(got[k]).tolist() == np.asarray(want[k]).tolist(), (tag, k)
    for k in TREE_BITS:
        a = np.asarray(got[k])
        b = np.asarray(want[k]).astype(a.dtype)
        assert a.tobytes() == b.tobytes(), (tag, k)


@pytest.fixture(scope="module")
def data():
    import lightgbm_rs_b200 as lgb
    from lightgbm_rs_b200 import synthetic

    X, y = synthetic.binary_c0(num_data=200_000, seed=5)
    ds = lgb.Dataset(X, y, {"max_bin": 255, "min_data_in_leaf": 50})
    metas = [{k: m[k] for k in ("num_bin", "default_bin", "most_freq_bin", "missing_type",
                                "bin_type")} for m in ds.mappers]
    return X, y, ds, metas


def _train(ds, params, rounds, lookahead):
    import lightgbm_rs_b200 as lgb

    old = os.environ.get("LGBM_B200_LOOKAHEAD")
    os.environ["LGBM_B200_LOOKAHEAD"] = "1" if lookahead else "0"
    try:
        booster = lgb.train(params, ds, num_boost_round=rounds)
        _, counts = booster.profile_iteration()
    finally:
        if old is None:
            del os.environ["LGBM_B200_LOOKAHEAD"]
        else:
            os.environ["LGBM_B200_LOOKAHEAD"] = old
    return booster, counts


@pytest.mark.parametrize("num_leaves", [255, 31])
def test_lookahead_quantized_bit_exact(data, num_leaves):
    import oracle

    X, y, ds, metas = data
    params = {"objective": "binary", "num_leaves": num_leaves, "min_data_in_leaf": 50,
              "learning_rate": 0.1, "use_quantized_grad": True, "num_grad_quant_bins": 4}
    on, c_on = _train(ds, params, 4, True)
    off, c_off = _train(ds, params, 4, False)
    assert c_on["fused"]
    assert c_on["lookahead_runs"] > 0 and c_on["lookahead_hits"] > 0, c_on
    assert c_on["lookahead_hits"] <= c_on["lookahead_runs"]
    assert c_off["lookahead_runs"] == 0 and c_off["lookahead_hits"] == 0, c_off
    # both count the partitions whose result the tree used
    assert c_on["rows_parted"] == c_off["rows_parted"]
    assert c_on["builds"] == c_off["builds"] and c_on["rows_built"] == c_off["rows_built"]
    ref = oracle.train(ds.bins, metas, y, objective="binary", num_iterations=5,
                       learning_rate=0.1, num_leaves=num_leaves, use_quantized_grad=True,
                       stochastic_rounding=True,
                       num_grad_quant_bins=4, min_data_in_leaf=50, nthreads=8)
    a, b = on.trees(), off.trees()
    assert len(a) == len(b) == len(ref["trees"]) == 5
    for i in range(5):
        _assert_trees_bit_equal(a[i], ref["trees"][i], f"on vs oracle, tree {i}")
        _assert_trees_bit_equal(b[i], ref["trees"][i], f"off vs oracle, tree {i}")
    s_on, s_off = on.train_scores(), off.train_scores()
    assert s_on.tobytes() == s_off.tobytes() == ref["scores"].tobytes()


def test_lookahead_f32_identical(data):
    X, y, ds, metas = data
    params = {"objective": "binary", "num_leaves": 127, "min_data_in_leaf": 50,
              "learning_rate": 0.1}
    on, c_on = _train(ds, params, 3, True)
    off, _ = _train(ds, params, 3, False)
    assert c_on["fused"] and c_on["lookahead_hits"] > 0, c_on
    for i, (a, b) in enumerate(zip(on.trees(), off.trees())):
        _assert_trees_bit_equal(a, b, f"f32 tree {i}")
    assert on.train_scores().tobytes() == off.train_scores().tobytes()


def test_lookahead_learner_grow_partition(data):
    """The single-tree learner path (eager launches on two streams) gives the oracle's
    tree and leaf row sets."""
    import lightgbm_rs_b200 as lgb
    import oracle

    X, y, ds, metas = data
    init = oracle.boost_from_score("binary", y)
    rng = np.random.default_rng(3)
    score = init + rng.normal(0, 0.3, len(y))  # a mid-training score
    g, h = oracle.binary_gradients(score, y)
    gq, hq, q, scales = oracle.quantize(g, h, 4)
    want, wpart, _ = oracle.grow_tree(ds.bins, metas, gq, hq, num_leaves=255, nthreads=8,
                                      min_data_in_leaf=50)
    learner = lgb.Learner(ds, {"num_leaves": 255, "min_data_in_leaf": 50})
    got, gpart = learner.grow(quantized=q, scales=[scales[0], scales[1], scales[2], 4])
    _assert_trees_bit_equal(got, want, "learner grow")
    for l in range(got["num_leaves"]):
        a = np.sort(gpart["indices"][gpart["leaf_begin"][l]:][:gpart["leaf_count"][l]])
        b = np.sort(wpart["indices"][wpart["leaf_begin"][l]:][:wpart["leaf_count"][l]])
        assert np.array_equal(a, b), l


def _train_env(ds, params, rounds, env):
    import lightgbm_rs_b200 as lgb

    old = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    try:
        booster = lgb.train(params, ds, num_boost_round=rounds)
        _, pc = booster.profile_pipeline(1)
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    return booster, pc


@pytest.mark.parametrize("env", [
    {"LGBM_B200_FUSE_MAIN": "0"},   # the main partition as its own launch
    {"LGBM_B200_LA_CANCEL": "0"},   # missed look-aheads run to the end
    {"LGBM_B200_WARM_PICK": "0"},   # no placeholder picks
    {"LGBM_B200_LA_BLOCKS": "120", "LGBM_B200_MAIN_LATE_BLOCKS": "148"},
])
def test_split_step_variants_same_trees(data, env):
    """The launch-shape variants of the split step (the main partition inside the next
    control step or its own launch, cancelled or finished look-aheads, the pick's
    instruction-cache warm-up, grid sizes) change when work runs, never its result: the
    same trees and scores, bit for bit. The default run's main partitions ran inside the
    control steps (their rows are counted there); with LGBM_B200_FUSE_MAIN=0 none did."""
    X, y, ds, metas = data
    params = {"objective": "binary", "num_leaves": 255, "min_data_in_leaf": 50,
              "learning_rate": 0.1, "use_quantized_grad": True, "num_grad_quant_bins": 4}
    base, pc_base = _train_env(ds, params, 3, {})
    var, pc_var = _train_env(ds, params, 3, env)
    assert pc_base["fused"] and pc_base["rows_parted_ctl"] > 0, pc_base
    if env.get("LGBM_B200_FUSE_MAIN") == "0":
        assert pc_var["rows_parted_ctl"] == 0, pc_var
    for i, (a, b) in enumerate(zip(base.trees(), var.trees())):
        _assert_trees_bit_equal(b, a, f"{env} tree {i}")
    assert base.train_scores().tobytes() == var.train_scores().tobytes()
