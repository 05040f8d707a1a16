"""Pin the CPU restatement (oracle/) against the reference's golden vectors.

Mirrors the reference's own replay tests:
crates/oracle-harness/tests/kernel_parity.rs (histogram :162, split :512,
partition :1162, subtract :1276) and learner_parity.rs (:1200, :1301).
"""

import numpy as np
import pytest

import _golden as G


def test_histogram_golden_bit_exact(oracle_lib):
    cases = G.histogram_cases()
    assert len(cases) == 18
    for c in cases:
        got = oracle_lib.construct_histogram(c["bins"], c["grad"], c["hess"], c["num_bin"])
        assert got.view(np.uint64).tolist() == c["hist"].view(np.uint64).tolist(), c["name"]


def test_split_golden_bit_exact(oracle_lib):
    cases = G.split_cases()
    assert cases
    for c in cases:
        cfg = oracle_lib.gain_config(
            min_data_in_leaf=c["min_data_in_leaf"],
            min_sum_hessian_in_leaf=c["min_sum_hessian_in_leaf"],
            lambda_l1=c["lambda_l1"], lambda_l2=c["lambda_l2"],
            min_gain_to_split=c["min_gain_to_split"])
        s = oracle_lib.find_best_split(c["hist"], cfg, c["num_bin"], c["offset"],
                                       c["default_bin"], c["skip_default_bin"],
                                       c["na_as_missing"], True, c["sum_gradient"],
                                       c["sum_hessian"], c["num_data"])
        w = c["win"]
        assert (s.gain != -np.inf) == w["is_splittable"], c["name"]
        if not w["is_splittable"]:
            continue
        for k in ("gain", "left_sum_gradient", "left_sum_hessian", "right_sum_gradient",
                  "right_sum_hessian", "left_output", "right_output"):
            assert G.bits_of_f64(getattr(s, k)) == w[k], (c["name"], k)
        assert s.threshold == w["threshold"], c["name"]
        assert s.left_count == w["left_count"] and s.right_count == w["right_count"], c["name"]
        assert bool(s.default_left) == w["default_left"], c["name"]


def test_subtract_golden_bit_exact(oracle_lib):
    for c in G.subtract_cases():
        got = oracle_lib.subtract(c["subparent"], c["subchild"])
        assert got.view(np.uint64).tolist() == c["subderived"].view(np.uint64).tolist()


def test_partition_golden_exact(oracle_lib):
    n = 0
    for c in G.partition_cases():
        if c["missing_type"] != 0:
            continue  # the reference replays missing_type == 0 only (kernel_parity.rs:1196)
        rows = np.arange(len(c["bins"]), dtype=np.uint32)
        order, left = oracle_lib.partition(c["bins"], rows, c["num_bin"], c["min_bin"],
                                           c["max_bin"], c["threshold"], c["most_freq_bin"])
        assert order.tolist() == c["order"].tolist(), c["name"]
        assert left == c["split"], c["name"]
        n += 1
    assert n >= 4


def _real_upper_bounds(num_bin, mfb_zero_sentinel=False):
    b = [np.nextafter(np.float64(i) + 0.5, np.inf) for i in range(num_bin)]
    if mfb_zero_sentinel:
        b[0] = float(np.float32(1e-35))
    return b


def _assert_real_tree(tree, golden, upper, shrinkage):
    nl = golden["num_leaves"]
    assert tree["num_leaves"] == nl
    assert tree["split_feature"].tolist() == golden["split_feature"].tolist()
    assert tree["decision_type"].tolist() == golden["decision_type"].tolist()
    assert tree["left_child"].tolist() == golden["left_child"].tolist()
    assert tree["right_child"].tolist() == golden["right_child"].tolist()
    assert tree["leaf_count"].tolist() == golden["leaf_count"].tolist()
    assert tree["internal_count"].tolist() == golden["internal_count"].tolist()
    thr = [G.g17(upper[b]) for b in tree["threshold_bin"]]
    assert thr == [G.g17(x) for x in golden["threshold"]]
    lv = tree["leaf_value"] * shrinkage
    lv = np.where(np.abs(lv) <= float(np.float32(1e-35)), 0.0, lv)
    assert [G.g17(x) for x in lv] == [G.g17(x) for x in golden["leaf_value"]]


@pytest.mark.parametrize("name,bins,grad", [
    ("spine_real.txt", [0, 0, 1, 1, 2, 2, 3, 3, 4, 4, 5, 5],
     [-6, -6, -5, -5, -1, -1, 1, 1, 5, 5, 6, 6]),
    ("mfb_pos_real.txt", [0, 1, 2, 2, 2, 2, 2, 2, 3, 3, 1, 0],
     [-6, -3, -1, -1, -1, 1, 1, 1, 4, 5, -3, -6]),
])
def test_learner_real_lightgbm_tree(oracle_lib, name, bins, grad):
    """learner_parity.rs:1200 / :1301 — one tree vs a real lib_lightgbm 4.6 tree."""
    golden = G.parse_model_text(G.read_text(name))
    assert len(golden) == 1
    num_bin = max(bins) + 1
    bins = np.array([bins], dtype=np.uint32)
    meta = [{"num_bin": num_bin, "default_bin": num_bin, "most_freq_bin": 0, "missing_type": 0}]
    g = np.array(grad, dtype=np.float32)
    h = np.ones_like(g)
    tree, part, _ = oracle_lib.grow_tree(bins, meta, g, h, num_leaves=4, max_depth=-1,
                                         min_data_in_leaf=1, min_sum_hessian_in_leaf=1e-3)
    upper = _real_upper_bounds(num_bin, mfb_zero_sentinel=(name == "mfb_pos_real.txt"))
    _assert_real_tree(tree, golden[0], upper, 0.1)
    # routing self-consistency: partition leaf counts equal tree leaf counts
    assert part["leaf_count"].tolist() == tree["leaf_count"].tolist()


def test_binary_gradients_and_scores_golden(oracle_lib):
    """boosting_parity.rs binary cell: 12 rows, 2 features, 10 iters, num_leaves 4.

    The corpus is identity-binned (bin == raw value, boosting_parity.rs:44-66), so the
    learner sees bins f0 in 0..5 and f1 in 0..2 with most_freq_bin 0."""
    f0 = [0, 0, 1, 1, 2, 2, 3, 3, 4, 4, 5, 5]
    f1 = [0, 1, 2, 0, 1, 2, 0, 1, 2, 0, 1, 2]
    labels = np.array([0, 0, 0, 0, 0, 1, 0, 1, 1, 0, 1, 1], dtype=np.float32)
    bins = np.array([f0, f1], dtype=np.uint32)
    metas = [{"num_bin": 6, "default_bin": 0, "most_freq_bin": 0, "missing_type": 0},
             {"num_bin": 3, "default_bin": 0, "most_freq_bin": 0, "missing_type": 0}]
    out = oracle_lib.train(bins, metas, labels, objective="binary", num_iterations=10,
                           learning_rate=0.1, num_leaves=4, min_data_in_leaf=1,
                           min_sum_hessian_in_leaf=1e-3, record=True)
    lines = G.data_lines("binary_scores.txt")
    assert len(lines) == len(out["iter_scores"]) == 10
    for k, line in enumerate(lines):
        want = G.bits_line(line)
        got = out["iter_scores"][k]
        assert got.view(np.uint64).tolist() == want.view(np.uint64).tolist(), f"iter {k + 1}"
    gh = G.data_lines("binary_gh_iter1.txt")
    g_want = G.bits_line(gh[0].split(None, 1)[1], "f32")
    h_want = G.bits_line(gh[1].split(None, 1)[1], "f32")
    g_got, h_got = out["iter_grad_hess"][0]
    np.testing.assert_allclose(g_got, g_want, atol=1e-6)
    np.testing.assert_allclose(h_got, h_want, atol=1e-6)
    # per-tree leaf values vs the lightgbm model text (boosting_parity.rs:205-236)
    model = G.parse_model_text(G.read_text("binary_spine_model.txt"))
    assert len(model) == len(out["trees"])
    for i, (t, m) in enumerate(zip(out["trees"], model)):
        lv = t["leaf_value"].copy()
        if "bias" in t:
            lv = lv + t["bias"]
        assert [G.g17(x) for x in lv] == [G.g17(x) for x in m["leaf_value"]], f"tree {i}"


@pytest.mark.parametrize("name", ["cat_onehot", "cat_manyvsmany"])
def test_categorical_learner_real_lightgbm_tree(oracle_lib, name):
    """oracle-harness learner_parity.rs:1486-1535 categorical cells: one categorical feature,
    hessian 1, grown by the oracle, against the tree lib_lightgbm 4.6 grew (one-hot and
    sorted many-vs-many splits, the categorical decision bit, cat_boundaries, and the real
    category bitset cat_threshold)."""
    import json

    import oracle

    side = json.loads(G.read_text(f"{name}.bins.json"))
    gold = G.parse_model_text(G.read_text(f"{name}.txt"))[0]
    gold_raw = dict(l.split("=", 1) for l in G.read_text(f"{name}.txt").splitlines()
                    if "=" in l and l.split("=", 1)[0] in ("cat_boundaries", "cat_threshold",
                                                            "num_cat"))
    bins = np.array(side["bins"], dtype=np.uint32).reshape(1, -1)
    nb, mfb = int(side["num_bin"]), int(side["most_freq_bin"])
    metas = [{"num_bin": nb, "default_bin": nb, "most_freq_bin": mfb, "missing_type": 0,
              "bin_type": 1}]
    g = np.array(side["grad"], dtype=np.float32)
    h = np.ones_like(g)
    tree, _, _ = oracle.grow_tree(bins, metas, g, h, num_leaves=int(side["num_leaves"]),
                                  min_data_in_leaf=1, min_sum_hessian_in_leaf=1e-3,
                                  cat_l2=side["cat_l2"], cat_smooth=side["cat_smooth"],
                                  min_data_per_group=int(side["min_data_per_group"]),
                                  max_cat_threshold=int(side["max_cat_threshold"]),
                                  max_cat_to_onehot=int(side["max_cat_to_onehot"]))
    assert tree["num_leaves"] == gold["num_leaves"]
    for k in ("split_feature", "decision_type", "left_child", "right_child", "leaf_count",
              "internal_count"):
        assert tree[k].tolist() == gold[k].tolist(), k
    assert [G.g17(float(t)) for t in tree["threshold_bin"]] == \
        [G.g17(t) for t in gold["threshold"]]
    b2c = side["bin_2_categorical"]
    bounds, words = oracle.categorical_bitsets(tree, lambda f: b2c)
    assert len(bounds) - 1 == int(gold_raw["num_cat"])
    assert bounds == [int(x) for x in gold_raw["cat_boundaries"].split()]
    assert words == [int(x) for x in gold_raw["cat_threshold"].split()]
    shrink = float(side.get("shrinkage", 0.1))
    lv = [0.0 if abs(v * shrink) <= 1e-35 else v * shrink for v in tree["leaf_value"]]
    assert [G.g17(v) for v in lv] == [G.g17(v) for v in gold["leaf_value"]]


RANK_PARAMS = dict(max_bin=255, min_data_in_bin=1, min_data_in_leaf=1, pre_filter=False,
                   bin_construct_sample_cnt=1_000_000)


def test_lambdarank_gradients_real_lightgbm(oracle_lib):
    """rank/lambdarank_gh_iter1.txt: lib_lightgbm 4.6's iteration-1 lambdas and hessians
    (zero scores, sigmoid 1, lambdarank_norm, truncation level 5), bit-exact."""
    import oracle

    _, labels, qb, G1, H1, _ = G.rank_case()
    g, h = oracle.lambdarank_gradients(np.zeros(len(labels)), labels, qb, 1.0, True, 5)
    assert g.view(np.uint32).tolist() == G1.view(np.uint32).tolist()
    assert h.view(np.uint32).tolist() == H1.view(np.uint32).tolist()


def test_lambdarank_training_real_lightgbm(oracle_lib):
    """rank_lambdarank_byq0_es0_model.txt + lambdarank_scores.txt: 10 lambdarank
    iterations (7 leaves, f32 gradients) replayed by the oracle: every tree's structure
    and %.17g leaf values, and the final raw scores bit-exact."""
    import lightgbm_rs_b200 as lgb
    import oracle

    X, labels, qb, _, _, final = G.rank_case()
    mappers, cols = [], []
    for j in range(X.shape[1]):
        m, b = lgb.bin_column(X[:, j], **RANK_PARAMS)
        mappers.append(m)
        cols.append(b.astype(np.uint8))
    metas = [{k: m[k] for k in ("num_bin", "default_bin", "most_freq_bin", "missing_type")}
             for m in mappers]
    out = oracle.train(np.stack(cols), metas, labels, objective="lambdarank",
                       num_iterations=10, learning_rate=0.1, num_leaves=7,
                       query_boundaries=qb, lambdarank_truncation_level=5,
                       min_data_in_leaf=1, min_sum_hessian_in_leaf=1e-3)
    model = G.parse_model_text(G.read_text("rank_lambdarank_byq0_es0_model.txt"))
    assert len(out["trees"]) == len(model) == 10
    for i, (t, m) in enumerate(zip(out["trees"], model)):
        for k in ("split_feature", "left_child", "right_child", "leaf_count",
                  "internal_count"):
            assert t[k].tolist() == m[k].tolist(), (i, k)
        assert [G.g17(x) for x in t["leaf_value"]] == [G.g17(x) for x in m["leaf_value"]], i
    assert out["scores"].view(np.uint64).tolist() == final.view(np.uint64).tolist()


def test_oracle_numeric_binning_golden_bit_exact(oracle_lib):
    """The oracle's own BinMapper restatement (oracle/bin_mapper.cpp) replays the
    reference's 45 numeric binning goldens (crates/lgbm-dataset/tests/golden/)."""
    cases = G.binning_cases()
    assert len(cases) == 45
    for c in cases:
        m, bins = oracle_lib.bin_column(c["values"], max_bin=c["max_bin"],
                                        min_data_in_bin=c["min_data_in_bin"],
                                        min_data_in_leaf=c["min_split_data"],
                                        pre_filter=c["pre_filter"], use_missing=c["use_missing"],
                                        zero_as_missing=c["zero_as_missing"],
                                        bin_construct_sample_cnt=c["sample_cnt"],
                                        data_random_seed=c["seed"])
        gold = c["golden"]
        for k in ("num_bin", "missing_type", "default_bin", "most_freq_bin", "is_trivial"):
            assert m[k] == gold[k], (c["name"], k)
        gn, wn = np.isnan(m["upper"]), np.isnan(gold["upper"])
        assert gn.tolist() == wn.tolist(), c["name"]
        assert m["upper"].view(np.uint64)[~gn].tolist() == \
            gold["upper"].view(np.uint64)[~wn].tolist(), c["name"]
        assert bins.tolist() == c["assign"].tolist(), c["name"]


def test_oracle_categorical_binning_golden(oracle_lib):
    """categorical_folding.txt through the oracle's BinMapper restatement."""
    cases = G.categorical_binning_cases()
    assert len(cases) == 6
    for c in cases:
        m, bins = oracle_lib.bin_column(c["values"], max_bin=c["max_bin"],
                                        min_data_in_bin=c["min_data_in_bin"],
                                        min_data_in_leaf=c["min_split_data"],
                                        pre_filter=c["pre_filter"], use_missing=c["use_missing"],
                                        zero_as_missing=c["zero_as_missing"],
                                        bin_construct_sample_cnt=max(len(c["values"]), 1),
                                        categorical=True)
        gm = c["mapper"]
        for k in ("num_bin", "missing_type", "default_bin", "most_freq_bin"):
            assert m[k] == gm[k], (c["name"], k)
        assert m["is_trivial"] == bool(gm["is_trivial"]), c["name"]
        assert m["bin_to_category"].tolist() == c["b2c"], c["name"]
        assert bins.tolist() == c["assign"].tolist(), c["name"]


@pytest.mark.parametrize("kind", ["normal", "skewed_nan", "categorical", "sparse"])
def test_oracle_binning_equals_product_binning(oracle_lib, kind):
    """The product's host binning and the oracle's restatement agree on sampled
    columns larger than the sample (200k of 400k rows), including NaN, zero-heavy and
    categorical columns like those of the bench workloads."""
    import lightgbm_rs_b200 as lgb

    r = np.random.default_rng(hash(kind) % 2**32)
    n = 400_000
    cat = False
    if kind == "normal":
        x = r.normal(size=n)
    elif kind == "skewed_nan":
        x = np.exp(r.normal(size=n))
        x[r.random(n) < 0.1] = np.nan
    elif kind == "categorical":
        x = np.minimum(r.zipf(1.2, n), 900).astype(np.float64)
        cat = True
    else:
        x = np.where(r.random(n) < 0.8, 0.0, r.exponential(size=n))
    for max_bin, min_leaf in ((255, 20), (63, 100)):
        kw = dict(max_bin=max_bin, min_data_in_leaf=min_leaf, categorical=cat)
        mo, bo = oracle_lib.bin_column(x, **kw)
        mp, bp = lgb.bin_column(x, **kw)
        for k in ("num_bin", "missing_type", "default_bin", "most_freq_bin", "is_trivial"):
            assert mo[k] == mp[k], (kind, k)
        key = "bin_to_category" if cat else "upper"
        assert np.array_equal(mo[key], mp[key], equal_nan=not cat), kind
        assert np.array_equal(bo, bp), kind


def test_partition_golden_missing_fanout(oracle_lib):
    """Every partition.txt case, the six missing_type != 0 ones included, through the
    oracle's restatement of the kernel router with its whole missing-value fan-out
    (crates/oracle-harness/tests/partition_parity.rs:112-190 replays them the same way)."""
    cases = G.partition_cases()
    missing = 0
    for c in cases:
        rows = np.arange(len(c["bins"]), dtype=np.uint32)
        order, left = oracle_lib.partition_missing(c["bins"], rows, c["min_bin"], c["max_bin"],
                                                   c["threshold"], c["most_freq_bin"],
                                                   c["default_bin"], c["missing_type"],
                                                   c["default_left"])
        assert order.tolist() == c["order"].tolist(), c["name"]
        assert left == c["split"], c["name"]
        missing += c["missing_type"] != 0
    assert missing == 6


def _xorshift_offsets(seed, count):
    """Pure-Python restatement of the reference's next_u01 stream
    (lgbm-treelearner/src/gradient_discretizer.rs:252-262), seeded as new_stochastic
    (:78-83) does: state = seed ^ 0x9E3779B97F4A7C15."""
    m = (1 << 64) - 1
    x = (seed ^ 0x9E3779B97F4A7C15) & m
    out = []
    for _ in range(count):
        x ^= (x << 13) & m
        x ^= x >> 7
        x ^= (x << 17) & m
        out.append((x >> 11) / float(1 << 53))
    return out


def test_oracle_stochastic_rounding_matches_python_restatement(oracle_lib):
    """Each row draws the gradient offset then the hessian offset; q = trunc(v * inv +-
    offset) (gradient_discretizer.rs:167-191). The C++ oracle against a Python loop."""
    rng = np.random.default_rng(3)
    n = 3000
    g = rng.normal(size=n).astype(np.float32)
    h = rng.uniform(0.01, 0.25, n).astype(np.float32)
    seed = oracle_lib.stochastic_seed(5)
    assert seed == (5 << 20) ^ 0x51702010
    _, _, q, scales = oracle_lib.quantize(g, h, 4, stochastic=True, seed=seed)
    off = _xorshift_offsets(seed, 2 * n)
    igs, ihs = 1.0 / scales[0], 1.0 / scales[1]
    want_g = [int(np.trunc(float(g[i]) * igs + (off[2 * i] if g[i] >= 0 else -off[2 * i])))
              for i in range(n)]
    want_h = [int(np.trunc(float(h[i]) * ihs + off[2 * i + 1])) for i in range(n)]
    assert q[:, 0].tolist() == want_g
    assert q[:, 1].tolist() == want_h


def test_oracle_stochastic_rounding_properties(oracle_lib):
    """The reference's own property tests (gradient_discretizer.rs:337-374): reproducible
    per seed, different for another seed, and unbiased where deterministic rounding is
    biased to the grid point."""
    grad = ((np.arange(200) - 100.0) * 0.013).astype(np.float32)
    hess = np.ones(200, dtype=np.float32)
    a = oracle_lib.quantize(grad, hess, 16, stochastic=True, seed=42)[2]
    b = oracle_lib.quantize(grad, hess, 16, stochastic=True, seed=42)[2]
    c = oracle_lib.quantize(grad, hess, 16, stochastic=True, seed=43)[2]
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    n = 20_002
    grad = np.full(n, 0.3, dtype=np.float32)
    grad[0], grad[1] = 1.0, -1.0
    hess = np.ones(n, dtype=np.float32)
    _, _, qd, sd = oracle_lib.quantize(grad, hess, 4)
    _, _, qs, ss = oracle_lib.quantize(grad, hess, 4, stochastic=True, seed=7)
    det_mean = qd[2:, 0].astype(np.int64).sum() * sd[0] / (n - 2)
    sto_mean = qs[2:, 0].astype(np.int64).sum() * ss[0] / (n - 2)
    assert abs(det_mean - 0.5) < 1e-9
    assert abs(sto_mean - 0.3) < 0.01
