"""Batch prediction on the device and the model-text writer of trained boosters.

The predictor is pinned to lib_lightgbm's own predictions on its own model files
(predict_modes numeric and categorical, the binary spine model, the rank model), to the
oracle's tree walk on adversarial inputs (NaN, zeros, negative and unseen categories,
huge values) for every golden model, and to the boosters' own training scores. The writer
reproduces lib_lightgbm's lambdarank model file byte for byte up to its parameters block.
"""

import numpy as np
import pytest

import _golden as G
from test_model_text import check_prediction, prediction_cases

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", prediction_cases(), ids=lambda c: c[0])
def test_device_prediction_real_lightgbm(case):
    import lightgbm_rs_b200 as lgb

    _, fname, X, expected, kind = case
    b = lgb.Booster(model_str=G.read_text(fname))
    raw = b.predict(X, raw_score=True)
    check_prediction(kind, raw, expected, b.predict(X))


def _adversarial_rows(nf, n, seed):
    rng = np.random.default_rng(seed)
    X = rng.normal(0, 3, (n, nf))
    X[rng.random((n, nf)) < 0.1] = np.nan
    X[rng.random((n, nf)) < 0.1] = 0.0
    X[rng.random((n, nf)) < 0.05] = -0.0
    ints = rng.random((n, nf)) < 0.3
    X[ints] = rng.integers(-2, 70, int(ints.sum()))
    X[rng.random((n, nf)) < 0.01] = 1e300
    X[rng.random((n, nf)) < 0.01] = 1e-36
    return X


@pytest.mark.parametrize("name", G.MODEL_TEXTS)
def test_device_prediction_matches_oracle(name):
    import lightgbm_rs_b200 as lgb
    import oracle
    from lightgbm_rs_b200 import model_text as MT

    model = MT.parse(G.read_text(name))
    X = _adversarial_rows(model.max_feature_idx + 1, 20000, seed=len(name))
    b = lgb.Booster(model_str=G.read_text(name))
    got = b.predict(X, raw_score=True)
    want = oracle.predict_raw(MT.flatten(model), X)
    assert got.view(np.uint64).tolist() == want.view(np.uint64).tolist()


def test_writer_reproduces_lightgbm_rank_model():
    """The device-trained lambdarank booster on the rank corpus, written as model text,
    equals lib_lightgbm's file up to its parameters block (header, feature_infos,
    tree_sizes, every tree block, feature importances)."""
    import lightgbm_rs_b200 as lgb
    from test_gpu_rank import GOLDEN_PARAMS, _golden_dataset

    ds, *_ = _golden_dataset()
    b = lgb.Booster(GOLDEN_PARAMS, ds)
    b.update(10)
    text = b.model_to_string()
    gold = _with_reference_zero_threshold(G.read_text("rank_lambdarank_byq0_es0_model.txt"))
    cut = gold.index("\nparameters:\n")
    assert text[:cut] == gold[:cut]


def _with_reference_zero_threshold(text):
    """lib_lightgbm's kZeroThreshold is the float 1e-35f, so the bin bound next to zero
    prints as 1.0000000180025095e-35; the reference's BinMapper (and its binning goldens,
    lgbm-core/src/types.rs:35) uses the double 1e-35, and so do this library's bins.
    Swap that one constant in lib_lightgbm's file and re-dump it (tree_sizes follow)."""
    from lightgbm_rs_b200 import model_text as MT

    m = MT.parse(text)
    f32 = float(np.float32(1e-35))
    for t in m.trees:
        thr = t["threshold"]
        thr[thr == f32] = 1e-35
        thr[thr == -f32] = -1e-35
    return MT.dump(m)


def test_trained_booster_predicts_its_training_scores(tmp_path):
    """predict() on the raw training rows (real thresholds, real category bitsets, the
    init score in the first tree) equals the training scores (bin routing) bit for bit,
    also after a save / load round trip."""
    import lightgbm_rs_b200 as lgb
    from test_gpu_categorical import _mixed_data

    X, y, cats = _mixed_data(n=20000, seed=4)
    X[np.random.default_rng(1).random(X.shape) < 0.05] = np.nan
    params = {"objective": "binary", "num_leaves": 31, "min_data_in_leaf": 20,
              "use_quantized_grad": True, "num_grad_quant_bins": 4}
    ds = lgb.Dataset(X, y, params, categorical_feature=cats)
    b = lgb.train(params, ds, num_boost_round=8)
    s = b.train_scores()
    p = b.predict(X, raw_score=True)
    assert p.view(np.uint64).tolist() == s.view(np.uint64).tolist()
    path = tmp_path / "model.txt"
    b.save_model(str(path))
    b2 = lgb.Booster(model_file=str(path))
    assert b2.predict(X, raw_score=True).view(np.uint64).tolist() == s.view(np.uint64).tolist()
    np.testing.assert_allclose(b2.predict(X), 1.0 / (1.0 + np.exp(-s)), rtol=1e-15, atol=0)
