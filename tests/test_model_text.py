"""LightGBM model text: the writer and reader against lib_lightgbm's own files, and the
oracle's prediction walk against lib_lightgbm's predictions (CPU only).

Goldens: oracle-harness predict_modes/{numeric,categorical} (model, X, the raw margins of
the early-stop cells and the per-feature contributions whose row sums are the raw
margins), boosting/binary_spine_{model,pred}, rank/ and the categorical, NaN and
regression models, all written by lib_lightgbm 4.6.
"""

import numpy as np
import pytest

import _golden as G


@pytest.mark.parametrize("name", G.MODEL_TEXTS)
def test_model_text_round_trip_byte_exact(name):
    """parse then dump reproduces lib_lightgbm's file byte for byte: header, tree_sizes,
    every tree block's number formats, feature importances, the parameters tail."""
    from lightgbm_rs_b200 import model_text as MT

    text = G.read_text(name)
    assert MT.dump(MT.parse(text)) == text


def _spine_rows():
    f0 = [0, 0, 1, 1, 2, 2, 3, 3, 4, 4, 5, 5]
    f1 = [0, 1, 2, 0, 1, 2, 0, 1, 2, 0, 1, 2]
    return np.array([f0, f1], dtype=np.float64).T


def prediction_cases():
    """(name, model file, X, expected, kind) with kind "raw" (exact raw margins),
    "sigmoid" (transformed predictions) or "contrib" (rows of contributions whose sums
    are the raw margins)."""
    cases = []
    Xn = G.bits_matrix("predict_numeric_X.txt")
    full = [c for c in G.early_stop_cells("predict_numeric_early_stop.txt")]
    cases.append(("numeric", "predict_numeric_model.txt", Xn, full[-1]["values"], "raw"))
    cases.append(("numeric_contrib", "predict_numeric_model.txt", Xn,
                  G.bits_matrix("predict_numeric_contrib.txt"), "contrib"))
    Xc = G.bits_matrix("predict_categorical_X.txt")
    cases.append(("categorical", "predict_categorical_model.txt", Xc,
                  G.bits_matrix("predict_categorical_contrib.txt"), "contrib"))
    pred = G.bits_line(G.data_lines("binary_spine_pred.txt")[0])
    cases.append(("binary_spine", "binary_spine_model.txt", _spine_rows(), pred, "sigmoid"))
    X, _, _, _, _, final = G.rank_case()
    cases.append(("rank", "rank_lambdarank_byq0_es0_model.txt", X, final, "raw"))
    return cases


def check_prediction(kind, raw, expected, sigmoid_out=None):
    if kind == "raw":
        assert raw.view(np.uint64).tolist() == expected.view(np.uint64).tolist()
    elif kind == "contrib":
        np.testing.assert_allclose(raw, expected.sum(axis=1), rtol=0, atol=1e-12)
    else:
        np.testing.assert_allclose(sigmoid_out, expected, rtol=1e-15, atol=0)


@pytest.mark.parametrize("case", prediction_cases(), ids=lambda c: c[0])
def test_oracle_prediction_real_lightgbm(oracle_lib, case):
    from lightgbm_rs_b200 import model_text as MT

    import oracle

    _, fname, X, expected, kind = case
    model = MT.parse(G.read_text(fname))
    flat = MT.flatten(model)
    raw = oracle.predict_raw(flat, X)
    sig = 1.0 / (1.0 + np.exp(-model.sigmoid * raw))
    check_prediction(kind, raw, expected, sig)


def test_writer_from_oracle_rank_trees(oracle_lib):
    """model_text.from_booster + dump on the oracle's 10 lambdarank trees (the trees the
    device booster reproduces bit for bit) equals lib_lightgbm's file up to its
    parameters block, with the zero-threshold constant of the reference's bins."""
    import lightgbm_rs_b200 as lgb
    from lightgbm_rs_b200 import model_text as MT
    from test_gpu_predict import _with_reference_zero_threshold

    import oracle

    X, labels, qb, _, _, _ = G.rank_case()
    mappers, cols = [], []
    for j in range(X.shape[1]):
        m, b = lgb.bin_column(X[:, j], max_bin=255, min_data_in_bin=1, min_data_in_leaf=1,
                              pre_filter=False, bin_construct_sample_cnt=1_000_000)
        mappers.append(m)
        cols.append(b.astype(np.uint8))
    metas = [{k: m[k] for k in ("num_bin", "default_bin", "most_freq_bin", "missing_type")}
             for m in mappers]
    out = oracle.train(np.stack(cols), metas, labels, objective="lambdarank",
                       num_iterations=10, learning_rate=0.1, num_leaves=7,
                       query_boundaries=qb, lambdarank_truncation_level=5,
                       min_data_in_leaf=1, min_sum_hessian_in_leaf=1e-3)

    class _Trained:  # the attributes from_booster reads from a booster
        objective = "lambdarank"
        params = {"learning_rate": 0.1, "sigmoid": 1.0}

        class train_set:
            pass

        def init_score(self):
            return 0.0

        def trees(self):
            return out["trees"]

    tb = _Trained()
    tb.train_set.mappers = mappers
    text = MT.dump(MT.from_booster(tb))
    gold = _with_reference_zero_threshold(G.read_text("rank_lambdarank_byq0_es0_model.txt"))
    cut = gold.index("\nparameters:\n")
    assert text[:cut] == gold[:cut]
