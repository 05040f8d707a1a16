"""Binning on the device: BinMapper::value_to_bin (crates/lgbm-dataset/src/bin_mapper.rs:
148-199) over raw values, and the pre-binned path's range check, both writing the row-major
u8 matrix. Pinned to the reference's numeric and categorical binning goldens (assignments
of every value) and to the host binning on mixed data."""

import ctypes

import numpy as np
import pytest

import _golden as G

pytestmark = pytest.mark.gpu


def _device_bins_one(values, mapper):
    import lightgbm_rs_b200 as lgb

    ds = lgb.Dataset(bins=np.zeros((1, len(values)), np.uint8), mappers=[mapper])
    ds._bins = None
    ds._values = np.ascontiguousarray(np.asarray(values, np.float64).reshape(1, -1))
    return ds.device_bins()[0]


def test_device_binning_numeric_goldens():
    import lightgbm_rs_b200 as lgb

    n = 0
    for c in G.binning_cases():
        if len(c["values"]) == 0:
            continue
        m, _ = lgb.bin_column(c["values"], max_bin=c["max_bin"],
                              min_data_in_bin=c["min_data_in_bin"],
                              min_data_in_leaf=c["min_split_data"], pre_filter=c["pre_filter"],
                              use_missing=c["use_missing"], zero_as_missing=c["zero_as_missing"],
                              bin_construct_sample_cnt=c["sample_cnt"],
                              data_random_seed=c["seed"], want_bins=False)
        if m["num_bin"] > 256:
            continue
        got = _device_bins_one(c["values"], m)
        assert got.tolist() == c["assign"].tolist(), c["name"]
        n += 1
    assert n >= 30


def test_device_binning_categorical_goldens():
    import lightgbm_rs_b200 as lgb

    for c in G.categorical_binning_cases():
        if len(c["values"]) == 0:
            continue
        m, _ = lgb.bin_column(c["values"], max_bin=c["max_bin"],
                              min_data_in_bin=c["min_data_in_bin"],
                              min_data_in_leaf=c["min_split_data"], pre_filter=c["pre_filter"],
                              use_missing=c["use_missing"], zero_as_missing=c["zero_as_missing"],
                              bin_construct_sample_cnt=max(len(c["values"]), 1),
                              want_bins=False, categorical=True)
        got = _device_bins_one(c["values"], m)
        assert got.tolist() == c["assign"].tolist(), c["name"]


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_device_binning_equals_host_binning(dtype):
    import lightgbm_rs_b200 as lgb

    rng = np.random.default_rng(7)
    n = 300_000
    X = np.empty((n, 37))
    X[:, :20] = rng.normal(0, 2, (n, 20))
    X[:, 20:25] = np.where(rng.random((n, 5)) < 0.7, 0.0, rng.exponential(1.0, (n, 5)))
    X[:, 25:30] = rng.integers(-3, 200, (n, 5))          # categorical, with negatives
    X[:, 30:37] = rng.uniform(-1e6, 1e6, (n, 7))
    X[rng.random(X.shape) < 0.05] = np.nan
    X[rng.random(X.shape) < 0.01] = np.inf
    X[:3, 25] = [2.0 ** 40, -2.0 ** 40, 7.9]
    ds = lgb.Dataset(X.astype(dtype), rng.random(n), {"max_bin": 255},
                     categorical_feature=list(range(25, 30)))
    assert ds.device_bins().tolist() == ds.bins.tolist()


@pytest.mark.parametrize("width", [1, 2, 4])
def test_prebinned_columns_and_range_check(width):
    import lightgbm_rs_b200 as lgb
    from lightgbm_rs_b200 import _lib as C

    rng = np.random.default_rng(width)
    F, n = 19, 70_001
    nb = rng.integers(2, 257, F)
    nb[7], nb[12] = 100, 50
    dt = {1: np.uint8, 2: np.uint16, 4: np.uint32}[width]
    bins = np.stack([rng.integers(0, nb[f], n) for f in range(F)]).astype(dt)
    mappers = [{"num_bin": int(nb[f]), "default_bin": 0, "most_freq_bin": 0,
                "missing_type": 0} for f in range(F)]
    ds = lgb.Dataset(bins=bins, mappers=mappers)
    assert ds.device_bins().tolist() == bins.astype(np.uint8).tolist()
    # out-of-range bins: the first in row-major order is reported
    bad = bins.copy()
    bad[12, 50_000] = 60
    bad[7, 50_000] = 100
    bad[2, 60_000] = nb[2] if nb[2] < 256 else 255 if width == 1 else 300
    ds2 = lgb.Dataset(bins=bad, mappers=mappers)
    with pytest.raises(lgb.LightGBMError) as e:
        ds2.construct()
    assert e.value.code == C.BIN_OUT_OF_RANGE
    assert "feature 7 row 50000" in str(e.value)
