"""Bin finding on the device (lgbm_b200_find_bins): for numerical columns it must return
exactly the mappers of the host BinMapper restatement (lgbm_b200_bin_column) and of the
reference's binning goldens: every field, every upper bound bit for bit."""

import numpy as np
import pytest

import _golden as G

pytestmark = pytest.mark.gpu

FIELDS = ("num_bin", "missing_type", "default_bin", "most_freq_bin", "is_trivial")


def _same(dev, host, tag):
    for k in FIELDS:
        assert dev[k] == host[k], (tag, k, dev[k], host[k])
    a, b = dev["upper"], host["upper"]
    assert np.isnan(a).tolist() == np.isnan(b).tolist(), tag
    assert a.view(np.uint64)[~np.isnan(a)].tolist() == \
        b.view(np.uint64)[~np.isnan(b)].tolist(), tag
    assert dev["min_val"] == host["min_val"] and dev["max_val"] == host["max_val"], tag
    assert dev["sparse_rate"] == host["sparse_rate"], tag


def test_device_find_bins_replays_numeric_goldens():
    import lightgbm_rs_b200 as lgb

    cases = G.binning_cases()
    assert len(cases) == 45
    for c in cases:
        kw = dict(max_bin=c["max_bin"], min_data_in_bin=c["min_data_in_bin"],
                  min_data_in_leaf=c["min_split_data"], pre_filter=c["pre_filter"],
                  use_missing=c["use_missing"], zero_as_missing=c["zero_as_missing"],
                  bin_construct_sample_cnt=c["sample_cnt"], data_random_seed=c["seed"])
        (dev,) = lgb.find_bins([np.asarray(c["values"], dtype=np.float64)], **kw)
        gold = c["golden"]
        for k in FIELDS:
            assert dev[k] == gold[k], (c["name"], k)
        gn, wn = np.isnan(dev["upper"]), np.isnan(gold["upper"])
        assert gn.tolist() == wn.tolist(), c["name"]
        assert dev["upper"].view(np.uint64)[~gn].tolist() == \
            gold["upper"].view(np.uint64)[~wn].tolist(), c["name"]


@pytest.mark.parametrize("n", [1_000, 150_000, 700_001])
def test_device_find_bins_equal_host(n):
    """Columns of many shapes, more rows than the 200k sample and fewer: normal,
    exponential, NaN-holed, zero-heavy with signed values, mixed signed zeros, integer
    codes, constant, all NaN; f32 and f64; with and without the pre-filter and
    zero_as_missing."""
    import lightgbm_rs_b200 as lgb

    r = np.random.default_rng(n)
    cols = [r.normal(size=n), np.exp(r.normal(size=n)),
            np.where(r.random(n) < 0.2, np.nan, r.normal(size=n)),
            np.where(r.random(n) < 0.9, 0.0, r.normal(size=n)),
            np.where(r.random(n) < 0.5, -0.0, 0.0) + np.where(r.random(n) < 0.3, 1.5, 0.0),
            r.integers(-3, 40, n).astype(np.float64), np.full(n, 7.25), np.full(n, np.nan)]
    for dt in (np.float64, np.float32):
        cs = [c.astype(dt) for c in cols]
        for kw in (dict(max_bin=255, min_data_in_leaf=20),
                   dict(max_bin=63, min_data_in_leaf=100, pre_filter=True),
                   dict(max_bin=15, zero_as_missing=True, min_data_in_bin=5)):
            dev = lgb.find_bins(cs, **kw)
            for j, c in enumerate(cs):
                host, _ = lgb.bin_column(c, want_bins=False, **kw)
                _same(dev[j], host, (n, np.dtype(dt).name, j, tuple(kw.items())))


def test_dataset_uses_device_bins():
    """Dataset from raw values: mappers found on the device, bins on the device, equal to
    the host binning of the same columns."""
    import lightgbm_rs_b200 as lgb
    from lightgbm_rs_b200 import synthetic

    X, y = synthetic.binary_c0(num_data=300_000, seed=5)
    ds = lgb.Dataset(X, y, {"max_bin": 255, "device_binning": True})  # ("auto": host at 28)
    host = lgb.Dataset(X, y, {"max_bin": 255, "device_binning": False})
    for a, b in zip(ds.mappers, host.mappers):
        _same(a, b, "dataset")
    assert np.array_equal(ds.device_bins(), host.bins.astype(np.uint8))
