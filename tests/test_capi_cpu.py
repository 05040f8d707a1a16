"""CPU checks of the C-ABI library: it loads, exports every declared symbol, and its
host-only entry points (binning) match the reference's golden vectors.

Binning goldens: crates/lgbm-dataset/tests/fixtures/numeric_binning.txt replayed as in
crates/lgbm-dataset/tests/bin_mapper_internals.rs and numeric_assignment.rs.
"""

import ctypes

import numpy as np
import pytest

import _golden as G


@pytest.fixture(scope="module")
def capi():
    from lightgbm_rs_b200 import build

    build.build()
    from lightgbm_rs_b200 import _lib

    return _lib


def test_library_exports_every_header_symbol(capi):
    L = capi.lib()
    names = capi.header_symbols()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert L.lgbm_b200_abi_version() == 104


def test_device_count_never_errors(capi):
    assert capi.device_count() >= 0


def test_binning_matches_reference_golden(capi):
    import lightgbm_rs_b200 as lgb

    cases = G.binning_cases()
    assert len(cases) == 45
    for c in cases:
        m, bins = lgb.bin_column(c["values"], max_bin=c["max_bin"],
                                 min_data_in_bin=c["min_data_in_bin"],
                                 min_data_in_leaf=c["min_split_data"],
                                 pre_filter=c["pre_filter"], use_missing=c["use_missing"],
                                 zero_as_missing=c["zero_as_missing"],
                                 bin_construct_sample_cnt=c["sample_cnt"],
                                 data_random_seed=c["seed"])
        gold = c["golden"]
        assert m["num_bin"] == gold["num_bin"], c["name"]
        assert m["missing_type"] == gold["missing_type"], c["name"]
        assert m["default_bin"] == gold["default_bin"], c["name"]
        assert m["most_freq_bin"] == gold["most_freq_bin"], c["name"]
        assert m["is_trivial"] == gold["is_trivial"], c["name"]
        got_bits = m["upper"].view(np.uint64)
        want_bits = gold["upper"].view(np.uint64)
        # NaN sentinel bound: compare by NaN-ness, everything else bit-exact
        gn, wn = np.isnan(m["upper"]), np.isnan(gold["upper"])
        assert gn.tolist() == wn.tolist(), c["name"]
        assert got_bits[~gn].tolist() == want_bits[~wn].tolist(), c["name"]
        assert bins.tolist() == c["assign"].tolist(), c["name"]


def test_categorical_binning_matches_reference_golden(capi):
    """categorical_folding.txt: descending-count fold, the 0.99 cut, the min_data_in_bin
    fold break, negative values and the NaN dummy bin 0 (bin_mapper.rs:416-641)."""
    import lightgbm_rs_b200 as lgb

    cases = G.categorical_binning_cases()
    assert len(cases) == 6
    for c in cases:
        m, bins = lgb.bin_column(c["values"], max_bin=c["max_bin"],
                                 min_data_in_bin=c["min_data_in_bin"],
                                 min_data_in_leaf=c["min_split_data"],
                                 pre_filter=c["pre_filter"], use_missing=c["use_missing"],
                                 zero_as_missing=c["zero_as_missing"],
                                 bin_construct_sample_cnt=max(len(c["values"]), 1),
                                 categorical=True)
        gm = c["mapper"]
        assert m["bin_type"] == gm["bin_type"] == 1, c["name"]
        for k in ("num_bin", "missing_type", "default_bin", "most_freq_bin"):
            assert m[k] == gm[k], (c["name"], k)
        assert m["is_trivial"] == bool(gm["is_trivial"]), c["name"]
        assert m["bin_to_category"].tolist() == c["b2c"], c["name"]
        c2b = {int(cat): b for b, cat in enumerate(m["bin_to_category"])}
        assert c2b == c["c2b"], c["name"]
        assert bins.tolist() == c["assign"].tolist(), c["name"]


def test_errors_are_typed_not_crashes(capi):
    L = capi.lib()
    out = np.zeros(4, dtype=np.float64)
    bins = np.array([0, 1, 5], dtype=np.uint32)
    g = np.zeros(3, dtype=np.float32)
    rc = L.lgbm_b200_construct_histograms(capi.ptr(bins), capi.ptr(g), capi.ptr(g), 3, 2,
                                          capi.ptr(out))
    assert rc == capi.BIN_OUT_OF_RANGE
    assert b"bin 5" in L.lgbm_b200_last_error()
    rc = L.lgbm_b200_construct_histograms(capi.ptr(bins), capi.ptr(g), capi.ptr(g), 3, 300,
                                          capi.ptr(out))
    assert rc == capi.CAPABILITY_UNAVAILABLE
    h = ctypes.c_void_p()
    rc = L.lgbm_b200_dataset_create(0, None, 1, 0, 1, None, ctypes.byref(h))
    assert rc == capi.INVALID_ARGUMENT
