"""Per-op device entry points (the Backend-trait mirror) against the reference goldens.

Same fixtures and assertions as crates/oracle-harness/tests/kernel_parity.rs
(histogram :162, split :512, partition :1162, subtract :1276), run through the C ABI.
"""

import ctypes

import numpy as np
import pytest

import _golden as G

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def capi():
    from lightgbm_rs_b200 import _lib

    assert _lib.device_count() > 0, "no CUDA device"
    return _lib


def test_histogram_golden(capi):
    L = capi.lib()
    n_cases = 0
    for c in G.histogram_cases():
        if c["num_bin"] > 256:
            continue  # the u8 bin matrix holds at most 256 bins per feature
        out = np.empty(2 * c["num_bin"], dtype=np.float64)
        capi.check(L.lgbm_b200_construct_histograms(
            capi.ptr(c["bins"]), capi.ptr(c["grad"]), capi.ptr(c["hess"]), len(c["bins"]),
            c["num_bin"], capi.ptr(out)))
        want = c["hist"]
        # f32 g/h accumulate in 64-bit fixed point: within 1e-6 relative of the f64 fold
        # (relative to the sum of magnitudes in the cell).
        mag = np.zeros_like(want)
        np.add.at(mag, 2 * c["bins"].astype(np.int64), np.abs(c["grad"].astype(np.float64)))
        np.add.at(mag, 2 * c["bins"].astype(np.int64) + 1, np.abs(c["hess"].astype(np.float64)))
        assert np.all(np.abs(out - want) <= 1e-6 * mag + 1e-300), c["name"]
        n_cases += 1
    assert n_cases >= 6


def test_histogram_exact_for_dyadic_gradients(capi):
    """Gradients that are multiples of a power of two sum exactly: bit-exact result."""
    L = capi.lib()
    rng = np.random.default_rng(3)
    n, nb = 200_000, 255
    bins = rng.integers(0, nb, n).astype(np.uint32)
    g = (rng.integers(-64, 64, n) / 128.0).astype(np.float32)
    h = (rng.integers(1, 64, n) / 256.0).astype(np.float32)
    out = np.empty(2 * nb, dtype=np.float64)
    capi.check(L.lgbm_b200_construct_histograms(capi.ptr(bins), capi.ptr(g), capi.ptr(h), n, nb,
                                                capi.ptr(out)))
    import oracle

    want = oracle.construct_histogram(bins, g, h, nb)
    assert out.view(np.uint64).tolist() == want.view(np.uint64).tolist()


def test_split_golden_bit_exact(capi):
    L = capi.lib()
    for c in G.split_cases():
        cfg = capi.gain_config(c["min_data_in_leaf"], c["min_sum_hessian_in_leaf"], 0.0,
                               c["lambda_l1"], c["lambda_l2"], c["min_gain_to_split"])
        s = capi.SplitInfo()
        capi.check(L.lgbm_b200_find_best_split(
            capi.ptr(c["hist"]), ctypes.byref(cfg), c["num_bin"], c["offset"], c["default_bin"],
            0, int(c["skip_default_bin"]), int(c["na_as_missing"]), 1, c["sum_gradient"],
            c["sum_hessian"], c["num_data"], ctypes.byref(s)))
        w = c["win"]
        assert (s.gain != -np.inf) == w["is_splittable"], c["name"]
        if not w["is_splittable"]:
            continue
        for k in ("gain", "left_sum_gradient", "left_sum_hessian", "right_sum_gradient",
                  "right_sum_hessian", "left_output", "right_output"):
            assert G.bits_of_f64(getattr(s, k)) == w[k], (c["name"], k)
        assert s.threshold == w["threshold"], c["name"]
        assert (s.left_count, s.right_count) == (w["left_count"], w["right_count"]), c["name"]
        assert bool(s.default_left) == w["default_left"], c["name"]


def _random_scan_case(rng, num_bin, offset, missing, with_cfg):
    hist = np.empty(2 * num_bin)
    hist[0::2] = rng.normal(0, 1, num_bin)
    hist[1::2] = rng.uniform(0.01, 2.0, num_bin)
    if offset:
        hist[-2:] = 0.0
    sg = float(hist[0::2].sum() + rng.normal())
    sh = float(hist[1::2].sum() + rng.uniform(0, 1))
    nd = int(rng.integers(num_bin * 5, num_bin * 50))
    kw = dict(min_data_in_leaf=int(rng.integers(1, 30)), min_sum_hessian_in_leaf=1e-3)
    if with_cfg:
        kw.update(lambda_l1=float(rng.uniform(0, 1)), lambda_l2=float(rng.uniform(0, 2)),
                  min_gain_to_split=float(rng.uniform(0, 0.5)),
                  max_delta_step=float(rng.choice([0.0, 0.3])),
                  path_smooth=float(rng.choice([0.0, 2.0])),
                  parent_output=float(rng.normal(0, 0.1)))
    return hist, sg, sh, nd, kw


def test_scan_matches_oracle_random_configs(capi):
    """Random histograms through every gain axis (L1, L2, max_delta_step, path_smooth),
    every missing type and both offsets: device scan bit-exact with the oracle."""
    import oracle

    L = capi.lib()
    rng = np.random.default_rng(11)
    for it in range(300):
        num_bin = int(rng.choice([2, 3, 5, 17, 64, 200, 256]))
        offset = int(rng.integers(0, 2))
        missing = int(rng.integers(0, 3))
        hist, sg, sh, nd, kw = _random_scan_case(rng, num_bin, offset, missing, it % 2 == 1)
        default_bin = int(rng.integers(0, num_bin))
        skip = num_bin > 2 and missing == 1
        na = num_bin > 2 and missing == 2
        fwd = num_bin > 2 and missing != 0
        ocfg = oracle.gain_config(**kw)
        want = oracle.find_best_split(hist, ocfg, num_bin, offset, default_bin, skip, na, fwd,
                                      sg, sh, nd)
        cfg = capi.gain_config(**kw)
        s = capi.SplitInfo()
        capi.check(L.lgbm_b200_find_best_split(capi.ptr(hist), ctypes.byref(cfg), num_bin, offset,
                                               default_bin, 0, int(skip), int(na), int(fwd), sg,
                                               sh, nd, ctypes.byref(s)))
        for k, _ in capi.SplitInfo._fields_:
            a, b = getattr(s, k), getattr(want, k)
            if isinstance(a, float):
                assert G.bits_of_f64(a) == G.bits_of_f64(b), (it, k, a, b)
            else:
                assert a == b, (it, k, a, b)


def test_subtract_golden_bit_exact(capi):
    L = capi.lib()
    for c in G.subtract_cases():
        out = np.empty_like(c["subparent"])
        capi.check(L.lgbm_b200_subtract_histograms(capi.ptr(c["subparent"]),
                                                   capi.ptr(c["subchild"]), len(out),
                                                   capi.ptr(out)))
        assert out.view(np.uint64).tolist() == c["subderived"].view(np.uint64).tolist()


def test_partition_golden_exact(capi):
    L = capi.lib()
    n = 0
    for c in G.partition_cases():
        if c["missing_type"] != 0:
            continue
        order = np.empty(len(c["bins"]), dtype=np.uint32)
        sp = ctypes.c_int64(0)
        capi.check(L.lgbm_b200_data_partition(capi.ptr(c["bins"]), len(c["bins"]), c["num_bin"],
                                              c["min_bin"], c["max_bin"], c["threshold"],
                                              c["most_freq_bin"], capi.ptr(order),
                                              ctypes.byref(sp)))
        assert order.tolist() == c["order"].tolist(), c["name"]
        assert sp.value == c["split"], c["name"]
        n += 1
    assert n >= 4


def test_partition_golden_missing_fanout_exact(capi):
    """Every partition.txt case, the six with missing_type != 0 included (missing zero /
    NA with both default directions, the most frequent bin at the zero or NA bin),
    through the device router, as crates/oracle-harness/tests/partition_parity.rs:112-190
    replays them."""
    L = capi.lib()
    missing = 0
    for c in G.partition_cases():
        order = np.empty(len(c["bins"]), dtype=np.uint32)
        sp = ctypes.c_int64(0)
        capi.check(L.lgbm_b200_data_partition_missing(
            capi.ptr(c["bins"]), len(c["bins"]), c["num_bin"], c["min_bin"], c["max_bin"],
            c["threshold"], c["most_freq_bin"], c["default_bin"], c["missing_type"],
            c["default_left"], capi.ptr(order), ctypes.byref(sp)))
        assert order.tolist() == c["order"].tolist(), c["name"]
        assert sp.value == c["split"], c["name"]
        missing += c["missing_type"] != 0
    assert missing == 6


@pytest.mark.parametrize("missing_type", [1, 2])
def test_partition_missing_random_matches_oracle(capi, missing_type):
    """Multi-tile partitions with every missing-route flag combination against the
    oracle's restatement of the same router."""
    import oracle

    L = capi.lib()
    rng = np.random.default_rng(40 + missing_type)
    n = 300_001
    for trial in range(24):
        num_bin = int(rng.integers(3, 40))
        min_bin = int(rng.integers(0, 3))
        max_bin = int(rng.integers(min_bin, num_bin)) if trial % 6 else min_bin
        mfb = int(rng.integers(0, num_bin))
        default_bin = mfb if trial % 4 == 0 else int(rng.integers(0, num_bin))
        if missing_type == 2 and trial % 5 == 0 and max_bin > min_bin:
            mfb = max_bin - min_bin  # the most frequent bin is the NA bin
        thr = int(rng.integers(0, num_bin))
        dl = int(trial % 2)
        bins = rng.integers(0, num_bin, n).astype(np.uint32)
        order = np.empty(n, dtype=np.uint32)
        sp = ctypes.c_int64(0)
        capi.check(L.lgbm_b200_data_partition_missing(
            capi.ptr(bins), n, num_bin, min_bin, max_bin, thr, mfb, default_bin, missing_type,
            dl, capi.ptr(order), ctypes.byref(sp)))
        want, left = oracle.partition_missing(bins, np.arange(n, dtype=np.uint32), min_bin,
                                              max_bin, thr, mfb, default_bin, missing_type, dl)
        assert sp.value == left, trial
        assert np.array_equal(order, want), trial


def test_partition_large_random_matches_oracle(capi):
    """Multi-tile decoupled look-back path: 3M rows, every tile boundary case."""
    import oracle

    L = capi.lib()
    rng = np.random.default_rng(5)
    for n in (1, 2047, 2048, 2049, 3_000_001):
        bins = rng.integers(0, 256, n).astype(np.uint32)
        thr = int(rng.integers(0, 255))
        order = np.empty(n, dtype=np.uint32)
        sp = ctypes.c_int64(0)
        capi.check(L.lgbm_b200_data_partition(capi.ptr(bins), n, 256, 0, 255, thr, 7,
                                              capi.ptr(order), ctypes.byref(sp)))
        want, left = oracle.partition(bins, np.arange(n, dtype=np.uint32), 256, 0, 255, thr, 7)
        assert sp.value == left
        assert np.array_equal(order, want)


def test_empty_inputs(capi):
    L = capi.lib()
    out = np.full(8, 7.0)
    e = np.zeros(0, dtype=np.uint32)
    f = np.zeros(0, dtype=np.float32)
    capi.check(L.lgbm_b200_construct_histograms(capi.ptr(e), capi.ptr(f), capi.ptr(f), 0, 4,
                                                capi.ptr(out)))
    assert np.all(out == 0.0)
    sp = ctypes.c_int64(5)
    order = np.zeros(1, dtype=np.uint32)
    capi.check(L.lgbm_b200_data_partition(capi.ptr(e), 0, 4, 0, 3, 1, 0, capi.ptr(order),
                                          ctypes.byref(sp)))
    assert sp.value == 0
