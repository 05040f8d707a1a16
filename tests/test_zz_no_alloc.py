"""Allocation-free row partition (lgbm_b200_data_partition_noalloc) through the C ABI.

The entry point takes device buffers and keeps its scratch in a fixed array inside the
library; its results must equal those of lgbm_b200_data_partition (the allocating,
host-buffer entry point) on the same inputs. Row indices and split points are integers,
so the comparison is exact. Two or more calls run back to back to show that each call
clears the shared scratch it uses.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def capi():
    from lightgbm_rs_b200 import _lib

    assert _lib.device_count() > 0, "no CUDA device"
    return _lib


def _host_partition(capi, bins, num_bin, min_bin, max_bin, thr, mfb):
    L = capi.lib()
    b32 = bins.astype(np.uint32)
    order = np.empty(len(bins), dtype=np.uint32)
    sp = ctypes.c_int64(-1)
    capi.check(L.lgbm_b200_data_partition(capi.ptr(b32), len(bins), num_bin, min_bin, max_bin,
                                          thr, mfb, capi.ptr(order), ctypes.byref(sp)))
    return order, sp.value


def _noalloc_partition(capi, bins, num_bin, min_bin, max_bin, thr, mfb):
    import torch

    L = capi.lib()
    n = len(bins)
    d_bins = torch.from_numpy(bins.astype(np.uint8)).cuda()
    d_order = torch.full((max(n, 1),), -1, dtype=torch.int32, device="cuda")
    d_sp = torch.full((1,), -1, dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    capi.check(L.lgbm_b200_data_partition_noalloc(d_bins.data_ptr(), n, num_bin, min_bin,
                                                  max_bin, thr, mfb, d_order.data_ptr(),
                                                  d_sp.data_ptr(), stream))
    torch.cuda.synchronize()
    order = d_order.cpu().numpy().view(np.uint32)[:n]
    return order, int(d_sp.cpu().item())


CASES = [
    # n, num_bin, min_bin, max_bin, most_freq_bin, seed
    (3_000_001, 256, 0, 255, 7, 1),
    (100_003, 63, 1, 62, 0, 2),  # most_freq_bin 0: offset threshold path
    (2048, 16, 0, 15, 3, 3),  # exactly one tile
    (1, 4, 0, 3, 1, 4),
]


def test_noalloc_matches_allocating_entry_point(capi):
    rng = np.random.default_rng(11)
    calls = 0
    for n, num_bin, min_bin, max_bin, mfb, seed in CASES + CASES[:1]:
        r = np.random.default_rng(seed)
        bins = r.integers(min_bin, max_bin + 1, n).astype(np.uint8)
        thr = int(rng.integers(0, num_bin - 1)) if num_bin > 1 else 0
        want_order, want_sp = _host_partition(capi, bins, num_bin, min_bin, max_bin, thr, mfb)
        got_order, got_sp = _noalloc_partition(capi, bins, num_bin, min_bin, max_bin, thr, mfb)
        assert got_sp == want_sp, (n, num_bin, thr)
        assert np.array_equal(got_order, want_order), (n, num_bin, thr)
        calls += 1
    assert calls >= 2


def test_noalloc_repeated_identical_calls(capi):
    """The same large input twice in a row: the second call must not see the first's
    look-back words."""
    r = np.random.default_rng(21)
    bins = r.integers(0, 256, 1_500_000).astype(np.uint8)
    want = _host_partition(capi, bins, 256, 0, 255, 100, 5)
    for _ in range(2):
        got = _noalloc_partition(capi, bins, 256, 0, 255, 100, 5)
        assert got[1] == want[1]
        assert np.array_equal(got[0], want[0])


def test_noalloc_keeps_device_memory_unchanged(capi):
    """After a warm-up call (which loads the module and looks the scratch array up), a
    batch of calls leaves the device's free memory exactly as it was: nothing is
    allocated and kept."""
    import torch

    L = capi.lib()
    r = np.random.default_rng(31)
    n = 2_000_000
    d_bins = torch.from_numpy(r.integers(0, 256, n).astype(np.uint8)).cuda()
    d_order = torch.empty(n, dtype=torch.int32, device="cuda")
    d_sp = torch.empty(1, dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def call():
        capi.check(L.lgbm_b200_data_partition_noalloc(d_bins.data_ptr(), n, 256, 0, 255, 77,
                                                      3, d_order.data_ptr(),
                                                      d_sp.data_ptr(), stream))

    call()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(8):
        call()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert 0 <= int(d_sp.item()) <= n


def test_noalloc_empty_and_limit(capi):
    import torch

    L = capi.lib()
    order, sp = _noalloc_partition(capi, np.zeros(0, dtype=np.uint8), 4, 0, 3, 1, 0)
    assert sp == 0 and len(order) == 0
    # beyond the fixed scratch: rejected before any work is enqueued
    limit = 67108864
    d = torch.zeros(16, dtype=torch.int64, device="cuda")
    rc = L.lgbm_b200_data_partition_noalloc(d.data_ptr(), limit + 1, 256, 0, 255, 3, 0,
                                            d.data_ptr(), d.data_ptr(), None)
    assert rc == capi.CAPABILITY_UNAVAILABLE
    assert b"LGBM_B200_NOALLOC_MAX_ROWS" in L.lgbm_b200_last_error()
    torch.cuda.synchronize()
    assert int(d.abs().sum().item()) == 0
