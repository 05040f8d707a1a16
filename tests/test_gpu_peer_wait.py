"""Failure detection of the peer-memory exchange without a GPU fault.

The exchange's consumers wait on flags that the other ranks set. Every wait is bounded
(%globaltimer): when a rank stops answering, the kernel records the spin-timeout error bit,
ends the tree, and the host call returns LGBM_B200_RUNTIME with the error bits. The test
makes a one-device booster wait on a second rank that never publishes (the
LGBM_B200_PEER_EXCHANGE=silent-peer hook), so the wait runs out on a flag nothing sets;
the context stays usable afterwards.
"""

import os
import time

import pytest

from test_gpu_handles import _dataset

pytestmark = pytest.mark.gpu


def test_silent_peer_wait_runs_out_and_reports():
    import lightgbm_rs_b200 as lgb
    from lightgbm_rs_b200 import _lib as C

    ds, p = _dataset()
    saved = {k: os.environ.get(k) for k in ("LGBM_B200_PEER_EXCHANGE", "LGBM_B200_PEER_WAIT_MS")}
    os.environ["LGBM_B200_PEER_EXCHANGE"] = "silent-peer"
    os.environ["LGBM_B200_PEER_WAIT_MS"] = "50"
    try:
        b = lgb.Booster(p, ds)
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    t0 = time.perf_counter()
    with pytest.raises(lgb.LightGBMError) as e:
        b.update(3)
    assert time.perf_counter() - t0 < 20.0
    assert e.value.code == C.RUNTIME
    assert "device error bits 0x1" in str(e.value)
    del b
    # the device still trains normally
    b2 = lgb.Booster(p, ds)
    assert b2.update(2) == 2
    assert b2.trees()[0]["num_leaves"] > 1
