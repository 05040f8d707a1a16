"""Data-parallel training on 2 GPUs (one spawned process per GPU) against one GPU.

Quantized gradients: trees and scores of every rank must be bit-identical to training
on all rows on one GPU. f32 gradients: same tree structure, scores within 1e-9.
With 255 leaves most splits come from look-ahead partitions, whose child histograms are
exchanged over peer memory like the main ones; the last iteration is profiled and must
show them used. Needs at least 2 GPUs; never runs two ranks on one GPU.
"""

import multiprocessing as mp
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

PARAMS = {"objective": "binary", "num_leaves": 31, "min_data_in_leaf": 20,
          "learning_rate": 0.1, "max_bin": 255}
ROWS = 50_001
ITERS = 5


def _data(wide=False):
    import lightgbm_rs_b200 as lgb
    from lightgbm_rs_b200 import synthetic

    if wide:  # the C2 shape: many 63-bin features, every rank scans its own slice
        X, y = synthetic.wide_c2(num_data=ROWS, num_features=600, seed=7)
        return lgb.Dataset(X, y, dict(PARAMS, max_bin=63))
    X, y = synthetic.binary_c0(num_data=ROWS, seed=7)
    return lgb.Dataset(X, y, dict(PARAMS))  # host binning only, deterministic


def _worker(rank, world, uid, quantized, leaves, q, wide=False, slices=True):
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        # on: every rank scans its own half of the features (forced for narrow data, where
        # the default keeps every feature on every rank); off: every rank scans all
        os.environ["LGBM_B200_FEATURE_SLICES"] = "1" if slices else "0"
        import sys
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        import lightgbm_rs_b200 as lgb
        from lightgbm_rs_b200 import distributed as D

        full = _data(wide)
        b, e = D.shard_range(full.num_data, world, rank)
        p = dict(PARAMS, device=rank, use_quantized_grad=quantized, num_grad_quant_bins=4,
                 num_leaves=leaves, max_bin=63 if wide else 255)
        shard = lgb.Dataset(bins=full.bins[:, b:e], mappers=full.mappers,
                            label=full.label[b:e], params=p)
        comm = D.Communicator(rank, world, rank, uid)
        booster = lgb.train(p, shard, num_boost_round=ITERS - 1, comm=comm)
        _, counts = booster.profile_iteration()  # the last iteration, with counters
        q.put((rank, booster.trees(), booster.train_scores(), counts))
        del booster
        comm.close()
    except Exception as ex:
        q.put((rank, "error", repr(ex)))


@pytest.mark.parametrize("quantized,leaves,wide,slices", [
    (True, 31, False, True), (False, 31, False, True), (True, 255, False, True),
    (True, 63, True, True), (True, 255, False, False)])
def test_two_gpus_match_one(quantized, leaves, wide, slices):
    """Feature slices on (each rank scans half the features, the slices' best splits are
    exchanged before the pick) and off (every rank scans every feature)."""
    import lightgbm_rs_b200 as lgb
    from lightgbm_rs_b200 import distributed as D

    if lgb._lib.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    uid = D.unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, uid, quantized, leaves, q, wide, slices))
             for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(2):
            r = q.get(timeout=300)
            out[r[0]] = r
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(2):
        assert out[r][1] != "error", out[r]
    if leaves == 255:
        for r in range(2):
            c = out[r][3]
            assert c["lookahead_runs"] > 0 and c["lookahead_hits"] > 0, (r, c)
    full = _data(wide)
    p = dict(PARAMS, use_quantized_grad=quantized, num_grad_quant_bins=4, num_leaves=leaves,
             max_bin=63 if wide else 255)
    ref = lgb.train(p, full, num_boost_round=ITERS)
    want_trees, want_scores = ref.trees(), ref.train_scores()
    scores = np.concatenate([out[0][2], out[1][2]])
    for r in range(2):
        trees = out[r][1]
        assert len(trees) == len(want_trees)
        for a, b in zip(trees, want_trees):
            for k in ("split_feature", "threshold_bin", "left_child", "right_child",
                      "leaf_count", "internal_count"):
                assert a[k].tolist() == b[k].tolist(), (r, k)
            if quantized:
                assert a["leaf_value"].tobytes() == b["leaf_value"].tobytes()
            else:
                np.testing.assert_allclose(a["leaf_value"], b["leaf_value"], rtol=1e-9)
    if quantized:
        assert scores.view(np.uint64).tolist() == want_scores.view(np.uint64).tolist()
    else:
        np.testing.assert_allclose(scores, want_scores, rtol=0, atol=1e-9)
