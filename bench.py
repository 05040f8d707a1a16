"""Benchmark: boosting iterations/s of the B200 histogram tree learner.

Default workload C1: 10,500,000 rows x 28 dense features from
the configs[0] generator (seeded synthetic: no public dataset is named), max_bin=255,
num_leaves=255, min_data_in_leaf=100, objective=binary, learning_rate=0.1.
Default gradients: use_quantized_grad with 4 quantization bins (`--grad f32` for the
f32-gradient variant). One step = one boosting iteration (gradients, quantization,
one tree, shrinkage, score update) over all rows.

`--workload c0`: configs[0] itself, 100,000 rows x 28, 31 leaves, 100 iterations.
`--workload c2`: 400,000 rows x 2,000 features ~ U(-1,1), max_bin=63, 127 leaves.
`--workload c3`: 2,000,000 rows, 90 numeric features with 10 % NaN and 10 categorical
features, L2 regression, 63 leaves. `--workload c4`: lambdarank over 20,000 queries
(about 473k rows) x 700 sparse features, 255 leaves. All are seeded synthetic stand-ins
with the configurations' shapes (lightgbm_rs_b200/synthetic.py).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload c0|c1|c2|c3|c4] [--grad quantized|f32]

Prints ONE JSON line on rank 0. Besides the timed steps, the default line carries:
  parity    the first trees and the scores after them, grown on the device and by the
            CPU oracle from the same binned data, compared bit for bit (N = 1);
  digest    SHA-256 of every tree the timed booster grew (equal for every N);
  f32       the same workload with f32 gradients;
  full      a full-length run (C1: all 500 iterations) with its tree digest;
  roofline  per-kernel device spans of the pipelined step (%globaltimer stamps in a
            graph of the same launch sequence) against the algorithmic bytes.
`--impl reference` times the reference CPU learner (the C++ restatement in oracle/, the
reference's Rust crates cannot be built here) on the host cores; that process bins its
data with the oracle's own BinMapper restatement and never loads the product library.
"""

import argparse
import hashlib
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LEARNING_RATE = 0.1
PARITY_TREES = 3

# name -> rows, features, leaves, min_data_in_leaf, max_bin, objective, full-length
# iterations, description
WORKLOADS = {
    "c0": dict(rows=100_000, features=28, leaves=31, min_data=20, max_bin=255,
               objective="binary", iterations=100,
               desc="C0 binary {rows}x28 num_leaves=31 max_bin=255"),
    "c1": dict(rows=10_500_000, features=28, leaves=255, min_data=100, max_bin=255,
               objective="binary", iterations=500,
               desc="C1 binary {rows}x28 num_leaves=255 min_data_in_leaf=100 max_bin=255"),
    "c2": dict(rows=400_000, features=2000, leaves=127, min_data=20, max_bin=63,
               objective="binary", iterations=200,
               desc="C2 binary {rows}x2000 U(-1,1) num_leaves=127 max_bin=63"),
    "c3": dict(rows=2_000_000, features=100, leaves=63, min_data=20, max_bin=255,
               objective="regression", iterations=300,
               desc="C3 l2 {rows}x100 (90 numeric, 10% NaN; 10 categorical, 16-240 "
                    "categories, Zipf 1.2) num_leaves=63 max_bin=255"),
    "c4": dict(rows=473_000, features=700, leaves=255, min_data=20, max_bin=255,
               objective="lambdarank", iterations=300,
               desc="C4 lambdarank {rows} rows / {queries} queries x700 (80% zeros) "
                    "num_leaves=255 max_bin=255"),
}

# DRAM bytes per algorithmic byte of each tree kernel, from the small-case ncu captures
# summarised in profiles/ (dram__bytes_read.sum + dram__bytes_write.sum of the captured
# launches over the algorithmic bytes of the same launches). The bench scales them to
# its own launches to fill roofline.traffic.
TRAFFIC_PER_ALGO_BYTE = {
    "partition": 5.37,  # warm capture: 4,076 MB DRAM for 759 MB algorithmic
    "build": 1.20,      # cold capture: 179.8 MB DRAM for 150 MB algorithmic
    "fixscan": 0.56,    # warm capture: 80.8 MB DRAM for 145 MB algorithmic (L2-resident)
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--grad", default="quantized", choices=["quantized", "f32"])
    ap.add_argument("--workload", default="c1", choices=sorted(WORKLOADS))
    ap.add_argument("--rows", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the f32 and full-length runs and the parity check")
    ap.add_argument("--measure", default="boosting",
                    choices=["boosting", "binning", "profile", "atomics"],
                    help="binning: time Dataset construction from raw C1 values (device "
                         "value_to_bin) against host value_to_bin on all cores; profile: "
                         "W warm-up iterations, then one iteration with every kernel launched "
                         "on its own (the case the committed ncu captures are taken on), "
                         "printing its algorithmic bytes per kernel class; atomics: the root "
                         "histogram build's shared-memory atomic rate on bin patterns that "
                         "set the bank conflicts (conflict-free, random, one address)")
    args = ap.parse_args()
    w = WORKLOADS[args.workload]
    if args.rows is None:
        args.rows = w["rows"]
    return args


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_synthetic():
    """lightgbm_rs_b200/synthetic.py loaded by path, so that importing the generators
    does not import (or load the library of) the product package."""
    path = os.path.join(ROOT, "lightgbm_rs_b200", "synthetic.py")
    spec = importlib.util.spec_from_file_location("lgbm_b200_synthetic_gen", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class Data:
    """A binned workload: feature-major bins, mappers, labels, query sizes (ranking)."""

    def __init__(self, bins, mappers, y, group=None):
        self.bins, self.mappers, self.y, self.group = bins, mappers, y, group
        self.rows = bins.shape[1]
        self.features = bins.shape[0]
        self.qb = None if group is None else \
            np.concatenate([[0], np.cumsum(group)]).astype(np.int32)


def make_data(workload, rows, seed=0, binner="product"):
    """Seeded synthetic data of the workload, binned on the host with the reference
    BinMapper: the product's (`binner="product"`, lightgbm_rs_b200.bin_column) or the
    oracle's restatement (`binner="oracle"`, used by the CPU reference arm so that its
    process never loads the product library).

    The binned result is cached under the system temp directory so repeated runs on
    one machine skip generation (keyed by workload, rows, seed and binner)."""
    import concurrent.futures as cf
    import pickle
    import tempfile

    cache = os.path.join(tempfile.gettempdir(),
                         f"lgbm_b200_{workload}_{rows}_{seed}_{binner}.pkl")
    if os.path.exists(cache):
        with open(cache, "rb") as f:
            return pickle.load(f)
    if binner == "oracle":
        import oracle

        oracle.build()
        bin_column = oracle.bin_column
    else:
        import lightgbm_rs_b200 as lgb

        bin_column = lgb.bin_column
    synthetic = load_synthetic()
    w = WORKLOADS[workload]
    group, cats = None, []
    if workload in ("c0", "c1"):  # C1 is C0's generator at 10.5M rows
        X, y = synthetic.binary_c0(num_data=rows, num_features=w["features"], seed=seed)
    elif workload == "c2":
        X, y = synthetic.wide_c2(num_data=rows, num_features=w["features"], seed=seed)
    elif workload == "c3":
        X, y, cats = synthetic.mixed_c3(num_data=rows, seed=seed)
    else:
        X, y, group = synthetic.rank_c4(num_queries=max(1, round(rows / 23.65)),
                                        num_features=w["features"], seed=seed)
    F = X.shape[1]
    mappers = [None] * F
    bins = np.empty((F, X.shape[0]), dtype=np.uint8)

    def one(j):
        m, b = bin_column(X[:, j], max_bin=w["max_bin"], min_data_in_leaf=w["min_data"],
                          categorical=j in cats)
        assert m["num_bin"] <= 256, f"feature {j}: {m['num_bin']} bins do not fit u8"
        mappers[j] = m
        bins[j] = b.astype(np.uint8)

    with cf.ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 4)) as ex:
        list(ex.map(one, range(F)))
    del X
    data = Data(bins, mappers, y, group)
    try:
        with open(cache + ".tmp", "wb") as f:
            pickle.dump(data, f, protocol=4)
        os.replace(cache + ".tmp", cache)
    except OSError:
        pass
    return data


def params(workload, grad):
    w = WORKLOADS[workload]
    p = {"objective": w["objective"], "num_leaves": w["leaves"],
         "min_data_in_leaf": w["min_data"], "learning_rate": LEARNING_RATE,
         "max_bin": w["max_bin"], "feature_pre_filter": False}
    if grad == "quantized":
        # stochastic_rounding=false: the deterministic rounding of the bit-exact gate
        p.update(use_quantized_grad=True, num_grad_quant_bins=4, stochastic_rounding=False)
    return p


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.15)  # the first sample lands inside the timed region
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


def kernel_bytes(counts, rows, grad, features):
    """Algorithmic bytes per iteration of the tree kernels, from the device counters.

    Partition: per parent row 1 B (split-feature bin) + 4 B (index write) + 4 B (index read,
    none for the root's identity order). Build: per built row F B of bins + its gradient
    pair (2 B quantized, 8 B f32) + 4 B index (none at the root). In the fused mode the
    partition kernel builds the child itself, so those built rows are charged to it, minus
    the split-feature byte and the index it has already read. On one device the control
    step runs the main partition of the splits the look-ahead missed (rows_parted_ctl /
    rows_built_ctl, the root's among them): those bytes are charged to the control step
    ("partition_ctl"), the rest to the partition launches. Control step (fixscan): per
    split, the accumulated child, the parent's integer histogram and the written child
    histograms: about 5 x 8 B per histogram cell, cells = 2 x bins (L2-resident)."""
    s_gh = 2 if grad == "quantized" else 8
    F = features
    rp, rb = counts["rows_parted"], counts["rows_built"]
    rpc, rbc = counts.get("rows_parted_ctl", 0), counts.get("rows_built_ctl", 0)
    root_in_ctl = rpc >= rows  # the root's partition ran inside a control step

    def part_bytes(rp_, child_rows_, has_root):
        b = rp_ * 5 + max(rp_ - (rows if has_root else 0), 0) * 4
        ch = child_rows_ * (F - 1 + s_gh) if counts["fused"] else 0
        return b + ch, ch

    root_build = rows * (F + s_gh)
    child_rows = max(rb - rows, 0)
    part, ch_a = part_bytes(rp - rpc, child_rows - rbc, not root_in_ctl)
    part_ctl, ch_b = part_bytes(rpc, rbc, root_in_ctl)
    if counts["fused"]:
        build = root_build
    else:
        build = root_build + child_rows * (F + s_gh + 4)
    return {"partition": part, "partition_ctl": part_ctl, "build": build,
            "child_hist_fused": ch_a + ch_b, "bin_bytes": rb * F + rp}


TREE_EXACT = ["split_feature", "threshold_bin", "decision_type", "left_child", "right_child",
              "leaf_count", "internal_count"]
TREE_BITS = ["leaf_value", "leaf_weight", "internal_value", "split_gain"]


def tree_digest(trees):
    """SHA-256 over every tree's structure and the bits of its values."""
    h = hashlib.sha256()
    for t in trees:
        h.update(np.int32(t["num_leaves"]).tobytes())
        for k in TREE_EXACT + TREE_BITS:
            h.update(np.ascontiguousarray(t[k]).tobytes())
    return h.hexdigest()


def trees_equal(got, want):
    """First difference between a device tree and an oracle tree, or None."""
    if got["num_leaves"] != want["num_leaves"]:
        return f"num_leaves {got['num_leaves']} != {want['num_leaves']}"
    for k in TREE_EXACT:
        if np.asarray(got[k]).tolist() != np.asarray(want[k]).tolist():
            return k
    for k in TREE_BITS:
        a = np.asarray(got[k])
        if a.tobytes() != np.asarray(want[k]).astype(a.dtype).tobytes():
            return k
    return None


def oracle_step(workload, data, score, grad, nt):
    """One boosting iteration of the reference CPU learner (oracle/) on `score` in place.
    Returns the tree (after shrinkage) and the f32 gradients it was grown from."""
    import oracle

    w = WORKLOADS[workload]
    metas = [{k: m[k] for k in ("num_bin", "default_bin", "most_freq_bin", "missing_type",
                                "bin_type")} for m in data.mappers]
    if w["objective"] == "binary":
        g, h = oracle.binary_gradients(score, data.y, 1.0, nt)
    elif w["objective"] == "lambdarank":
        g, h = oracle.lambdarank_gradients(score, data.y, data.qb, 1.0, True, 30, None, nt)
    else:
        g, h = oracle.l2_gradients(score, data.y, nt)
    g32, h32 = g, h
    if grad == "quantized":
        g, h, _, _ = oracle.quantize(g, h, 4)
    tree, part, _ = oracle.grow_tree(data.bins, metas, g, h, w["leaves"], -1, nt,
                                     min_data_in_leaf=w["min_data"])
    oracle.tree_shrinkage(tree, LEARNING_RATE)
    oracle.add_prediction_to_score(tree, part, score)
    return tree, (g32, h32)


def oracle_init_score(workload, data):
    import oracle

    obj = WORKLOADS[workload]["objective"]
    init = 0.0 if obj == "lambdarank" else oracle.boost_from_score(obj, data.y)
    return np.full(data.rows, init, dtype=np.float64)


def cpu_run(workload, data, grad, seconds_budget=25.0, keep=PARITY_TREES):
    """The reference CPU learner (oracle/) on all host threads: boosting iterations on the
    full workload until ~seconds_budget of training time is used (at least `keep` + 1).
    Returns the rate, the thread count, the iterations, the seconds, and the first `keep`
    trees with the scores after them and the first iteration's f32 gradients."""
    import oracle

    oracle.build()
    nt = os.cpu_count() or 1
    score = oracle_init_score(workload, data)
    el, iters, trees, score_k, grad0 = 0.0, 0, [], None, None
    while True:
        t0 = time.perf_counter()
        tree, gh = oracle_step(workload, data, score, grad, nt)
        el += time.perf_counter() - t0
        iters += 1
        if iters == 1:
            grad0 = gh
        if iters <= keep:
            trees.append(tree)
        if iters == keep:
            score_k = score.copy()
        if iters > keep and (el >= seconds_budget or iters >= 50):
            break
    return {"rate": iters / el, "threads": nt, "iters": iters, "seconds": el,
            "trees": trees, "score_k": score_k, "grad0": grad0}


def workload_desc(args, data):
    w = WORKLOADS[args.workload]
    q = 0 if data.qb is None else len(data.qb) - 1
    return w["desc"].format(rows=data.rows, queries=q) + f" grad={args.grad}"


def run_reference(args):
    """The reference arm: the oracle port of the reference's CPU learner, timed on all
    host cores. Its data is binned by the oracle's BinMapper; the product library is
    never imported or loaded in this process."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    data = make_data(args.workload, args.rows, binner="oracle")
    import oracle

    oracle.build()
    nt = os.cpu_count() or 1
    score = oracle_init_score(args.workload, data)
    for _ in range(args.warmup):
        oracle_step(args.workload, data, score, args.grad, nt)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle_step(args.workload, data, score, args.grad, nt)
    el = time.perf_counter() - t0
    v = args.steps / el
    w = WORKLOADS[args.workload]
    loaded = sorted({ln.split()[-1] for ln in open("/proc/self/maps")
                     if ln.rstrip().endswith(".so") and ROOT in ln})
    out = {
        "metric": "boosting_iters_per_sec", "value": v, "unit": "iters/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * el / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": workload_desc(args, data), "rows": data.rows,
                   "num_leaves": w["leaves"], "max_bin": w["max_bin"]},
        "cpu_baseline": {"value": v, "unit": "iters/s", "cores": nt, "kind": "port",
                         "sample": f"{args.steps} full boosting iterations on all {data.rows} "
                                   f"rows after {args.warmup} warm-up iterations, {nt} threads "
                                   f"(C++ restatement; reference Rust crates unbuildable "
                                   f"here); data binned by the oracle's BinMapper"},
        "e2e": {"value": v, "unit": "iters/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "repo_libraries_loaded": loaded,
    }
    print(json.dumps(out), flush=True)


def run_ours(args):
    import lightgbm_rs_b200 as lgb
    from lightgbm_rs_b200 import build as libbuild
    from lightgbm_rs_b200 import distributed as D

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        # host plumbing only (barriers, the NCCL id, max over ranks); the data path's
        # exchanges run inside the library
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=900))
    if rank == 0:
        libbuild.build()
        make_data(args.workload, args.rows)  # generates and caches for the other ranks
    if dist:
        dist.barrier()
    assert lgb._lib.device_count() > 0, "no CUDA device"
    data = make_data(args.workload, args.rows)
    w = WORKLOADS[args.workload]
    p = params(args.workload, args.grad)
    p["device"] = local
    # shards: contiguous rows, whole queries for a ranking objective
    if data.qb is not None:
        q0, q1 = D.shard_range(len(data.qb) - 1, world, rank)
        b0, b1 = int(data.qb[q0]), int(data.qb[q1])
        group = data.group[q0:q1]
    else:
        b0, b1 = D.shard_range(data.rows, world, rank)
        group = None
    local_rows = b1 - b0
    shard_bins = np.ascontiguousarray(data.bins[:, b0:b1]) if world > 1 else data.bins
    shard_y = np.ascontiguousarray(data.y[b0:b1])
    comm = D.from_torch(local) if dist else None

    def max_over_ranks(x):
        if not dist:
            return x
        import torch

        t = torch.tensor([float(x)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def barrier():
        if dist:
            dist.barrier()

    def resident_booster(pp, warmup, steps):
        ds_ = lgb.Dataset(bins=shard_bins, mappers=data.mappers, label=shard_y, params=pp,
                          group=group)
        b_ = lgb.Booster(pp, ds_, comm=comm)
        b_.update(warmup)
        barrier()
        done_ = b_.update(steps)
        ms_ = max_over_ranks(b_.last_train_ms())
        assert done_ == steps, f"training stopped early ({done_} of {steps})"
        return ds_, b_, ms_

    # ---- context and modules loaded, then every cached device block released: the
    # end-to-end leg below starts from a cold buffer cache, as a fresh lgb.train does ----
    tiny = lgb.Dataset(bins=np.zeros((data.features, 256), dtype=np.uint8),
                       mappers=data.mappers, label=(np.arange(256) % 2).astype(np.float32),
                       params=p, group=None if group is None else [256])
    # every rank trains one tiny iteration, through the exchange when data-parallel: each
    # kernel variant the job launches is loaded before the timed region
    lgb.train(p, tiny, num_boost_round=1, comm=comm)
    del tiny
    lgb._lib.lib().lgbm_b200_release_cached_memory(-1, None)
    barrier()

    # ---- end to end through the public API from host buffers (cold buffer cache) ----
    t0 = time.perf_counter()
    ds2 = lgb.Dataset(bins=shard_bins, mappers=data.mappers, label=shard_y, params=p,
                      group=group)
    ds2.construct()  # the upload (lgb.train would do it first)
    t1 = time.perf_counter()
    b2 = lgb.Booster(p, ds2, comm=comm)  # device buffers, labels, the iteration's graph
    t2 = time.perf_counter()
    b2.update(args.steps)
    t3 = time.perf_counter()
    trees = b2.trees()
    scores = b2.train_scores()
    t4 = time.perf_counter()
    e2e_s = max_over_ranks(t4 - t0)
    e2e_parts = {"dataset_upload_s": t1 - t0, "booster_create_s": t2 - t1,
                 "train_s": t3 - t2, "readback_s": t4 - t3}
    h2d = shard_bins.nbytes + shard_y.nbytes + (0 if group is None else (len(group) + 1) * 4)
    d2h = scores.nbytes + sum(sum(np.asarray(v).nbytes for k, v in t.items()
                                  if isinstance(v, np.ndarray)) for t in trees)
    del b2, ds2, trees, scores

    # ---- device-resident run: inputs already in HBM when the timed region starts ----
    ds = lgb.Dataset(bins=shard_bins, mappers=data.mappers, label=shard_y, params=p,
                     group=group)
    booster = lgb.Booster(p, ds, comm=comm)
    booster.update(args.warmup)
    barrier()
    with ClockSampler(local) as clk:
        done = booster.update(args.steps)
        dev_ms = booster.last_train_ms()
    barrier()
    assert done == args.steps, f"training stopped early ({done} of {args.steps})"
    dev_ms = max_over_ranks(dev_ms)
    value = args.steps / (dev_ms / 1000.0)
    digest = tree_digest(booster.trees())

    # ---- per-kernel device spans of the pipelined step (same launch sequence, kernels
    # stamping %globaltimer at entry and exit), and the kernels' own work counters ----
    spans, pc = booster.profile_pipeline(5)
    chain = booster.profile_chain()  # the last of those iterations, step by step
    # the part of the split chain that holds the tree longest, and inside the control step
    # its longest phase
    parts = {k: chain[k] for k in ("control_step", "main_partition_past", "build_past",
                                   "lookahead_past", "launch_gap")}
    top = max(parts, key=parts.get)
    ph = chain.get("control_phases") or {}
    chain["limiting_phase"] = {
        "part": top, "ms_per_tree": parts[top],
        "share_of_tree": parts[top] / chain["tree"] if chain["tree"] else None,
        "control_step_phase": max(ph, key=ph.get) if ph else None}
    kb = kernel_bytes(pc, local_rows, args.grad, data.features)
    peak, peak_kind = load_peaks()
    part_ms = spans["partition"] + pc["lookahead"]

    def entry(label, ms, nbytes, traffic_key=None):
        ach = nbytes / (ms / 1000.0) / 1e9 if ms > 0 else 0.0
        e = {"kernel": label, "ms_per_iter": ms, "bytes_per_iter": nbytes, "achieved": ach,
             "frac": ach / peak if peak else None}
        if traffic_key in TRAFFIC_PER_ALGO_BYTE:
            e["traffic_per_iter"] = nbytes * TRAFFIC_PER_ALGO_BYTE[traffic_key]
        return e

    fused = pc["fused"]
    in_ctl = pc.get("rows_parted_ctl", 0) > 0  # main partitions inside the control steps
    cells = 2 * sum(int(m["num_bin"]) for m in data.mappers)
    fix_bytes = pc["splits"] * cells * 8 * 5
    kern = {
        "partition": entry(("k_partition_q4 (row partition + fused child histogram; the "
                            "look-ahead launches and the last split's main partition)")
                           if in_ctl else
                           ("k_partition_q4 (row partition + fused child histogram; main and "
                            "look-ahead launches)") if fused else "k_partition (row partition)",
                           part_ms, kb["partition"], "partition"),
        "build": entry("k_build_q4 (root histogram)" if fused else
                       "k_build / k_build_q4 (histogram build)", spans["build"], kb["build"],
                       "build"),
        "fixscan": entry(("k_fixscan_part (control step: decode, FixHistogram, subtraction, "
                          "threshold scans, pick; L2-resident; and the main partition of the "
                          "splits the look-ahead missed, with its child histogram)") if in_ctl
                         else ("k_fixscan (control step: decode, FixHistogram, subtraction, "
                               "threshold scans, pick; L2-resident)"),
                         spans["fixscan"], fix_bytes + kb["partition_ctl"]),
    }
    kern["fixscan"]["traffic_per_iter"] = (fix_bytes * TRAFFIC_PER_ALGO_BYTE["fixscan"] +
                                           kb["partition_ctl"] *
                                           TRAFFIC_PER_ALGO_BYTE["partition"])
    dom = max(kern, key=lambda k: kern[k]["ms_per_iter"])
    hist = {"root": kern["build"],
            "child_fused": {"bytes_per_iter": kb["child_hist_fused"],
                            "share_of_partition_bytes":
                                kb["child_hist_fused"] / kb["partition"] if kb["partition"]
                                else 0.0}}
    launches_per_step = pc["stamped_launches"] + 10  # + gradient, init, prepare, finish
    del booster

    # ---- the first trees vs the CPU oracle on the same binned data (one device) ----
    extras = {}
    cpu = None
    cpu_res = None
    if world == 1 and not args.no_cpu_baseline:
        cpu_res = cpu_run(args.workload, data, args.grad)
        cpu = {"value": cpu_res["rate"], "unit": "iters/s", "cores": cpu_res["threads"],
               "kind": "port",
               "sample": f"{cpu_res['iters']} full boosting iterations on all {data.rows} rows "
                         f"({cpu_res['seconds']:.1f} s of training), {cpu_res['threads']} "
                         f"threads"}
    if cpu_res is not None and not args.no_extras:
        bp = lgb.Booster(p, ds, comm=comm)
        bp.update(1)
        g0, h0 = bp.last_gradients()
        bp.update(PARITY_TREES - 1)
        got = bp.trees()
        s_dev = bp.train_scores()
        diffs = [trees_equal(a, b) for a, b in zip(got, cpu_res["trees"])]
        gw, hw = cpu_res["grad0"]
        extras["parity"] = {
            "trees": PARITY_TREES, "rows": data.rows,
            "bit_exact": all(d is None for d in diffs) and
            s_dev.tobytes() == cpu_res["score_k"].tobytes(),
            "tree_mismatch": [d for d in diffs],
            "scores_bit_exact": s_dev.tobytes() == cpu_res["score_k"].tobytes(),
            "grad_f32_mismatches_iter0": int(np.sum(g0.view(np.uint32) !=
                                                    gw.astype(np.float32).view(np.uint32)) +
                                             np.sum(h0.view(np.uint32) !=
                                                    hw.astype(np.float32).view(np.uint32))),
            "checked_against": "oracle/ (CPU restatement pinned to the reference's goldens), "
                               "same binned data, both from the initial score"}
        del bp

    # ---- the same workload with f32 gradients, and a full-length run ----
    if not args.no_extras and args.grad == "quantized":
        pf = params(args.workload, "f32")
        pf["device"] = local
        ds_f, bf, ms_f = resident_booster(pf, args.warmup, args.steps)
        extras["f32"] = {"value": args.steps / (ms_f / 1000.0), "unit": "iters/s",
                         "steps": args.steps, "warmup": args.warmup,
                         "ms_per_step": ms_f / args.steps}
        del bf, ds_f
        ps = dict(p, stochastic_rounding=True)
        ds_s, bs, ms_s = resident_booster(ps, args.warmup, args.steps)
        extras["stochastic_rounding"] = {"value": args.steps / (ms_s / 1000.0),
                                         "unit": "iters/s", "steps": args.steps,
                                         "ms_per_step": ms_s / args.steps,
                                         "digest": tree_digest(bs.trees())}
        del bs, ds_s
    if not args.no_extras:
        n_full = w["iterations"]
        bfull = lgb.Booster(p, ds, comm=comm)
        barrier()
        done_full = bfull.update(n_full)
        ms_full = max_over_ranks(bfull.last_train_ms())
        extras["full"] = {"iterations": done_full, "value": done_full / (ms_full / 1000.0),
                          "unit": "iters/s", "ms": ms_full,
                          "digest": tree_digest(bfull.trees())}
        del bfull
    del ds

    par = "single GPU" if world == 1 else (
        f"data-parallel, {world} GPUs: rows sharded, the integer child histogram of every "
        f"split exchanged over peer memory (NCCL when the peers cannot be mapped)")
    out = {
        "metric": "boosting_iters_per_sec",
        "value": value,
        "unit": "iters/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dev_ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int64+f64" if args.grad == "quantized" else "f32+f64",
        "data": "synthetic",
        "config": {"workload": workload_desc(args, data),
                   "rows": data.rows, "rows_per_gpu": local_rows, "features": data.features,
                   "num_leaves": w["leaves"], "max_bin": w["max_bin"], "grad": args.grad,
                   "parallelism": par,
                   "l2": f"inputs larger than L2 (bin matrix "
                         f"{data.rows * ((data.features + 15) // 16 * 16) / 1e6:.0f} MB "
                         f"> 126 MB)" if data.rows * data.features > 126e6 else
                         "bin matrix smaller than L2; no flush between iterations"},
        "roofline": {"bound": "hbm", "kernel": kern[dom]["kernel"],
                     "achieved": kern[dom]["achieved"], "peak": peak, "unit": "GB/s",
                     "frac": kern[dom]["frac"], "peak_kind": peak_kind,
                     "traffic": kern[dom].get("traffic_per_iter"),
                     "traffic_note": "DRAM bytes per iteration of the kernel's launches, like "
                                     "achieved (bytes per iteration / span ms per iteration): "
                                     "its algorithmic bytes times the DRAM/algorithmic ratio "
                                     "of the 5M-row ncu captures in profiles/"
                                     "tree_kernels_dram_traffic_c1_5M.md",
                     "algorithmic_bytes_per_iter": kern[dom]["bytes_per_iter"],
                     "ms_per_iter": kern[dom]["ms_per_iter"],
                     "timing": "device spans (%globaltimer, first CTA entry to last CTA exit) "
                               "of each launch in a CUDA graph of the training pipeline, "
                               "look-ahead stream included; mean of 5 iterations",
                     "pipeline_ms_per_iter": pc["ms_per_iter"],
                     "kernels": kern,
                     "histogram": hist,
                     "rows_parted_per_iter": pc["rows_parted"],
                     "rows_built_per_iter": pc["rows_built"],
                     "splits_per_iter": pc["splits"],
                     "lookahead_runs_per_iter": pc["lookahead_runs"],
                     "lookahead_hits_per_iter": pc["lookahead_hits"],
                     "chain": chain},
        "kernel_span_ms_per_iter": spans,
        "cpu_baseline": cpu,
        "e2e": {"value": args.steps / e2e_s, "unit": "iters/s",
                "h2d_bytes_per_step": h2d / args.steps, "d2h_bytes_per_step": d2h / args.steps,
                "parts_rank0": e2e_parts,
                "note": "lgb.train from host bins+labels: upload, K iterations, model+scores "
                        "readback (binning excluded on both arms); run first, with the "
                        "library's device-buffer cache emptied (cold)"},
        "digest": digest,
        "gpu_launches": int(round(launches_per_step * args.steps)),
        "clocks": clk.summary(),
    }
    out.update(extras)
    if comm is not None:
        comm.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def run_binning(args):
    """Binning of the C1 raw matrix on the device against the host on all cores: bin
    finding (find_bin_from_column on each column's 200k-row sample; find_bins against
    bin_column), and value_to_bin into the row-major u8 matrix (f32 feature-major upload
    + k_bin_rows, against the host's value_to_bin of the same mappers)."""
    import concurrent.futures as cf

    import lightgbm_rs_b200 as lgb
    from lightgbm_rs_b200 import build as libbuild

    synthetic = load_synthetic()
    libbuild.build()
    X, y = synthetic.binary_c0(num_data=args.rows, num_features=28, seed=0)
    p = {"max_bin": 255, "min_data_in_leaf": 100, "feature_pre_filter": False}
    t0 = time.perf_counter()
    ds = lgb.Dataset(X, y, p)  # mappers from the samples (device; first CUDA use: context)
    t_map = time.perf_counter() - t0
    kw = ds._bin_kwargs()
    cols = list(ds._values)
    # bin finding (find_bin_from_column of every column's sample), device and host, warm
    find_dev = []
    for _ in range(max(args.steps, 1)):
        t0 = time.perf_counter()
        dev_maps = lgb.find_bins(cols, **kw)
        find_dev.append(time.perf_counter() - t0)
    nt = os.cpu_count() or 1
    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(max_workers=nt) as ex:
        host_maps = list(ex.map(lambda c: lgb.bin_column(c, want_bins=False, **kw)[0], cols))
    t_find_host = time.perf_counter() - t0
    maps_same = all(a["num_bin"] == b["num_bin"] and a["default_bin"] == b["default_bin"]
                    and np.asarray(a["upper"]).tobytes() == np.asarray(b["upper"]).tobytes()
                    for a, b in zip(dev_maps, host_maps))
    dev_s = []
    for _ in range(max(args.steps, 1)):
        ds._handle = None
        t0 = time.perf_counter()
        ds.construct()
        dev_s.append(time.perf_counter() - t0)
        lgb._lib.lib().lgbm_b200_dataset_destroy(ds._handle)
        ds._handle = None
    ds.construct()
    dev_bins = ds.device_bins()
    t0 = time.perf_counter()

    def one(j):
        return lgb.bin_column(ds._values[j], **kw)[1]

    with cf.ThreadPoolExecutor(max_workers=nt) as ex:
        host = list(ex.map(one, range(ds.num_features)))
    t_host = time.perf_counter() - t0
    same = all(np.array_equal(dev_bins[j], host[j]) for j in range(ds.num_features))
    vals = args.rows * 28
    dev = min(dev_s)
    out = {"metric": "binning_values_per_sec", "value": vals / dev, "unit": "values/s",
           "impl": "ours", "data": "synthetic", "dtype": "f32",
           "config": {"workload": f"C1 raw values {args.rows}x28 f32, max_bin=255"},
           "device_s": dev, "host_value_to_bin_s": t_host, "host_threads": nt,
           "host_note": "host time includes each column's find_bin on its sample",
           "dataset_with_context_s": t_map, "bins_identical": bool(same),
           "find_bins_device_s": min(find_dev), "find_bins_host_s": t_find_host,
           "mappers_identical": bool(maps_same),
           "h2d_bytes": vals * 4}
    print(json.dumps(out), flush=True)


def run_profile_case(args):
    """The capture case of the committed ncu summaries: W warm-up iterations through the
    training graph, then one iteration whose kernels run one at a time
    (Booster.profile_iteration), with the algorithmic bytes of that iteration's launches.
    Skip 761 x W tree-kernel launches (C1: 1 root build + 254 control steps + 254 main
    and 252 look-ahead partitions per iteration) to capture the profiled iteration."""
    import lightgbm_rs_b200 as lgb
    from lightgbm_rs_b200 import build as libbuild

    libbuild.build()
    data = make_data(args.workload, args.rows)
    p = params(args.workload, args.grad)
    ds = lgb.Dataset(bins=data.bins, mappers=data.mappers, label=data.y, params=p,
                     group=data.group)
    b = lgb.Booster(p, ds)
    b.update(args.warmup)
    kms, counts = b.profile_iteration()
    kb = kernel_bytes(counts, data.rows, args.grad, data.features)
    launches = b.profile_launches()
    per = {}
    for cls, ms in launches:
        e = per.setdefault(cls, {"launches": 0, "ms": 0.0})
        e["launches"] += 1
        e["ms"] += ms
    print(json.dumps({"measure": "profile", "workload": workload_desc(args, data),
                      "warmup": args.warmup, "counts": counts, "algorithmic_bytes": kb,
                      "event_ms_by_class": kms, "launches_by_class": per}), flush=True)


def run_atomics(args):
    """Shared-memory atomic ceiling of the root build k_build_q4, measured with the kernel
    itself. The build adds one packed 32-bit atomic per (row, feature) into cell
    (feature << 8) + bin; a warp's lanes take consecutive rows, so the bin pattern decides
    the bank conflicts of each warp-wide atomic:
      lanes   bin = row % 32: every lane its own bank (conflict-free, distinct cells)
      random  uniform bins over 256 (the C1 matrix's quantile bins are close to this)
      c1      the C1 matrix itself
      same    every row bin 0: all lanes on one cell
      skewed  bin 0 for 90 % of rows, uniform otherwise (a heavily skewed feature)
    Each pattern runs with one atomic per (row, feature) and with warp-aggregated atomics
    (LGBM_B200_WARP_AGG=1: lanes with the same bin summed with __match_any_sync and
    __reduce_add_sync, one atomic per group).
    The first boosting iteration of a fresh booster (binary, from the initial score: a
    constant hessian, so exactly F atomics per row); the root build's device span comes
    from the pipeline stamps, best of `--steps` boosters."""
    import lightgbm_rs_b200 as lgb
    from lightgbm_rs_b200 import build as libbuild

    libbuild.build()
    n, F = args.rows, 28
    rng = np.random.default_rng(0)
    y = (rng.random(n) < 0.5).astype(np.float32)
    mappers = [{"num_bin": 256, "default_bin": 0, "most_freq_bin": 0, "missing_type": 0,
                "bin_type": 0, "upper": np.arange(256, dtype=np.float64) + 0.5,
                "is_trivial": False} for _ in range(F)]
    rows = np.arange(n, dtype=np.int64)
    patterns = {
        "lanes": lambda f: ((rows + 7 * f) % 32).astype(np.uint8),
        "random": lambda f: rng.integers(0, 256, n).astype(np.uint8),
        "same": lambda f: np.zeros(n, dtype=np.uint8),
        "skewed": lambda f: np.where(rng.random(n) < 0.9, 0,
                                     rng.integers(0, 256, n)).astype(np.uint8),
    }
    out = {"measure": "atomics", "rows": n, "features": F, "patterns": {}}
    p = {"objective": "binary", "num_leaves": 2, "min_data_in_leaf": 100,
         "learning_rate": 0.1, "use_quantized_grad": True, "num_grad_quant_bins": 4,
         "stochastic_rounding": False}
    sources = list(patterns.items())
    if n == WORKLOADS["c1"]["rows"]:
        c1 = make_data("c1", n)
        sources.append(("c1", lambda f: c1.bins[f]))
        y_c1 = c1.y
    for name, gen in sources:
        bins = np.ascontiguousarray(np.stack([gen(f) for f in range(F)]))
        lab = y_c1 if name == "c1" else y
        maps = c1.mappers if name == "c1" else mappers
        ds = lgb.Dataset(bins=bins, mappers=maps, label=lab, params=p)
        for agg in ("0", "1"):
            os.environ["LGBM_B200_WARP_AGG"] = agg
            ms = []
            digests = set()
            for _ in range(max(3, args.steps)):
                # the first iteration of a fresh booster: constant hessian, F atomics per row
                b = lgb.Booster(p, ds)
                spans, _ = b.profile_pipeline(1)
                ms.append(spans["build"])
                digests.add(tree_digest(b.trees()))
                del b
            t = min(ms)
            out["patterns"][name + ("_warp_aggregated" if agg == "1" else "")] = {
                "build_ms": t, "atomics_per_s": n * F / (t / 1e3),
                "atomics_per_sm_clock_at_1965mhz": n * F / (t / 1e3) / (148 * 1.965e9),
                "bytes_per_s": n * (F + 2) / (t / 1e3), "tree_digests": sorted(digests)}
        os.environ.pop("LGBM_B200_WARP_AGG", None)
        del ds
    print(json.dumps(out), flush=True)


def main():
    args = parse()
    if args.warmup < 3:
        args.warmup = 3
    if args.measure == "binning":
        run_binning(args)
        return
    if args.measure == "profile":
        run_profile_case(args)
        return
    if args.measure == "atomics":
        run_atomics(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
