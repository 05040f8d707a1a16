"""Benchmark: boosting iterations/s of the B200 histogram tree learner.

Default workload C1: 10,500,000 rows x 28 dense features from
the configs[0] generator (seeded synthetic: no public dataset is named), max_bin=255,
num_leaves=255, min_data_in_leaf=100, objective=binary, learning_rate=0.1.
Default gradients: use_quantized_grad with 4 quantization bins (`--grad f32` for the
f32-gradient variant). One step = one boosting iteration (gradients, quantization,
one tree, shrinkage, score update) over all rows.

`--workload c3`: 2,000,000 rows, 90 numeric features with 10 % NaN and 10 categorical
features, L2 regression, 63 leaves. `--workload c4`: lambdarank over 20,000 queries
(about 473k rows) x 700 sparse features, 255 leaves. Both are seeded synthetic
stand-ins with the configurations' shapes (lightgbm_rs_b200/synthetic.py).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload c1|c3|c4] [--grad quantized|f32]

Prints ONE JSON line on rank 0. `--impl reference` times the reference CPU learner
(the C++ restatement in oracle/, the reference's Rust crates cannot be built here)
on the host cores.
"""

import argparse
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

# name -> rows, features, leaves, min_data_in_leaf, objective, description
WORKLOADS = {
    "c1": dict(rows=10_500_000, features=28, leaves=255, min_data=100, objective="binary",
               desc="C1 binary {rows}x28 num_leaves=255 min_data_in_leaf=100 max_bin=255"),
    "c3": dict(rows=2_000_000, features=100, leaves=63, min_data=20, objective="regression",
               desc="C3 l2 {rows}x100 (90 numeric, 10% NaN; 10 categorical, 16-240 "
                    "categories, Zipf 1.2) num_leaves=63 max_bin=255"),
    "c4": dict(rows=473_000, features=700, leaves=255, min_data=20, objective="lambdarank",
               desc="C4 lambdarank {rows} rows / {queries} queries x700 (80% zeros) "
                    "num_leaves=255 max_bin=255"),
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
    ap.add_argument("--measure", default="boosting", choices=["boosting", "binning"],
                    help="binning: time Dataset construction from raw C1 values (device "
                         "value_to_bin) against host value_to_bin on all cores")
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


class Data:
    """A binned workload: feature-major bins, mappers, labels, query sizes (ranking)."""

    def __init__(self, bins, mappers, y, group=None):
        self.bins, self.mappers, self.y, self.group = bins, mappers, y, group
        self.rows = bins.shape[1]
        self.features = bins.shape[0]
        self.qb = None if group is None else \
            np.concatenate([[0], np.cumsum(group)]).astype(np.int32)


def make_data(workload, rows, seed=0):
    """Seeded synthetic data of the workload, binned with the reference BinMapper (host).

    The binned result is cached under the system temp directory so repeated runs on
    one machine skip generation (the cache is keyed by workload, rows and seed)."""
    import concurrent.futures as cf
    import pickle
    import tempfile

    import lightgbm_rs_b200 as lgb
    from lightgbm_rs_b200 import synthetic

    cache = os.path.join(tempfile.gettempdir(), f"lgbm_b200_{workload}_{rows}_{seed}.pkl")
    if os.path.exists(cache):
        with open(cache, "rb") as f:
            return pickle.load(f)
    w = WORKLOADS[workload]
    group, cats = None, []
    if workload == "c1":
        X, y = synthetic.binary_c0(num_data=rows, num_features=w["features"], seed=seed)
    elif workload == "c3":
        X, y, cats = synthetic.mixed_c3(num_data=rows, seed=seed)
    else:
        X, y, group = synthetic.rank_c4(num_queries=max(1, round(rows / 23.65)),
                                        num_features=w["features"], seed=seed)
    F = X.shape[1]
    mappers = [None] * F
    bins = np.empty((F, X.shape[0]), dtype=np.uint8)

    def one(j):
        m, b = lgb.bin_column(X[:, j], max_bin=255, min_data_in_leaf=w["min_data"],
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
         "min_data_in_leaf": w["min_data"], "learning_rate": LEARNING_RATE, "max_bin": 255}
    if grad == "quantized":
        p.update(use_quantized_grad=True, num_grad_quant_bins=4)
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
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
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
    the split-feature byte and the index it has already read."""
    s_gh = 2 if grad == "quantized" else 8
    F = features
    rp, rb = counts["rows_parted"], counts["rows_built"]
    part = rp * 5 + max(rp - rows, 0) * 4
    root_build = rows * (F + s_gh)
    child_rows = max(rb - rows, 0)
    if counts["fused"]:
        part += child_rows * (F - 1 + s_gh)
        build = root_build
    else:
        build = root_build + child_rows * (F + s_gh + 4)
    return {"partition": part, "build": build, "bin_bytes": rb * F + rp}


def oracle_step(workload, data, score, grad, nt):
    """One boosting iteration of the reference CPU learner (oracle/) on `score` in place."""
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
    if grad == "quantized":
        g, h, _, _ = oracle.quantize(g, h, 4)
    tree, part, _ = oracle.grow_tree(data.bins, metas, g, h, w["leaves"], -1, nt,
                                     min_data_in_leaf=w["min_data"])
    oracle.tree_shrinkage(tree, LEARNING_RATE)
    oracle.add_prediction_to_score(tree, part, score)


def oracle_init_score(workload, data):
    import oracle

    obj = WORKLOADS[workload]["objective"]
    init = 0.0 if obj == "lambdarank" else oracle.boost_from_score(obj, data.y)
    return np.full(data.rows, init, dtype=np.float64)


def cpu_baseline(workload, data, grad, seconds_budget=25.0):
    """The reference CPU learner (oracle/) on the host: boosting iterations on the full
    workload until ~seconds_budget is used (at least one)."""
    import oracle

    oracle.build()
    nt = os.cpu_count() or 1
    score = oracle_init_score(workload, data)
    t0 = time.perf_counter()
    iters = 0
    while True:
        oracle_step(workload, data, score, grad, nt)
        iters += 1
        el = time.perf_counter() - t0
        if el >= seconds_budget or iters >= 50:
            break
    return iters / el, nt, iters, el


def workload_desc(args, data):
    w = WORKLOADS[args.workload]
    q = 0 if data.qb is None else len(data.qb) - 1
    return w["desc"].format(rows=data.rows, queries=q) + f" grad={args.grad}"


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    data = make_data(args.workload, args.rows)
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
    out = {
        "metric": "boosting_iters_per_sec", "value": v, "unit": "iters/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * el / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": workload_desc(args, data), "rows": data.rows,
                   "num_leaves": w["leaves"], "max_bin": 255},
        "cpu_baseline": {"value": v, "unit": "iters/s", "cores": nt, "kind": "port",
                         "sample": f"{args.steps} full boosting iterations on all {data.rows} "
                                   f"rows, {nt} threads (C++ restatement; reference Rust "
                                   f"crates unbuildable here)"},
        "e2e": {"value": v, "unit": "iters/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
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
        # all-reduces run inside the library on its own NCCL communicator
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
    shard_bins = data.bins[:, b0:b1] if world > 1 else data.bins
    shard_y = data.y[b0:b1]
    comm = D.from_torch(local) if dist else None

    def max_over_ranks(x):
        if not dist:
            return x
        import torch

        t = torch.tensor([float(x)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident run: inputs already in HBM when the timed region starts ----
    ds = lgb.Dataset(bins=shard_bins, mappers=data.mappers, label=shard_y, params=p,
                     group=group)
    booster = lgb.Booster(p, ds, comm=comm)
    booster.update(args.warmup)
    if dist:
        dist.barrier()
    with ClockSampler(local) as clk:
        done = booster.update(args.steps)
        dev_ms = booster.last_train_ms()
    if dist:
        dist.barrier()
    assert done == args.steps, f"training stopped early ({done} of {args.steps})"
    dev_ms = max_over_ranks(dev_ms)
    value = args.steps / (dev_ms / 1000.0)

    # ---- per-kernel timing of one more iteration (CUDA events on the library stream) ----
    kms, counts = booster.profile_iteration()
    kb = kernel_bytes(counts, local_rows, args.grad, data.features)
    peak, peak_kind = load_peaks()
    per_kernel = {}
    for cls, label in (("partition", "k_partition_q4 (partition + child histogram)"
                        if counts["fused"] else "k_partition (row partition)"),
                       ("build", "k_build_q4 (root histogram)" if counts["fused"]
                        else "k_build / k_build_q4 (histogram build)")):
        ms = kms[cls]
        ach = kb[cls] / (ms / 1000.0) / 1e9 if ms > 0 else 0.0
        per_kernel[cls] = {"kernel": label, "ms_per_iter": ms, "bytes_per_iter": kb[cls],
                           "achieved": ach, "frac": ach / peak if peak else None}
    dom = max(per_kernel, key=lambda k: per_kernel[k]["ms_per_iter"])
    launches_per_step = counts["launches"]
    del booster

    # ---- end to end through the public API from host buffers ----
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    ds2 = lgb.Dataset(bins=shard_bins, mappers=data.mappers, label=shard_y, params=p,
                      group=group)
    b2 = lgb.train(p, ds2, num_boost_round=args.steps, comm=comm)
    trees = b2.trees()
    scores = b2.train_scores()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    h2d = np.ascontiguousarray(shard_bins).nbytes + shard_y.nbytes + \
        (0 if group is None else (len(group) + 1) * 4)
    d2h = scores.nbytes + sum(sum(np.asarray(v).nbytes for k, v in t.items()
                                  if isinstance(v, np.ndarray)) for t in trees)
    del b2, ds2

    cpu = None
    if not args.no_cpu_baseline and world == 1:
        v, cores, iters, el = cpu_baseline(args.workload, data, args.grad)
        cpu = {"value": v, "unit": "iters/s", "cores": cores, "kind": "port",
               "sample": f"{iters} full boosting iterations on all {data.rows} rows "
                         f"({el:.1f} s), {cores} threads"}

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
                   "num_leaves": w["leaves"], "grad": args.grad, "parallelism": par,
                   "l2": f"inputs larger than L2 (bin matrix "
                         f"{data.rows * ((data.features + 15) // 16 * 16) / 1e6:.0f} MB "
                         f"> 126 MB)"},
        "roofline": {"bound": "hbm", "kernel": per_kernel[dom]["kernel"],
                     "achieved": per_kernel[dom]["achieved"], "peak": peak, "unit": "GB/s",
                     "frac": per_kernel[dom]["frac"], "peak_kind": peak_kind, "traffic": None,
                     "algorithmic_bytes_per_iter": per_kernel[dom]["bytes_per_iter"],
                     "ms_per_iter": per_kernel[dom]["ms_per_iter"],
                     "other_kernels": {k: v for k, v in per_kernel.items() if k != dom},
                     "rows_parted_per_iter": counts["rows_parted"],
                     "rows_built_per_iter": counts["rows_built"],
                     "builds_per_iter": counts["builds"], "splits_per_iter": counts["splits"],
                     "lookahead_runs_per_iter": counts.get("lookahead_runs", 0),
                     "lookahead_hits_per_iter": counts.get("lookahead_hits", 0)},
        "kernel_ms_per_iter": kms,
        "cpu_baseline": cpu,
        "e2e": {"value": args.steps / e2e_s, "unit": "iters/s",
                "h2d_bytes_per_step": h2d / args.steps, "d2h_bytes_per_step": d2h / args.steps,
                "note": "lgb.train from host bins+labels: upload, K iterations, model+scores "
                        "readback (binning excluded on both arms)"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    if comm is not None:
        comm.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def run_binning(args):
    """Device binning of the C1 raw matrix (f32, feature-major upload + value_to_bin into
    the row-major u8 matrix) against the host value_to_bin of the same mappers on all
    cores. Bin boundaries come from each column's 200k-row sample on the host in both."""
    import concurrent.futures as cf

    import lightgbm_rs_b200 as lgb
    from lightgbm_rs_b200 import build as libbuild
    from lightgbm_rs_b200 import synthetic

    libbuild.build()
    X, y = synthetic.binary_c0(num_data=args.rows, num_features=28, seed=0)
    p = {"max_bin": 255, "min_data_in_leaf": 100}
    t0 = time.perf_counter()
    ds = lgb.Dataset(X, y, p)  # mappers from the samples (host)
    t_map = time.perf_counter() - t0
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
    nt = os.cpu_count() or 1
    kw = ds._bin_kwargs()
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
           "mapper_s": t_map, "bins_identical": bool(same),
           "h2d_bytes": vals * 4}
    print(json.dumps(out), flush=True)


def main():
    args = parse()
    if args.warmup < 3:
        args.warmup = 3
    if args.measure == "binning":
        run_binning(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
