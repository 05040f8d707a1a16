"""ctypes binding of the CPU restatement in oracle/oracle.cpp.

TEST INFRASTRUCTURE ONLY: the parity checker for lightgbm_rs_b200. Only
tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg import this
module. The product path (lightgbm_rs_b200) never imports or calls it.
"""

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


class GainConfig(ctypes.Structure):
    _fields_ = [
        ("min_data_in_leaf", ctypes.c_int32),
        ("_pad", ctypes.c_int32),
        ("min_sum_hessian_in_leaf", ctypes.c_double),
        ("max_delta_step", ctypes.c_double),
        ("lambda_l1", ctypes.c_double),
        ("lambda_l2", ctypes.c_double),
        ("min_gain_to_split", ctypes.c_double),
        ("path_smooth", ctypes.c_double),
        ("parent_output", ctypes.c_double),
        ("min_data_per_group", ctypes.c_int32),
        ("max_cat_threshold", ctypes.c_int32),
        ("max_cat_to_onehot", ctypes.c_int32),
        ("_pad2", ctypes.c_int32),
        ("cat_l2", ctypes.c_double),
        ("cat_smooth", ctypes.c_double),
    ]


class SplitInfo(ctypes.Structure):
    _fields_ = [
        ("threshold", ctypes.c_uint32),
        ("default_left", ctypes.c_int32),
        ("left_count", ctypes.c_int32),
        ("right_count", ctypes.c_int32),
        ("gain", ctypes.c_double),
        ("left_sum_gradient", ctypes.c_double),
        ("left_sum_hessian", ctypes.c_double),
        ("right_sum_gradient", ctypes.c_double),
        ("right_sum_hessian", ctypes.c_double),
        ("left_output", ctypes.c_double),
        ("right_output", ctypes.c_double),
    ]


class FeatureMeta(ctypes.Structure):
    _fields_ = [
        ("num_bin", ctypes.c_int32),
        ("offset", ctypes.c_int32),
        ("default_bin", ctypes.c_int32),
        ("most_freq_bin", ctypes.c_int32),
        ("missing_type", ctypes.c_int32),
        ("is_categorical", ctypes.c_int32),
    ]


class LearnerConfig(ctypes.Structure):
    _fields_ = [
        ("num_leaves", ctypes.c_int32),
        ("max_depth", ctypes.c_int32),
        ("gain", GainConfig),
    ]


_P = ctypes.c_void_p


class OracleBinMapper(ctypes.Structure):
    _fields_ = [("num_bin", ctypes.c_int32), ("missing_type", ctypes.c_int32),
                ("default_bin", ctypes.c_int32), ("most_freq_bin", ctypes.c_int32),
                ("is_trivial", ctypes.c_int32), ("is_categorical", ctypes.c_int32),
                ("min_val", ctypes.c_double), ("max_val", ctypes.c_double),
                ("sparse_rate", ctypes.c_double)]


class Tree(ctypes.Structure):
    _fields_ = [
        ("num_leaves", ctypes.c_int32),
        ("_pad", ctypes.c_int32),
        ("left_child", _P),
        ("right_child", _P),
        ("split_feature", _P),
        ("threshold_bin", _P),
        ("split_gain", _P),
        ("decision_type", _P),
        ("leaf_value", _P),
        ("leaf_weight", _P),
        ("leaf_count", _P),
        ("internal_value", _P),
        ("internal_count", _P),
        ("leaf_depth", _P),
        ("leaf_parent", _P),
        ("cat_bins", _P),
    ]


TREE_ARRAYS = [
    ("left_child", np.int32, -1),
    ("right_child", np.int32, -1),
    ("split_feature", np.int32, -1),
    ("threshold_bin", np.uint32, -1),
    ("split_gain", np.float32, -1),
    ("decision_type", np.int8, -1),
    ("leaf_value", np.float64, 0),
    ("leaf_weight", np.float64, 0),
    ("leaf_count", np.int32, 0),
    ("internal_value", np.float64, -1),
    ("internal_count", np.int32, -1),
    ("leaf_depth", np.int32, 0),
    ("leaf_parent", np.int32, 0),
]

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.oracle_construct_histogram.argtypes = [_P, _P, _P, ctypes.c_int64, ctypes.c_uint32, _P]
        L.oracle_construct_leaf_histogram.argtypes = [
            _P, _P, ctypes.c_int64, _P, _P, ctypes.c_uint32, _P]
        L.oracle_find_best_split.argtypes = [
            _P, ctypes.POINTER(GainConfig), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
            ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_double, ctypes.c_double,
            ctypes.c_int32, ctypes.POINTER(SplitInfo)]
        L.oracle_find_best_split.restype = ctypes.c_int
        L.oracle_subtract.argtypes = [_P, _P, ctypes.c_int64, _P]
        L.oracle_fix_histogram.argtypes = [_P, ctypes.c_int32, ctypes.c_int32, ctypes.c_double,
                                           ctypes.c_double]
        L.oracle_compact_histogram.argtypes = [_P, ctypes.c_int32, ctypes.c_int32]
        L.oracle_partition.argtypes = [_P, _P, ctypes.c_int64, ctypes.c_uint32, ctypes.c_uint32,
                                       ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                       ctypes.c_int32, ctypes.c_int32]
        L.oracle_partition.restype = ctypes.c_int64
        L.oracle_partition_missing.argtypes = [_P, _P, ctypes.c_int64] + [ctypes.c_uint32] * 5 + [
            ctypes.c_int32, ctypes.c_int32]
        L.oracle_partition_missing.restype = ctypes.c_int64
        L.oracle_grow_tree.argtypes = [
            _P, ctypes.c_int32, ctypes.c_int64, ctypes.c_int32, _P, _P, _P,
            ctypes.POINTER(LearnerConfig), ctypes.c_int32, ctypes.POINTER(Tree), _P, _P, _P, _P]
        L.oracle_grow_tree.restype = ctypes.c_int32
        L.oracle_binary_gradients.argtypes = [_P, _P, ctypes.c_int64, ctypes.c_double, _P, _P,
                                              ctypes.c_int32]
        L.oracle_l2_gradients.argtypes = [_P, _P, ctypes.c_int64, _P, _P, ctypes.c_int32]
        L.oracle_lambdarank_gradients.argtypes = [
            _P, _P, ctypes.c_int64, _P, ctypes.c_int32, ctypes.c_double, ctypes.c_int32,
            ctypes.c_int32, _P, ctypes.c_int32, _P, _P, ctypes.c_int32]
        L.oracle_lambdarank_gradients.restype = ctypes.c_int32
        L.oracle_predict_raw.argtypes = [ctypes.c_int32, ctypes.c_int32] + [_P] * 11 + [
            ctypes.c_int64, _P]
        L.oracle_binary_boost_from_score.argtypes = [_P, ctypes.c_int64, ctypes.c_double]
        L.oracle_binary_boost_from_score.restype = ctypes.c_double
        L.oracle_l2_boost_from_score.argtypes = [_P, ctypes.c_int64]
        L.oracle_l2_boost_from_score.restype = ctypes.c_double
        L.oracle_quantize.argtypes = [_P, _P, ctypes.c_int64, ctypes.c_int32, _P, _P]
        L.oracle_quantize_ex.argtypes = [_P, _P, ctypes.c_int64, ctypes.c_int32, _P, _P,
                                         ctypes.c_int32, ctypes.c_uint64]
        L.oracle_tree_shrinkage.argtypes = [_P, ctypes.c_int32, _P, ctypes.c_double]
        L.oracle_add_prediction_to_score.argtypes = [_P, ctypes.c_int32, _P, _P, _P, _P]
        L.oracle_max_threads.restype = ctypes.c_int32
        L.oracle_bin_column.argtypes = [_P, ctypes.c_int64] + [ctypes.c_int32] * 9 + [
            ctypes.POINTER(OracleBinMapper), _P, _P, ctypes.c_int32, _P]
        L.oracle_bin_column.restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def gain_config(min_data_in_leaf=20, min_sum_hessian_in_leaf=1e-3, max_delta_step=0.0,
                lambda_l1=0.0, lambda_l2=0.0, min_gain_to_split=0.0, path_smooth=0.0,
                parent_output=0.0, min_data_per_group=100, max_cat_threshold=32,
                max_cat_to_onehot=4, cat_l2=10.0, cat_smooth=10.0):
    return GainConfig(int(min_data_in_leaf), 0, float(min_sum_hessian_in_leaf),
                      float(max_delta_step), float(lambda_l1), float(lambda_l2),
                      float(min_gain_to_split), float(path_smooth), float(parent_output),
                      int(min_data_per_group), int(max_cat_threshold), int(max_cat_to_onehot),
                      0, float(cat_l2), float(cat_smooth))


def bin_column(values, max_bin=255, min_data_in_bin=3, min_data_in_leaf=20, pre_filter=False,
               use_missing=True, zero_as_missing=False, bin_construct_sample_cnt=200000,
               data_random_seed=1, want_bins=True, categorical=False):
    """The reference's BinMapper::find_bin_from_column + value_to_bin
    (crates/lgbm-dataset/src/bin_mapper.rs:642-675, 148-199), restated in bin_mapper.cpp.
    Returns (mapper dict, bins u32 or None) with the keys the learner needs."""
    col = np.ascontiguousarray(values, dtype=np.float64)
    cap = max(int(max_bin) + 2, 4)
    if categorical:
        cap = max(cap, min(len(col), 1 << 20) + 2)
    upper = np.zeros(cap, dtype=np.float64)
    b2c = np.zeros(cap, dtype=np.int32)
    bins = np.empty(len(col), dtype=np.uint32) if want_bins else None
    m = OracleBinMapper()
    rc = lib().oracle_bin_column(_ptr(col), len(col), int(max_bin), int(min_data_in_bin),
                                 int(min_data_in_leaf), int(bool(pre_filter)),
                                 int(bool(use_missing)), int(bool(zero_as_missing)),
                                 int(bin_construct_sample_cnt), int(data_random_seed),
                                 int(bool(categorical)), ctypes.byref(m), _ptr(upper), _ptr(b2c),
                                 cap, _ptr(bins))
    if rc != 0:
        raise RuntimeError("oracle_bin_column: bin capacity too small")
    mapper = {"num_bin": m.num_bin, "missing_type": m.missing_type,
              "default_bin": m.default_bin, "most_freq_bin": m.most_freq_bin,
              "is_trivial": bool(m.is_trivial), "min_val": m.min_val, "max_val": m.max_val,
              "sparse_rate": m.sparse_rate, "bin_type": 1 if categorical else 0}
    if categorical:
        mapper["bin_to_category"] = b2c[: m.num_bin].copy()
    else:
        mapper["upper"] = upper[: m.num_bin].copy()
    return mapper, bins


def construct_histogram(bins, g, h, num_bin):
    bins = np.ascontiguousarray(bins, dtype=np.uint32)
    g = np.ascontiguousarray(g, dtype=np.float32)
    h = np.ascontiguousarray(h, dtype=np.float32)
    out = np.empty(2 * num_bin, dtype=np.float64)
    lib().oracle_construct_histogram(_ptr(bins), _ptr(g), _ptr(h), len(bins), num_bin, _ptr(out))
    return out


def construct_leaf_histogram(bins, rows, g, h, num_bin):
    bins = np.ascontiguousarray(bins, dtype=np.uint32)
    rows = np.ascontiguousarray(rows, dtype=np.uint32)
    g = np.ascontiguousarray(g, dtype=np.float32)
    h = np.ascontiguousarray(h, dtype=np.float32)
    out = np.empty(2 * num_bin, dtype=np.float64)
    lib().oracle_construct_leaf_histogram(_ptr(bins), _ptr(rows), len(rows), _ptr(g), _ptr(h),
                                          num_bin, _ptr(out))
    return out


def find_best_split(hist, cfg, num_bin, offset, default_bin, skip_default_bin, na_as_missing,
                    run_forward, sum_gradient, sum_hessian, num_data):
    hist = np.ascontiguousarray(hist, dtype=np.float64)
    out = SplitInfo()
    rc = lib().oracle_find_best_split(_ptr(hist), ctypes.byref(cfg), num_bin, offset, default_bin,
                                      int(skip_default_bin), int(na_as_missing), int(run_forward),
                                      float(sum_gradient), float(sum_hessian), int(num_data),
                                      ctypes.byref(out))
    if rc != 0:
        raise ValueError("oracle_find_best_split rejected its inputs")
    return out


def subtract(parent, child):
    parent = np.ascontiguousarray(parent, dtype=np.float64)
    child = np.ascontiguousarray(child, dtype=np.float64)
    out = np.empty_like(parent)
    lib().oracle_subtract(_ptr(parent), _ptr(child), len(parent), _ptr(out))
    return out


def partition(bins_of_rows, rows, num_bin, min_bin, max_bin, threshold, most_freq_bin,
              na_as_missing=False, default_left=False):
    b = np.ascontiguousarray(bins_of_rows, dtype=np.uint32)
    r = np.array(rows, dtype=np.uint32)
    left = lib().oracle_partition(_ptr(b), _ptr(r), len(r), num_bin, min_bin, max_bin, threshold,
                                  most_freq_bin, int(na_as_missing), int(default_left))
    return r, int(left)


def partition_missing(bins_of_rows, rows, min_bin, max_bin, threshold, most_freq_bin,
                      default_bin, missing_type, default_left):
    """The kernel partition with the missing-value routing fan-out
    (partition_leaf_stable, lgbm-compute/src/kernels/data_partition.rs:487)."""
    b = np.ascontiguousarray(bins_of_rows, dtype=np.uint32)
    r = np.array(rows, dtype=np.uint32)
    left = lib().oracle_partition_missing(_ptr(b), _ptr(r), len(r), min_bin, max_bin,
                                          threshold, most_freq_bin, default_bin,
                                          int(missing_type), int(default_left))
    return r, int(left)


def feature_metas(metas):
    """metas: list of dicts with num_bin, default_bin, most_freq_bin, missing_type."""
    arr = (FeatureMeta * len(metas))()
    for i, m in enumerate(metas):
        mfb = int(m["most_freq_bin"])
        arr[i] = FeatureMeta(int(m["num_bin"]), 1 if mfb == 0 else 0, int(m["default_bin"]), mfb,
                             int(m.get("missing_type", 0)), int(m.get("bin_type", 0)))
    return arr


def grow_tree(bins_cols, metas, g, h, num_leaves, max_depth=-1, nthreads=1, **gain_kw):
    """Grow one tree. bins_cols: 2-D array [num_features, num_data] (u8/u16/u32)."""
    bins_cols = np.ascontiguousarray(bins_cols)
    F, N = bins_cols.shape
    if F != len(metas):
        raise ValueError(f"{F} bin columns but {len(metas)} feature metas")
    if N:
        top = bins_cols.max(axis=1)
        for f in range(F):  # a bin past num_bin would index past the feature's histogram
            if int(top[f]) >= max(int(metas[f]["num_bin"]), 1):
                raise ValueError(f"feature {f}: bin {int(top[f])} >= num_bin "
                                 f"{int(metas[f]['num_bin'])}")
    width = bins_cols.dtype.itemsize
    col_ptrs = (ctypes.c_void_p * F)(*[bins_cols[f].ctypes.data for f in range(F)])
    g = np.ascontiguousarray(g, dtype=np.float32)
    h = np.ascontiguousarray(h, dtype=np.float32)
    m = feature_metas(metas)
    cfg = LearnerConfig(int(num_leaves), int(max_depth), gain_config(**gain_kw))
    arrays = {}
    t = Tree()
    for name, dt, delta in TREE_ARRAYS:
        n = max(num_leaves + delta, 1)
        arrays[name] = np.zeros(n, dtype=dt)
        setattr(t, name, arrays[name].ctypes.data)
    cat_bins = np.zeros((max(num_leaves - 1, 1), 8), dtype=np.uint32)
    t.cat_bins = cat_bins.ctypes.data
    idx = np.empty(N, dtype=np.uint32)
    lb = np.empty(num_leaves, dtype=np.int32)
    lc = np.empty(num_leaves, dtype=np.int32)
    trace = np.zeros(4 * max(num_leaves, 1), dtype=np.int32)
    rc = lib().oracle_grow_tree(col_ptrs, width, N, F, ctypes.cast(m, ctypes.c_void_p), _ptr(g),
                                _ptr(h), ctypes.byref(cfg), int(nthreads), ctypes.byref(t),
                                _ptr(idx), _ptr(lb), _ptr(lc), _ptr(trace))
    if rc < 0:
        raise ValueError(f"oracle_grow_tree failed ({rc})")
    nl = t.num_leaves
    tree = {"num_leaves": nl}
    for name, dt, delta in TREE_ARRAYS:
        tree[name] = arrays[name][: max(nl + delta, 0)].copy()
    tree["cat_bins"] = cat_bins[: max(nl - 1, 0)].copy()
    part = {"indices": idx, "leaf_begin": lb[:nl].copy(), "leaf_count": lc[:nl].copy()}
    return tree, part, trace[: 4 * rc].reshape(-1, 4)


def binary_gradients(score, label, sigmoid=1.0, nthreads=1):
    score = np.ascontiguousarray(score, dtype=np.float64)
    label = np.ascontiguousarray(label, dtype=np.float32)
    g = np.empty(len(score), dtype=np.float32)
    h = np.empty(len(score), dtype=np.float32)
    lib().oracle_binary_gradients(_ptr(score), _ptr(label), len(score), float(sigmoid), _ptr(g),
                                  _ptr(h), int(nthreads))
    return g, h


def l2_gradients(score, label, nthreads=1):
    score = np.ascontiguousarray(score, dtype=np.float64)
    label = np.ascontiguousarray(label, dtype=np.float32)
    g = np.empty(len(score), dtype=np.float32)
    h = np.empty(len(score), dtype=np.float32)
    lib().oracle_l2_gradients(_ptr(score), _ptr(label), len(score), _ptr(g), _ptr(h),
                              int(nthreads))
    return g, h


def lambdarank_gradients(score, label, query_boundaries, sigmoid=1.0, norm=True,
                         truncation_level=30, label_gain=None, nthreads=1):
    """Lambdarank::get_gradients (lgbm-objective/src/rank.rs:264-366): f32 g, h."""
    score = np.ascontiguousarray(score, dtype=np.float64)
    label = np.ascontiguousarray(label, dtype=np.float32)
    qb = np.ascontiguousarray(query_boundaries, dtype=np.int32)
    lg = None if label_gain is None else np.ascontiguousarray(label_gain, dtype=np.float64)
    g = np.empty(len(score), dtype=np.float32)
    h = np.empty(len(score), dtype=np.float32)
    rc = lib().oracle_lambdarank_gradients(
        _ptr(score), _ptr(label), len(score), _ptr(qb), len(qb) - 1, float(sigmoid),
        int(bool(norm)), int(truncation_level), _ptr(lg), 0 if lg is None else len(lg),
        _ptr(g), _ptr(h), int(nthreads))
    if rc != 0:
        raise ValueError("invalid query boundaries or ranking labels")
    return g, h


def boost_from_score(objective, label, sigmoid=1.0):
    label = np.ascontiguousarray(label, dtype=np.float32)
    if objective == "binary":
        return lib().oracle_binary_boost_from_score(_ptr(label), len(label), float(sigmoid))
    return lib().oracle_l2_boost_from_score(_ptr(label), len(label))


def stochastic_seed(iteration, class_id=0):
    """The per-(iteration, class) seed of stochastic rounding (lgbm-boosting/src/gbdt.rs:950)."""
    return ((int(iteration) << 20) ^ int(class_id) ^ 0x51702010) & 0xFFFFFFFFFFFFFFFF


def quantize(g, h, num_grad_quant_bins, stochastic=False, seed=0):
    """Returns (dequantized g, dequantized h, int8 pairs [N,2] (qg, qh), scales).
    stochastic: stochastic rounding from the reference's seeded xorshift64
    (gradient_discretizer.rs:252-262) with `seed` (see stochastic_seed)."""
    g = np.array(g, dtype=np.float32)
    h = np.array(h, dtype=np.float32)
    q = np.empty((len(g), 2), dtype=np.int8)
    scales = np.empty(3, dtype=np.float64)
    lib().oracle_quantize_ex(_ptr(g), _ptr(h), len(g), int(num_grad_quant_bins), _ptr(q),
                             _ptr(scales), int(bool(stochastic)), ctypes.c_uint64(seed))
    return g, h, q, scales


def tree_shrinkage(tree, rate):
    lv = tree["leaf_value"]
    iv = tree["internal_value"]
    if len(iv) == 0:
        iv = np.zeros(1, dtype=np.float64)
    lib().oracle_tree_shrinkage(_ptr(lv), tree["num_leaves"], _ptr(iv), float(rate))


def add_prediction_to_score(tree, part, score):
    lib().oracle_add_prediction_to_score(
        _ptr(tree["leaf_value"]), tree["num_leaves"], _ptr(part["indices"]),
        _ptr(part["leaf_begin"]), _ptr(part["leaf_count"]), _ptr(score))


def max_threads():
    return lib().oracle_max_threads()


def train(bins_cols, metas, labels, objective="binary", num_iterations=10, learning_rate=0.1,
          num_leaves=31, max_depth=-1, use_quantized_grad=False, num_grad_quant_bins=4,
          stochastic_rounding=False, boost_from_average=True, sigmoid=1.0, nthreads=1,
          record=False,
          query_boundaries=None, lambdarank_norm=True, lambdarank_truncation_level=30,
          label_gain=None, **gain_kw):
    """Gbdt::train_one_iter loop (lgbm-boosting/src/gbdt.rs:691-1300), non-bagging GBDT.
    objective: "binary", "regression" (L2) or "lambdarank" (with query_boundaries; a
    ranking objective has no boost-from-average score).

    Returns dict(trees, init_score, scores, iter_scores?, iter_grad_hess?)."""
    labels = np.ascontiguousarray(labels, dtype=np.float32)
    N = len(labels)
    score = np.zeros(N, dtype=np.float64)
    init = 0.0
    if boost_from_average and objective != "lambdarank":
        init = boost_from_score(objective, labels, sigmoid)
        if abs(init) > float(np.float32(1e-15)):
            score += init
    trees = []
    iter_scores = []
    iter_gh = []
    for it in range(num_iterations):
        if objective == "binary":
            g, h = binary_gradients(score, labels, sigmoid, nthreads)
        elif objective == "lambdarank":
            g, h = lambdarank_gradients(score, labels, query_boundaries, sigmoid,
                                        lambdarank_norm, lambdarank_truncation_level,
                                        label_gain, nthreads)
        else:
            g, h = l2_gradients(score, labels, nthreads)
        if record:
            iter_gh.append((g.copy(), h.copy()))
        if use_quantized_grad:
            g, h, _, _ = quantize(g, h, num_grad_quant_bins, stochastic_rounding,
                                  stochastic_seed(it))
        tree, part, _ = grow_tree(bins_cols, metas, g, h, num_leaves, max_depth, nthreads,
                                  **gain_kw)
        if tree["num_leaves"] > 1:
            tree_shrinkage(tree, learning_rate)
            add_prediction_to_score(tree, part, score)
            if it == 0 and abs(init) > float(np.float32(1e-15)):
                tree["bias"] = init
            trees.append(tree)
        else:
            if it > 0:
                break
            tree["leaf_value"][0] = init
            trees.append(tree)
        if record:
            iter_scores.append(score.copy())
    out = {"trees": trees, "init_score": init, "scores": score}
    if record:
        out["iter_scores"] = iter_scores
        out["iter_grad_hess"] = iter_gh
    return out


def categorical_bitsets(tree, bin_to_category_of):
    """cat_boundaries / cat_threshold of a tree (Tree::split_categorical,
    lgbm-model/src/tree.rs:710-770): per categorical node, in node order, the bitset of
    the REAL categories of the bins sent left (Common::ConstructBitset)."""
    bounds, words = [0], []
    for node, dt in enumerate(tree["decision_type"]):
        if not (int(dt) & 1):
            continue
        f = int(tree["split_feature"][node])
        b2c = bin_to_category_of(f)
        bits = tree["cat_bins"][node]
        cats = [int(b2c[b]) for b in range(256) if (int(bits[b >> 5]) >> (b & 31)) & 1]
        n = max(cats) // 32 + 1 if cats else 0
        blk = [0] * n
        for c in cats:
            blk[c // 32] |= 1 << (c % 32)
        words.extend(blk)
        bounds.append(bounds[-1] + n)
    return bounds, words


def predict_raw(flat, rows):
    """Raw scores of a flattened ensemble (the dict lightgbm_rs_b200.model_text.flatten
    returns) over row-major f64 rows: the reference's tree walk, in tree order."""
    rows = np.ascontiguousarray(rows, dtype=np.float64)
    n = rows.shape[0]
    out = np.empty(n, dtype=np.float64)
    cb = flat["cat_boundaries"] if len(flat["cat_boundaries"]) else np.zeros(1, np.int32)
    ct = flat["cat_threshold"] if len(flat["cat_threshold"]) else np.zeros(1, np.uint32)
    lib().oracle_predict_raw(
        flat["num_trees"], flat["num_features"], _ptr(flat["node_offset"]),
        _ptr(flat["leaf_offset"]), _ptr(flat["split_feature"]), _ptr(flat["threshold"]),
        _ptr(flat["decision_type"]), _ptr(flat["left_child"]), _ptr(flat["right_child"]),
        _ptr(flat["leaf_value"]), _ptr(cb), _ptr(ct), _ptr(rows), n, _ptr(out))
    return out
