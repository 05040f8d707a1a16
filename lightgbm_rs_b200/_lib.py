"""ctypes binding of the C ABI declared in include/lgbm_b200.h."""

import ctypes
import os
import re

import numpy as np

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB_PATH = os.path.join(PKG, "liblgbm_b200.so")
HEADER = os.path.join(ROOT, "include", "lgbm_b200.h")

OK = 0
BIN_OUT_OF_RANGE = 1
LENGTH_MISMATCH = 2
CAPABILITY_UNAVAILABLE = 3
RUNTIME = 4
NON_FINITE = 5
INVALID_ARGUMENT = 6

MISSING_NONE, MISSING_ZERO, MISSING_NAN = 0, 1, 2
OBJECTIVE_BINARY, OBJECTIVE_L2, OBJECTIVE_LAMBDARANK = 0, 1, 2
GH_F32, GH_INT8_PAIR = 0, 1

_P = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_u32 = ctypes.c_uint32
_f64 = ctypes.c_double


class LightGBMError(RuntimeError):
    """Raised when a C-ABI call fails; .code carries the LGBM_B200_* status."""

    def __init__(self, code, msg):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class GainConfig(ctypes.Structure):
    _fields_ = [("min_data_in_leaf", _i32), ("_reserved", _i32),
                ("min_sum_hessian_in_leaf", _f64), ("max_delta_step", _f64),
                ("lambda_l1", _f64), ("lambda_l2", _f64), ("min_gain_to_split", _f64),
                ("path_smooth", _f64), ("parent_output", _f64),
                ("min_data_per_group", _i32), ("max_cat_threshold", _i32),
                ("max_cat_to_onehot", _i32), ("_reserved2", _i32), ("cat_l2", _f64),
                ("cat_smooth", _f64)]


class SplitInfo(ctypes.Structure):
    _fields_ = [("threshold", _u32), ("default_left", _i32), ("left_count", _i32),
                ("right_count", _i32), ("gain", _f64), ("left_sum_gradient", _f64),
                ("left_sum_hessian", _f64), ("right_sum_gradient", _f64),
                ("right_sum_hessian", _f64), ("left_output", _f64), ("right_output", _f64)]


class FeatureMeta(ctypes.Structure):
    _fields_ = [("num_bin", _i32), ("default_bin", _i32), ("most_freq_bin", _i32),
                ("missing_type", _i32), ("bin_type", _i32)]


class BatchedFeature(ctypes.Structure):
    _fields_ = [("slot_off", _i64), ("num_bin", _u32), ("offset", _i32), ("default_bin", _u32),
                ("most_freq_bin", _u32), ("skip_default_bin", _i32), ("na_as_missing", _i32),
                ("run_forward", _i32), ("_reserved", _i32)]


class TreeC(ctypes.Structure):
    _fields_ = [("num_leaves", _i32), ("max_leaves", _i32), ("left_child", _P),
                ("right_child", _P), ("split_feature", _P), ("threshold_bin", _P),
                ("split_gain", _P), ("decision_type", _P), ("leaf_value", _P),
                ("leaf_weight", _P), ("leaf_count", _P), ("internal_value", _P),
                ("internal_count", _P), ("cat_bins", _P)]


class LearnerConfig(ctypes.Structure):
    _fields_ = [("num_leaves", _i32), ("max_depth", _i32), ("gain", GainConfig)]


class TrainConfig(ctypes.Structure):
    _fields_ = [("learner", LearnerConfig), ("objective", _i32), ("use_quantized_grad", _i32),
                ("num_grad_quant_bins", _i32), ("boost_from_average", _i32), ("sigmoid", _f64),
                ("learning_rate", _f64), ("query_boundaries", _P), ("num_queries", _i32),
                ("lambdarank_truncation_level", _i32), ("lambdarank_norm", _i32),
                ("num_label_gain", _i32), ("label_gain", _P), ("stochastic_rounding", _i32),
                ("_reserved0", _i32)]


class BinConfig(ctypes.Structure):
    _fields_ = [("max_bin", _i32), ("min_data_in_bin", _i32), ("min_data_in_leaf", _i32),
                ("pre_filter", _i32), ("use_missing", _i32), ("zero_as_missing", _i32),
                ("bin_construct_sample_cnt", _i32), ("data_random_seed", _i32)]


class BinMapperC(ctypes.Structure):
    _fields_ = [("num_bin", _i32), ("missing_type", _i32), ("default_bin", _i32),
                ("most_freq_bin", _i32), ("is_trivial", _i32), ("_reserved", _i32),
                ("min_val", _f64), ("max_val", _f64), ("sparse_rate", _f64)]


class ModelC(ctypes.Structure):
    _fields_ = [("num_trees", _i32), ("num_features", _i32), ("node_offset", _P),
                ("leaf_offset", _P), ("split_feature", _P), ("threshold", _P),
                ("decision_type", _P), ("left_child", _P), ("right_child", _P),
                ("leaf_value", _P), ("num_cat", _i32), ("transform", _i32),
                ("cat_boundaries", _P), ("cat_threshold", _P), ("sigmoid", _f64)]


_SIGS = {
    "lgbm_b200_last_error": ([], ctypes.c_char_p),
    "lgbm_b200_abi_version": ([], _i32),
    "lgbm_b200_device_count": ([_P], ctypes.c_int),
    "lgbm_b200_release_cached_memory": ([_i32, _P], ctypes.c_int),
    "lgbm_b200_bin_column": ([_P, _i64, _P, _P, _P, _i32, _P], ctypes.c_int),
    "lgbm_b200_bin_column_categorical": ([_P, _i64, _P, _P, _P, _i32, _P], ctypes.c_int),
    "lgbm_b200_find_bins": ([_i32, _P, _i32, _i64, _i32, _P, _P, _P, _i32], ctypes.c_int),
    "lgbm_b200_construct_histograms": ([_P, _P, _P, _i64, _u32, _P], ctypes.c_int),
    "lgbm_b200_find_best_split": ([_P, _P, _u32, _i32, _u32, _u32, _i32, _i32, _i32, _f64, _f64,
                                   _i32, _P], ctypes.c_int),
    "lgbm_b200_find_best_splits_batched": ([_P, _i64, _P, _i32, _P, _f64, _f64, _i32, _P],
                                           ctypes.c_int),
    "lgbm_b200_data_partition": ([_P, _i64, _u32, _u32, _u32, _u32, _u32, _P, _P], ctypes.c_int),
    "lgbm_b200_data_partition_missing": ([_P, _i64, _u32, _u32, _u32, _u32, _u32, _u32, _i32,
                                          _i32, _P, _P], ctypes.c_int),
    "lgbm_b200_data_partition_noalloc": ([_P, _i64, _u32, _u32, _u32, _u32, _u32, _P, _P, _P],
                                         ctypes.c_int),
    "lgbm_b200_subtract_histograms": ([_P, _P, _i64, _P], ctypes.c_int),
    "lgbm_b200_dataset_create": ([_i32, _P, _i32, _i64, _i32, _P, _P], ctypes.c_int),
    "lgbm_b200_dataset_destroy": ([_P], ctypes.c_int),
    "lgbm_b200_dataset_num_data": ([_P, _P], ctypes.c_int),
    "lgbm_b200_learner_create": ([_P, _P, _P], ctypes.c_int),
    "lgbm_b200_learner_destroy": ([_P], ctypes.c_int),
    "lgbm_b200_learner_grow_tree": ([_P, _i32, _P, _P, _P, _P, _P, _P], ctypes.c_int),
    "lgbm_b200_booster_create": ([_P, _P, _P, _P], ctypes.c_int),
    "lgbm_b200_booster_destroy": ([_P], ctypes.c_int),
    "lgbm_b200_booster_train": ([_P, _i32, _P], ctypes.c_int),
    "lgbm_b200_booster_num_trees": ([_P, _P], ctypes.c_int),
    "lgbm_b200_booster_get_tree": ([_P, _i32, _P], ctypes.c_int),
    "lgbm_b200_booster_init_score": ([_P, _P], ctypes.c_int),
    "lgbm_b200_booster_get_scores": ([_P, _P], ctypes.c_int),
    "lgbm_b200_booster_get_gradients": ([_P, _P, _P], ctypes.c_int),
    "lgbm_b200_booster_phase_ms": ([_P, _P], ctypes.c_int),
    "lgbm_b200_booster_profile_iteration": ([_P, _P, _P], ctypes.c_int),
    "lgbm_b200_booster_profile_pipeline": ([_P, _i32, _P, _P, _P], ctypes.c_int),
    "lgbm_b200_booster_profile_launches": ([_P, _i32, _P, _P, _P], ctypes.c_int),
    "lgbm_b200_booster_profile_spans": ([_P, _i32, _P, _P, _P, _P], ctypes.c_int),
    "lgbm_b200_comm_unique_id": ([_P], ctypes.c_int),
    "lgbm_b200_comm_create": ([_i32, _i32, _i32, _P, _P], ctypes.c_int),
    "lgbm_b200_comm_destroy": ([_P], ctypes.c_int),
    "lgbm_b200_booster_create_distributed": ([_P, _P, _P, _P, _P], ctypes.c_int),
    "lgbm_b200_dataset_create_from_values": ([_i32, _P, _i32, _i64, _i32, _P, _P, _P, _P],
                                             ctypes.c_int),
    "lgbm_b200_dataset_copy_bins": ([_P, _P], ctypes.c_int),
    "lgbm_b200_predictor_create": ([_i32, _P, _P], ctypes.c_int),
    "lgbm_b200_predictor_destroy": ([_P], ctypes.c_int),
    "lgbm_b200_predict": ([_P, _P, _i64, _i32, _P], ctypes.c_int),
}

_lib = None


def header_symbols():
    """Every function name declared in include/lgbm_b200.h."""
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"\b(lgbm_b200_[a-z0-9_]+)\s*\(", text)))


def lib():
    """Load the in-tree library. Fails loudly when it is missing: there is no fallback."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing; build it with `python -m lightgbm_rs_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(rc):
    if rc != OK:
        msg = lib().lgbm_b200_last_error().decode(errors="replace")
        raise LightGBMError(rc, msg)


def ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def device_count():
    n = _i32(0)
    check(lib().lgbm_b200_device_count(ctypes.byref(n)))
    return n.value


def gain_config(min_data_in_leaf=20, min_sum_hessian_in_leaf=1e-3, max_delta_step=0.0,
                lambda_l1=0.0, lambda_l2=0.0, min_gain_to_split=0.0, path_smooth=0.0,
                parent_output=0.0, min_data_per_group=100, max_cat_threshold=32,
                max_cat_to_onehot=4, cat_l2=10.0, cat_smooth=10.0):
    return GainConfig(int(min_data_in_leaf), 0, float(min_sum_hessian_in_leaf),
                      float(max_delta_step), float(lambda_l1), float(lambda_l2),
                      float(min_gain_to_split), float(path_smooth), float(parent_output),
                      int(min_data_per_group), int(max_cat_threshold), int(max_cat_to_onehot),
                      0, float(cat_l2), float(cat_smooth))


TREE_FIELDS = [
    ("left_child", np.int32, -1), ("right_child", np.int32, -1),
    ("split_feature", np.int32, -1), ("threshold_bin", np.uint32, -1),
    ("split_gain", np.float32, -1), ("decision_type", np.int8, -1),
    ("leaf_value", np.float64, 0), ("leaf_weight", np.float64, 0),
    ("leaf_count", np.int32, 0), ("internal_value", np.float64, -1),
    ("internal_count", np.int32, -1),
]


def tree_buffers(max_leaves):
    arrays = {}
    t = TreeC()
    t.max_leaves = int(max_leaves)
    for name, dt, delta in TREE_FIELDS:
        arrays[name] = np.zeros(max(max_leaves + delta, 1), dtype=dt)
        setattr(t, name, arrays[name].ctypes.data)
    arrays["cat_bins"] = np.zeros((max(max_leaves - 1, 1), 8), dtype=np.uint32)
    t.cat_bins = arrays["cat_bins"].ctypes.data
    return t, arrays


def tree_dict(t, arrays):
    nl = t.num_leaves
    out = {"num_leaves": nl}
    for name, _, delta in TREE_FIELDS:
        out[name] = arrays[name][: max(nl + delta, 0)].copy()
    out["cat_bins"] = arrays["cat_bins"][: max(nl - 1, 0)].copy()
    return out
