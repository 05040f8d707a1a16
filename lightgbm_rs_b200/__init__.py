"""lightgbm_rs_b200 — B200-native histogram tree learner behind lightgbm_rs's surface.

The Python surface mirrors the reference's `lightgbm_rs` package for this path
(crates/lgbm-python/python/lightgbm_rs/engine.py:254 `train`, `Dataset`,
`Booster.predict`). All training work runs through the C ABI in
include/lgbm_b200.h on the GPU; there is no CPU fallback: without the built
library or a CUDA device the calls raise.
"""

import ctypes

import numpy as np

from . import _lib as C
from . import model_text as MT
from ._lib import LightGBMError
from . import distributed  # noqa: E402

__all__ = ["Dataset", "Booster", "Predictor", "train", "bin_column", "find_bins", "LightGBMError",
           "Learner", "distributed", "categorical_bitsets", "model_text"]

# Reference config defaults (crates/lgbm-core/src/config/mod.rs:430-587).
_DEFAULTS = {
    "objective": "regression",
    "num_leaves": 31,
    "max_depth": -1,
    "min_data_in_leaf": 20,
    "min_sum_hessian_in_leaf": 1e-3,
    "lambda_l1": 0.0,
    "lambda_l2": 0.0,
    "min_gain_to_split": 0.0,
    "max_delta_step": 0.0,
    "path_smooth": 0.0,
    "learning_rate": 0.1,
    "max_bin": 255,
    "min_data_in_bin": 3,
    "bin_construct_sample_cnt": 200000,
    "data_random_seed": 1,
    "use_missing": True,
    "zero_as_missing": False,
    "feature_pre_filter": True,
    "use_quantized_grad": False,
    "num_grad_quant_bins": 4,
    "stochastic_rounding": True,
    "min_data_per_group": 100,
    "max_cat_threshold": 32,
    "max_cat_to_onehot": 4,
    "cat_l2": 10.0,
    "cat_smooth": 10.0,
    "boost_from_average": True,
    "sigmoid": 1.0,
    "lambdarank_truncation_level": 30,
    "lambdarank_norm": True,
    "label_gain": None,
    "device": 0,
}

_ALIASES = {
    "min_child_samples": "min_data_in_leaf", "min_data": "min_data_in_leaf",
    "reg_alpha": "lambda_l1", "reg_lambda": "lambda_l2", "lr": "learning_rate",
    "eta": "learning_rate", "shrinkage_rate": "learning_rate", "num_leaf": "num_leaves",
    "max_leaves": "num_leaves", "min_split_gain": "min_gain_to_split",
    "min_sum_hessian": "min_sum_hessian_in_leaf", "min_child_weight": "min_sum_hessian_in_leaf",
    "application": "objective", "app": "objective", "loss": "objective",
    "data_seed": "data_random_seed", "subsample_for_bin": "bin_construct_sample_cnt",
    "device_id": "device", "gpu_device_id": "device",
}

_OBJECTIVES = {"binary": C.OBJECTIVE_BINARY, "regression": C.OBJECTIVE_L2,
               "regression_l2": C.OBJECTIVE_L2, "l2": C.OBJECTIVE_L2, "mse": C.OBJECTIVE_L2,
               "lambdarank": C.OBJECTIVE_LAMBDARANK}


def _resolve(params):
    p = dict(_DEFAULTS)
    for k, v in (params or {}).items():
        k = _ALIASES.get(k, k)
        p[k] = v
    return p


def _excluded(m):
    """A trivial feature's mapper as a one-bin feature that never splits. The reference
    leaves trivial features out of the dataset (lgbm-dataset/src/dataset.rs:106-126:
    used features are the non-trivial ones); a one-bin feature has no threshold, so the
    trees are the same while feature indices stay those of the input columns."""
    out = dict(m)
    out.update(num_bin=1, default_bin=0, most_freq_bin=0, missing_type=0, is_trivial=True)
    if m.get("bin_type", 0) == 1:
        out["bin_to_category"] = np.array([-1], dtype=np.int32)
    else:
        out["upper"] = np.array([np.inf], dtype=np.float64)
    return out


def bin_column(values, max_bin=255, min_data_in_bin=3, min_data_in_leaf=20, pre_filter=False,
               use_missing=True, zero_as_missing=False, bin_construct_sample_cnt=200000,
               data_random_seed=1, want_bins=True, categorical=False):
    """BinMapper::find_bin_from_column + value_to_bin (host-side; no GPU needed).
    categorical=True bins the column as categories (find_bin_categorical); the mapper
    then carries bin_to_category instead of upper bounds."""
    col = np.ascontiguousarray(values, dtype=np.float64)
    cfg = C.BinConfig(int(max_bin), int(min_data_in_bin), int(min_data_in_leaf),
                      int(bool(pre_filter)), int(bool(use_missing)), int(bool(zero_as_missing)),
                      int(bin_construct_sample_cnt), int(data_random_seed))
    m = C.BinMapperC()
    cap = max(int(max_bin) + 2, 4)
    bins = np.empty(len(col), dtype=np.uint32) if want_bins else None
    if categorical:
        # the 99 % cut may keep more categories than max_bin
        cap = max(cap, min(len(col), 1 << 20) + 2)
        b2c = np.zeros(cap, dtype=np.int32)
        C.check(C.lib().lgbm_b200_bin_column_categorical(C.ptr(col), len(col), ctypes.byref(cfg),
                                                         ctypes.byref(m), C.ptr(b2c), cap,
                                                         C.ptr(bins)))
    else:
        upper = np.zeros(cap, dtype=np.float64)
        C.check(C.lib().lgbm_b200_bin_column(C.ptr(col), len(col), ctypes.byref(cfg),
                                             ctypes.byref(m), C.ptr(upper), cap, C.ptr(bins)))
    mapper = {"num_bin": m.num_bin, "missing_type": m.missing_type,
              "default_bin": m.default_bin, "most_freq_bin": m.most_freq_bin,
              "is_trivial": bool(m.is_trivial), "min_val": m.min_val, "max_val": m.max_val,
              "sparse_rate": m.sparse_rate, "bin_type": 1 if categorical else 0}
    if categorical:
        mapper["bin_to_category"] = b2c[: m.num_bin].copy()
    else:
        mapper["upper"] = upper[: m.num_bin].copy()
    return mapper, bins


def find_bins(columns, max_bin=255, min_data_in_bin=3, min_data_in_leaf=20, pre_filter=False,
              use_missing=True, zero_as_missing=False, bin_construct_sample_cnt=200000,
              data_random_seed=1, device=0):
    """BinMapper::find_bin_from_column of numerical columns on the device: the mappers
    bin_column would return (bin_mapper.rs:642-675), for every row of `columns`
    (feature-major [F, n], f32 or f64). Needs a CUDA device."""
    if isinstance(columns, np.ndarray) and columns.ndim == 2:
        columns = list(columns)
    dt = np.float32 if all(np.asarray(c).dtype == np.float32 for c in columns) else np.float64
    cols = [np.ascontiguousarray(c, dtype=dt) for c in columns]
    F = len(cols)
    n = len(cols[0]) if F else 0
    if any(len(c) != n for c in cols):
        raise LightGBMError(C.INVALID_ARGUMENT, "columns differ in length")
    cfg = C.BinConfig(int(max_bin), int(min_data_in_bin), int(min_data_in_leaf),
                      int(bool(pre_filter)), int(bool(use_missing)), int(bool(zero_as_missing)),
                      int(bin_construct_sample_cnt), int(data_random_seed))
    cap = int(max_bin) + 2
    ptrs = (ctypes.c_void_p * max(F, 1))(*[c.ctypes.data for c in cols])
    ms = (C.BinMapperC * max(F, 1))()
    upper = np.zeros((max(F, 1), cap), dtype=np.float64)
    C.check(C.lib().lgbm_b200_find_bins(int(device), ptrs, np.dtype(dt).itemsize, n, F,
                                        ctypes.byref(cfg), ms, C.ptr(upper), cap))
    out = []
    for f in range(F):
        m = ms[f]
        out.append({"num_bin": m.num_bin, "missing_type": m.missing_type,
                    "default_bin": m.default_bin, "most_freq_bin": m.most_freq_bin,
                    "is_trivial": bool(m.is_trivial), "min_val": m.min_val,
                    "max_val": m.max_val, "sparse_rate": m.sparse_rate, "bin_type": 0,
                    "upper": upper[f, : m.num_bin].copy()})
    return out


class Dataset:
    """Binned training data resident on one GPU (lightgbm_rs.Dataset for this path).

    data: 2-D array [num_data, num_features] of raw values: the bin mappers are found on
    the host from each column's sample (the reference BinMapper), and the values are
    binned on the device when the dataset is constructed. Or pass `bins` / `mappers` to
    reuse an existing binning."""

    def __init__(self, data=None, label=None, params=None, bins=None, mappers=None,
                 categorical_feature=None, group=None):
        """categorical_feature: column indices binned as categories (non-negative integer
        codes; negatives and NaN count as missing), as lightgbm's Dataset takes them.
        group: query sizes in row order for ranking objectives (also accepted as
        params["group"], a comma-separated string as the reference's sklearn layer
        passes it)."""
        self.params = _resolve(params)
        if group is None and self.params.get("group") is not None:
            group = self.params["group"]
        self.set_group(group)
        cats = set(int(c) for c in (categorical_feature or []))
        self.label = None if label is None else np.ascontiguousarray(label, dtype=np.float32)
        self._cats = cats
        self._bins = None
        self._values = None
        if bins is None:
            X = np.asarray(data)
            if X.ndim != 2:
                raise LightGBMError(C.INVALID_ARGUMENT, "data must be 2-D")
            dt = np.float32 if X.dtype == np.float32 else np.float64
            # feature-major raw values, binned on the device by construct()
            self._values = np.ascontiguousarray(X.T, dtype=dt)
            self.num_features, self.num_data = self._values.shape
            # the binning settings the mappers were found with; the host view `bins`
            # applies the same ones whatever train() later merges into params
            self._bin_kw = self._bin_kwargs()
            self.mappers = self._find_mappers()
        else:
            self._bins = np.ascontiguousarray(bins)
            self.mappers = mappers
            self.num_features, self.num_data = self._bins.shape
        self._handle = None

    def _bin_kwargs(self):
        p = self.params
        return dict(max_bin=p["max_bin"], min_data_in_bin=p["min_data_in_bin"],
                    min_data_in_leaf=p["min_data_in_leaf"], pre_filter=p["feature_pre_filter"],
                    use_missing=p["use_missing"], zero_as_missing=p["zero_as_missing"],
                    bin_construct_sample_cnt=p["bin_construct_sample_cnt"],
                    data_random_seed=p["data_random_seed"])

    def _find_mappers(self):
        """BinMapper::find_bin_from_column of every column (its sample only): numerical
        columns on the device when one is present (find_bins), categorical ones on the
        host."""
        import concurrent.futures as cf
        import os

        kw = self._bin_kw
        maps = [None] * self.num_features
        numeric = [j for j in range(self.num_features) if j not in self._cats]
        # device_binning: True / False, or "auto" (the default): on the device when there
        # are at least 512 numerical columns. The device runs one thread per column, so its
        # time barely grows with the columns, while the host's grows with columns / cores:
        # for C1's 28 columns the device took 0.14 s against 0.095 s on 16 host threads.
        dev_bin = self.params.get("device_binning", "auto")
        if dev_bin == "auto":
            dev_bin = len(numeric) >= 512
        if numeric and dev_bin and C.device_count() > 0:
            found = find_bins([self._values[j] for j in numeric],
                              device=int(self.params.get("device", 0)), **kw)
            for j, m in zip(numeric, found):
                maps[j] = m

        def one(j):
            m = maps[j]
            if m is None:
                m, _ = bin_column(self._values[j], want_bins=False,
                                  categorical=j in self._cats, **kw)
            return _excluded(m) if m["is_trivial"] else m

        with cf.ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 4)) as ex:
            return list(ex.map(one, range(self.num_features)))

    @property
    def bins(self):
        """Feature-major bins [num_features, num_data]. For a dataset built from raw
        values these are computed on the host (value_to_bin per value) on first use."""
        if self._bins is None:
            kw = self._bin_kw
            cols = []
            for j in range(self.num_features):
                if self.mappers[j]["num_bin"] == 1:  # constant or left out: one bin
                    cols.append(np.zeros(self.num_data, dtype=np.uint32))
                    continue
                _, b = bin_column(self._values[j], categorical=j in self._cats, **kw)
                cols.append(b)
            wide = any(m["num_bin"] > 256 for m in self.mappers)
            self._bins = np.ascontiguousarray(
                np.stack(cols).astype(np.uint32 if wide else np.uint8))
        return self._bins

    def device_bins(self):
        """The device's row-major bin matrix, read back as feature-major [F, N] u8."""
        h = self.construct()
        stride = (self.num_features + 15) // 16 * 16
        out = np.empty((self.num_data, stride), dtype=np.uint8)
        C.check(C.lib().lgbm_b200_dataset_copy_bins(h, C.ptr(out)))
        return np.ascontiguousarray(out[:, : self.num_features].T)

    def set_group(self, group):
        """Query sizes (or None); stored as query boundaries (prefix sums)."""
        if group is None:
            self.query_boundaries = None
            return
        if isinstance(group, str):
            group = [int(t) for t in group.split(",") if t.strip()]
        sizes = np.asarray(group, dtype=np.int64).reshape(-1)
        if (sizes < 0).any():
            raise LightGBMError(C.INVALID_ARGUMENT, "group sizes must be non-negative")
        self.query_boundaries = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)

    def construct(self):
        if self._handle is None:
            metas = (C.FeatureMeta * self.num_features)()
            for f, m in enumerate(self.mappers):
                metas[f] = C.FeatureMeta(int(m["num_bin"]), int(m["default_bin"]),
                                         int(m["most_freq_bin"]), int(m.get("missing_type", 0)),
                                         int(m.get("bin_type", 0)))
            h = ctypes.c_void_p()
            dev = int(self.params.get("device", 0))
            if self._values is not None and self._bins is None:
                V = self._values
                cols = (ctypes.c_void_p * self.num_features)(
                    *[V[f].ctypes.data for f in range(self.num_features)])
                keep = []
                ups = (ctypes.c_void_p * self.num_features)()
                b2c = (ctypes.c_void_p * self.num_features)()
                for f, m in enumerate(self.mappers):
                    if m.get("bin_type", 0) == 1:
                        a = np.ascontiguousarray(m["bin_to_category"], dtype=np.int32)
                        b2c[f] = a.ctypes.data
                    else:
                        a = np.ascontiguousarray(m["upper"], dtype=np.float64)
                        ups[f] = a.ctypes.data
                    keep.append(a)
                C.check(C.lib().lgbm_b200_dataset_create_from_values(
                    dev, cols, V.dtype.itemsize, self.num_data, self.num_features,
                    ctypes.cast(metas, ctypes.c_void_p), ups, b2c, ctypes.byref(h)))
            else:
                B = self.bins
                cols = (ctypes.c_void_p * self.num_features)(
                    *[B[f].ctypes.data for f in range(self.num_features)])
                C.check(C.lib().lgbm_b200_dataset_create(
                    dev, cols, B.dtype.itemsize, self.num_data, self.num_features,
                    ctypes.cast(metas, ctypes.c_void_p), ctypes.byref(h)))
            self._handle = h
        return self._handle

    def __del__(self):
        try:
            if self._handle is not None:
                C.lib().lgbm_b200_dataset_destroy(self._handle)
                self._handle = None
        except Exception:
            pass


def _learner_config(p):
    return C.LearnerConfig(int(p["num_leaves"]), int(p["max_depth"]), C.gain_config(
        p["min_data_in_leaf"], p["min_sum_hessian_in_leaf"], p["max_delta_step"],
        p["lambda_l1"], p["lambda_l2"], p["min_gain_to_split"], p["path_smooth"], 0.0,
        p["min_data_per_group"], p["max_cat_threshold"], p["max_cat_to_onehot"], p["cat_l2"],
        p["cat_smooth"]))


class Learner:
    """SerialTreeLearner on the device: grows one tree from given gradients."""

    def __init__(self, dataset, params=None):
        self.dataset = dataset
        p = _resolve(params)
        self.num_leaves = int(p["num_leaves"])
        cfg = _learner_config(p)
        h = ctypes.c_void_p()
        C.check(C.lib().lgbm_b200_learner_create(dataset.construct(), ctypes.byref(cfg),
                                                 ctypes.byref(h)))
        self._handle = h

    def grow(self, g=None, h=None, quantized=None, scales=None, with_partition=True):
        """Grow one tree. f32 g/h, or quantized=int8 [N,2] pairs (qg, qh) + scales
        (grad_scale, hess_scale, is_constant_hessian, num_grad_quant_bins)."""
        N = self.dataset.num_data
        t, arrays = C.tree_buffers(self.num_leaves)
        idx = np.empty(N, dtype=np.uint32) if with_partition else None
        lb = np.empty(self.num_leaves, dtype=np.int32) if with_partition else None
        lc = np.empty(self.num_leaves, dtype=np.int32) if with_partition else None
        if quantized is None:
            gh = np.concatenate([np.asarray(g, np.float32), np.asarray(h, np.float32)])
            kind, sc = C.GH_F32, None
        else:
            gh = np.ascontiguousarray(quantized, dtype=np.int8).reshape(-1)
            kind = C.GH_INT8_PAIR
            sc = np.asarray(scales, dtype=np.float64)
        C.check(C.lib().lgbm_b200_learner_grow_tree(self._handle, kind, C.ptr(gh), C.ptr(sc),
                                                    ctypes.byref(t), C.ptr(idx), C.ptr(lb),
                                                    C.ptr(lc)))
        tree = C.tree_dict(t, arrays)
        part = None
        if with_partition:
            nl = tree["num_leaves"]
            part = {"indices": idx, "leaf_begin": lb[:nl].copy(), "leaf_count": lc[:nl].copy()}
        return tree, part

    def __del__(self):
        try:
            C.lib().lgbm_b200_learner_destroy(self._handle)
        except Exception:
            pass


class Predictor:
    """A tree ensemble on the device for batch prediction from raw feature values
    (lgbm_b200_predictor_*)."""

    def __init__(self, model, device=0):
        self.model = model
        f = MT.flatten(model)
        self._flat = f  # the create call borrows these arrays
        m = C.ModelC()
        m.num_trees, m.num_features = f["num_trees"], f["num_features"]
        for k in ("node_offset", "leaf_offset", "split_feature", "threshold", "decision_type",
                  "left_child", "right_child", "leaf_value", "cat_boundaries",
                  "cat_threshold"):
            setattr(m, k, f[k].ctypes.data if len(f[k]) else None)
        m.num_cat, m.transform, m.sigmoid = f["num_cat"], f["transform"], f["sigmoid"]
        h = ctypes.c_void_p()
        C.check(C.lib().lgbm_b200_predictor_create(int(device), ctypes.byref(m),
                                                   ctypes.byref(h)))
        self._handle = h

    def predict(self, data, raw_score=False):
        X = np.ascontiguousarray(data, dtype=np.float64)
        if X.ndim == 1:
            X = X.reshape(1, -1)
        nf = self.model.max_feature_idx + 1
        if X.ndim != 2 or X.shape[1] != nf:
            raise LightGBMError(C.LENGTH_MISMATCH,
                                f"data has {X.shape[-1]} columns, the model {nf} features")
        out = np.empty(X.shape[0], dtype=np.float64)
        C.check(C.lib().lgbm_b200_predict(self._handle, C.ptr(X), X.shape[0],
                                          int(bool(raw_score)), C.ptr(out)))
        return out

    def __del__(self):
        try:
            C.lib().lgbm_b200_predictor_destroy(self._handle)
        except Exception:
            pass


class Booster:
    """lightgbm_rs.Booster for this path: training on the device, model text, predict."""

    def __init__(self, params=None, train_set=None, model_file=None, model_str=None,
                 comm=None):
        """Train from `train_set`, or load LightGBM model text (`model_file` / `model_str`)
        for prediction. comm: a distributed.Communicator for data-parallel training;
        train_set then holds this rank's shard of the rows (in global row order, shards in
        rank order)."""
        self.params = _resolve(params)
        self.train_set = train_set
        self._model = None
        self._predictor = None
        self._handle = None
        if model_file is not None or model_str is not None:
            if model_str is None:
                with open(model_file) as fh:
                    model_str = fh.read()
            self._model = MT.parse(model_str)
            self.objective = self._model.objective_name
            self.params["sigmoid"] = self._model.sigmoid
            return
        if train_set is None:
            raise LightGBMError(C.INVALID_ARGUMENT, "Booster needs train_set or a model")
        p = self.params
        obj = str(p["objective"]).lower()
        if obj not in _OBJECTIVES:
            raise LightGBMError(C.CAPABILITY_UNAVAILABLE, f"objective {obj!r} not on the path")
        self.objective = {C.OBJECTIVE_BINARY: "binary", C.OBJECTIVE_L2: "regression",
                          C.OBJECTIVE_LAMBDARANK: "lambdarank"}[_OBJECTIVES[obj]]
        if train_set.label is None:
            raise LightGBMError(C.INVALID_ARGUMENT, "Dataset has no label")
        cfg = C.TrainConfig(_learner_config(p), _OBJECTIVES[obj], int(bool(p["use_quantized_grad"])),
                            int(p["num_grad_quant_bins"]), int(bool(p["boost_from_average"])),
                            float(p["sigmoid"]), float(p["learning_rate"]))
        cfg.stochastic_rounding = int(bool(p["stochastic_rounding"]))
        self._rank_arrays = None
        if obj == "lambdarank":
            qb = train_set.query_boundaries
            if qb is None:
                raise LightGBMError(C.INVALID_ARGUMENT,
                                    "lambdarank needs query sizes (Dataset group=)")
            if qb[-1] != train_set.num_data:
                raise LightGBMError(C.INVALID_ARGUMENT, f"group sizes sum to {qb[-1]}, "
                                    f"the dataset has {train_set.num_data} rows")
            lg = p.get("label_gain")
            if isinstance(lg, str):
                lg = [float(t) for t in lg.split(",") if t.strip()]
            lg = None if lg is None or len(lg) == 0 else np.asarray(lg, dtype=np.float64)
            self._rank_arrays = (qb, lg)  # borrowed by the create call
            cfg.query_boundaries = C.ptr(qb)
            cfg.num_queries = len(qb) - 1
            cfg.lambdarank_truncation_level = int(p["lambdarank_truncation_level"])
            cfg.lambdarank_norm = int(bool(p["lambdarank_norm"]))
            cfg.num_label_gain = 0 if lg is None else len(lg)
            cfg.label_gain = C.ptr(lg)
        h = ctypes.c_void_p()
        if comm is not None:
            C.check(C.lib().lgbm_b200_booster_create_distributed(
                train_set.construct(), C.ptr(train_set.label), ctypes.byref(cfg), comm._handle,
                ctypes.byref(h)))
        elif str(p.get("tree_learner", "serial")).lower() in ("data", "data_parallel"):
            raise LightGBMError(C.INVALID_ARGUMENT,
                                "tree_learner=data needs a distributed.Communicator (comm=)")
        else:
            C.check(C.lib().lgbm_b200_booster_create(train_set.construct(),
                                                     C.ptr(train_set.label),
                                                     ctypes.byref(cfg), ctypes.byref(h)))
        self._handle = h
        self._comm = comm  # keeps the communicator alive as long as the booster
        self.num_leaves = int(p["num_leaves"])
        self._trees = None

    def update(self, num_iterations=1):
        self._require_training()
        done = C._i32(0)
        C.check(C.lib().lgbm_b200_booster_train(self._handle, int(num_iterations),
                                                ctypes.byref(done)))
        self._trees = None
        self._model = None
        self._predictor = None
        return done.value

    def _require_training(self):
        if self._handle is None:
            raise LightGBMError(C.INVALID_ARGUMENT, "a booster loaded from model text "
                                "does not train")

    def model(self):
        """The ensemble as a model_text.Model (trained trees, or the loaded model)."""
        if self._model is None:
            self._model = MT.from_booster(self)
        return self._model

    def model_to_string(self):
        """LightGBM v4 model text (GBDT::SaveModelToString)."""
        return MT.dump(self.model())

    def save_model(self, filename):
        with open(filename, "w") as fh:
            fh.write(self.model_to_string())
        return self

    def num_trees(self):
        if self._handle is None:
            return len(self._model.trees)
        n = C._i32(0)
        C.check(C.lib().lgbm_b200_booster_num_trees(self._handle, ctypes.byref(n)))
        return n.value

    def init_score(self):
        self._require_training()
        v = C._f64(0.0)
        C.check(C.lib().lgbm_b200_booster_init_score(self._handle, ctypes.byref(v)))
        return v.value

    def trees(self):
        if self._trees is None:
            out = []
            for i in range(self.num_trees()):
                t, arrays = C.tree_buffers(self.num_leaves)
                C.check(C.lib().lgbm_b200_booster_get_tree(self._handle, i, ctypes.byref(t)))
                out.append(C.tree_dict(t, arrays))
            self._trees = out
        return self._trees

    def train_scores(self):
        s = np.empty(self.train_set.num_data, dtype=np.float64)
        C.check(C.lib().lgbm_b200_booster_get_scores(self._handle, C.ptr(s)))
        return s

    def last_gradients(self):
        n = self.train_set.num_data
        g = np.empty(n, dtype=np.float32)
        h = np.empty(n, dtype=np.float32)
        C.check(C.lib().lgbm_b200_booster_get_gradients(self._handle, C.ptr(g), C.ptr(h)))
        return g, h

    def last_train_ms(self):
        out = np.zeros(3, dtype=np.float64)
        C.check(C.lib().lgbm_b200_booster_phase_ms(self._handle, C.ptr(out)))
        return float(out[1])

    KERNEL_CLASSES = ("prepare", "build", "fixscan", "partition", "tree_init", "gradients",
                      "finish")

    def profile_iteration(self):
        """One extra iteration with per-kernel-class device timing (CUDA events on the
        library's stream). Returns (ms by class, counts dict)."""
        ms = np.zeros(7, dtype=np.float64)
        cnt = np.zeros(8, dtype=np.int64)
        C.check(C.lib().lgbm_b200_booster_profile_iteration(self._handle, C.ptr(ms), C.ptr(cnt)))
        self._trees = None
        return (dict(zip(self.KERNEL_CLASSES, ms.tolist())),
                {"launches": int(cnt[0]), "builds": int(cnt[1]), "rows_built": int(cnt[2]),
                 "splits": int(cnt[3]), "rows_parted": int(cnt[4]), "fused": bool(cnt[5]),
                 "lookahead_runs": int(cnt[6]), "lookahead_hits": int(cnt[7])})

    def profile_pipeline(self, iterations=5):
        """`iterations` more iterations through a graph of the training pipeline whose
        tree kernels stamp their device-time spans. Returns (mean summed span ms per
        iteration by kernel class, {"ms_per_iter": mean iteration ms, "lookahead": mean
        summed look-ahead partition spans, and the tree counters per iteration; rows_parted_ctl
        / rows_built_ctl: the rows of the main partitions that ran inside control steps})."""
        span = np.zeros(7, dtype=np.float64)
        it = np.zeros(2, dtype=np.float64)
        cnt = np.zeros(10, dtype=np.int64)
        C.check(C.lib().lgbm_b200_booster_profile_pipeline(self._handle, int(iterations),
                                                           C.ptr(span), C.ptr(it), C.ptr(cnt)))
        self._trees = None
        n = float(iterations)
        return (dict(zip(self.KERNEL_CLASSES, span.tolist())),
                {"ms_per_iter": float(it[0]), "lookahead": float(it[1]),
                 "stamped_launches": cnt[0] / n, "builds": cnt[1] / n, "rows_built": cnt[2] / n,
                 "splits": cnt[3] / n, "rows_parted": cnt[4] / n, "fused": bool(cnt[5]),
                 "lookahead_runs": cnt[6] / n, "lookahead_hits": cnt[7] / n,
                 "rows_parted_ctl": cnt[8] / n, "rows_built_ctl": cnt[9] / n})

    # control-step phase marks (CtlPhase), each the latest CTA's time at that point
    CONTROL_PHASES = ("prep", "loaded", "fixed", "scanned", "features", "staged", "picked",
                      "written")
    # partition phase marks (PartPhase), each the latest tile-holding CTA's time at that point
    PARTITION_PHASES = ("start", "ready", "loaded", "prefix", "tiles", "flushed")
    STEP_MARKS = len(CONTROL_PHASES) + 2 * len(PARTITION_PHASES)

    def profile_chain(self):
        """What held the split chain in the last iteration profile_pipeline ran, from the
        raw spans. Control step s + 1 starts after control step s, the main-stream
        partition s and the look-ahead partition s - 1 have ended (graph edges). Over the
        steps, the time from one control step's start to the next one's is split into the
        control step's own span, the main partition's run past it, the separate build's
        run past that (no fused partition), the look-ahead's run past all of them, and the
        gap from the last of them to the next control step's first CTA (launch and
        scheduling). ms summed over the steps of the tree; "lookahead_limited" counts the
        steps whose look-ahead ended last. "control_phases": the control step's span split
        at its phase marks (time to each mark from the previous one, summed). "main_noop" /
        "main_run": the main partitions shorter / longer than 8 us (it found its leaf
        partitioned by the look-ahead, or ran), with their mean delay after the control
        step and mean span in us (and [step, span us] of each run); "lookahead_span_us":
        the mean look-ahead span. "lookahead_phases_us" / "main_run_phases_us": the mean
        look-ahead span / main run split at the partition's marks (the latest tile-holding
        CTA's entry, its setup, first tile routed, that tile's prefix, last tile written,
        histogram flushed, then the launch's exit)."""
        n = C._i32(0)
        C.check(C.lib().lgbm_b200_booster_profile_spans(self._handle, 0, None, None, None,
                                                        ctypes.byref(n)))
        st = np.zeros(n.value, dtype=np.uint64)
        en = np.zeros(n.value, dtype=np.uint64)
        ph = np.zeros((n.value, self.STEP_MARKS), dtype=np.uint64)
        C.check(C.lib().lgbm_b200_booster_profile_spans(self._handle, n.value, C.ptr(st),
                                                        C.ptr(en), C.ptr(ph), ctypes.byref(n)))
        none = np.iinfo(np.uint64).max

        def span(k):
            if k < 0 or k >= len(st) or st[k] == none or en[k] < st[k]:
                return None
            return int(st[k]), int(en[k])

        out = {"control_step": 0.0, "main_partition_past": 0.0, "build_past": 0.0,
               "lookahead_past": 0.0,
               "launch_gap": 0.0, "steps": 0, "lookahead_limited": 0, "main_limited": 0,
               "before_first_step": 0.0, "tree": 0.0, "control_phases": {},
               "main_noop": {"n": 0, "launch_after_control_us": 0.0, "span_us": 0.0},
               "main_run": {"n": 0, "launch_after_control_us": 0.0, "span_us": 0.0,
                            "steps": []},
               "lookahead_span_us": 0.0, "lookahead_n": 0,
               "lookahead_phases_us": {}, "main_run_phases_us": {}}
        nc, npp = len(self.CONTROL_PHASES), len(self.PARTITION_PHASES)

        def part_phases(sp_, marks_, acc):
            # a partition launch's span split at its marks (the latest tile-holding CTA's
            # entry, setup, first tile routed, its prefix, last tile, flush), then its exit
            prev_ = sp_[0]
            for name_, t_ in zip(self.PARTITION_PHASES + ("exit",),
                                 [int(v) for v in marks_] + [sp_[1]]):
                if t_ == 0:
                    continue
                acc[name_] = acc.get(name_, 0.0) + max(t_ - prev_, 0) * 1e-3
                prev_ = max(prev_, t_)
        steps = (len(st) - 1) // 4
        first = span(1)
        root = span(0)
        if first and root:
            out["before_first_step"] = (first[0] - root[0]) * 1e-6
        for s in range(steps - 1):
            ctl, nxt = span(1 + 4 * s), span(1 + 4 * (s + 1))
            if ctl is None or nxt is None:
                break
            main = span(1 + 4 * s + 1)
            build = span(1 + 4 * s + 3)  # the separate build (no fused partition)
            la = span(1 + 4 * (s - 1) + 2) if s >= 1 else None
            t = ctl[1]
            out["control_step"] += (ctl[1] - ctl[0]) * 1e-6
            lim = "control"
            if main and main[1] > t:
                out["main_partition_past"] += (main[1] - t) * 1e-6
                t = main[1]
                lim = "main"
            if build and build[1] > t:
                out["build_past"] += (build[1] - t) * 1e-6
                t = build[1]
                lim = "build"
            if la and la[1] > t:
                out["lookahead_past"] += (la[1] - t) * 1e-6
                t = la[1]
                lim = "lookahead"
            out["launch_gap"] += max(nxt[0] - t, 0) * 1e-6
            out["lookahead_limited"] += lim == "lookahead"
            out["main_limited"] += lim == "main"
            out["steps"] += 1
            if main:  # a main partition that found its leaf done is short: a no-op
                kind = "noop" if main[1] - main[0] < 8000 else "run"
                m = out["main_" + kind]
                m["n"] += 1
                m["launch_after_control_us"] += (main[0] - ctl[1]) * 1e-3
                m["span_us"] += (main[1] - main[0]) * 1e-3
                if kind == "run":
                    m["steps"].append([s, round((main[1] - main[0]) * 1e-3, 1)])
                    part_phases(main, ph[s][nc + npp:nc + 2 * npp], out["main_run_phases_us"])
            own_la = span(1 + 4 * s + 2)
            if own_la:
                out["lookahead_span_us"] += (own_la[1] - own_la[0]) * 1e-3
                out["lookahead_n"] += 1
                part_phases(own_la, ph[s][nc:nc + npp], out["lookahead_phases_us"])
            # inside the control step: entry, the phase marks in order, exit
            marks = [ctl[0]] + [int(v) for v in ph[s][:nc]] + [ctl[1]]
            prev = marks[0]
            for name, t_m in zip(self.CONTROL_PHASES + ("exit",), marks[1:]):
                if t_m == 0:  # not reached (a scan-free step, or a CTA with no feature)
                    continue
                out["control_phases"][name] = out["control_phases"].get(name, 0.0) + \
                    max(t_m - prev, 0) * 1e-6
                prev = max(prev, t_m)
        if out["lookahead_n"]:
            out["lookahead_span_us"] /= out["lookahead_n"]
            for k in out["lookahead_phases_us"]:
                out["lookahead_phases_us"][k] /= out["lookahead_n"]
        if out["main_run"]["n"]:
            for k in out["main_run_phases_us"]:
                out["main_run_phases_us"][k] /= out["main_run"]["n"]
        for kind in ("main_noop", "main_run"):  # means per launch
            m = out[kind]
            if m["n"]:
                m["launch_after_control_us"] /= m["n"]
                m["span_us"] /= m["n"]
        ends = [e[1] for e in map(span, range(len(st))) if e is not None]
        if first and ends:
            out["tree"] = (max(ends) - (root[0] if root else first[0])) * 1e-6
        return out

    def profile_launches(self):
        """(kernel class name, device ms) of every span timed by the last
        profile_iteration, in launch order."""
        n = C._i32(0)
        C.check(C.lib().lgbm_b200_booster_profile_launches(self._handle, 0, None, None,
                                                           ctypes.byref(n)))
        cls = np.zeros(n.value, dtype=np.int32)
        ms = np.zeros(n.value, dtype=np.float32)
        C.check(C.lib().lgbm_b200_booster_profile_launches(self._handle, n.value, C.ptr(cls),
                                                           C.ptr(ms), ctypes.byref(n)))
        return [(self.KERNEL_CLASSES[c], float(m)) for c, m in zip(cls, ms)]

    def predict(self, data, raw_score=False):
        """Predictions for raw feature rows [n, num_features] on the device: the trees'
        leaf values summed in tree order (the boost-from-average score is in the first
        tree), then the sigmoid for a binary model unless raw_score."""
        if self._predictor is None:
            self._predictor = Predictor(self.model(), int(self.params.get("device", 0)))
        return self._predictor.predict(data, raw_score=raw_score)

    def __del__(self):
        try:
            if self._handle is not None:
                C.lib().lgbm_b200_booster_destroy(self._handle)
        except Exception:
            pass


def train(params, train_set, num_boost_round=100, comm=None):
    """lightgbm_rs.train (engine.py:254): boosting on the device for num_boost_round.
    With comm (distributed.Communicator), data-parallel over the ranks' row shards."""
    p = dict(params or {})
    for k in ("num_iterations", "num_iteration", "n_iter", "num_tree", "num_trees",
              "num_round", "num_rounds", "num_boost_round", "n_estimators"):
        if k in p:
            num_boost_round = int(p.pop(k))
    if isinstance(train_set, Dataset):
        # the parameters given here reach the dataset; its own binning stays as found
        train_set.params.update({_ALIASES.get(k, k): v for k, v in p.items()})
    b = Booster(p, train_set, comm=comm)
    b.update(int(num_boost_round))
    return b


def categorical_bitsets(tree, mappers):
    """cat_boundaries / cat_threshold of a tree as the LightGBM model text holds them
    (Tree::split_categorical, lgbm-model/src/tree.rs:710-770): for each categorical node
    in node order, the bitset of the categories whose bins the node sends left."""
    bounds, words = [0], []
    for node, dt in enumerate(tree["decision_type"]):
        if not (int(dt) & 1):
            continue
        b2c = mappers[int(tree["split_feature"][node])]["bin_to_category"]
        bits = tree["cat_bins"][node]
        cats = [int(b2c[b]) for b in range(min(len(b2c), 256))
                if (int(bits[b >> 5]) >> (b & 31)) & 1]
        blk = [0] * (max(cats) // 32 + 1 if cats else 0)
        for c in cats:
            blk[c // 32] |= 1 << (c % 32)
        words.extend(blk)
        bounds.append(bounds[-1] + len(blk))
    return bounds, words
