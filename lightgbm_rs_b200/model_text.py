"""LightGBM model text (v4) and the ensemble layout of the device predictor.

`dump` writes a model the way GBDT::SaveModelToString does (the reference's
lgbm-model/src/model_text.rs:216-320 and Tree::to_string, lgbm-model/src/tree.rs:800-830):
the header, one `Tree=i` block per tree with `tree_sizes` holding each block's byte
length, `end of trees`, the split-count feature importances, then a parameters block.
Per-tree number formats are load-bearing: `%.17g` for threshold, leaf_value and
leaf_weight; `%g` for split_gain, internal_value, internal_weight and shrinkage.

`parse` reads model text back (model_text.rs:53-196, Tree::parse), and `flatten` lays an
ensemble out for `lgbm_b200_predictor_create` and for the oracle's checker.

`from_booster` turns a trained booster into a model: real thresholds from the bin upper
bounds (the BinMapper value of the split bin), categorical nodes as bitsets of real
categories (Tree::split_categorical, tree.rs:710-770), the boost-from-average score
folded into the first tree (Tree::add_bias, tree.rs:1161-1168), and each internal node's
hessian sum (LightGBM writes the pre-split leaf weight; it is printed with 6 digits, so
the sum of the node's leaf weights gives the same text).
"""

import numpy as np

__all__ = ["Model", "parse", "dump", "flatten", "from_booster"]

_OBJECTIVE_TEXT = {"binary": "binary sigmoid:{sigmoid:g}", "regression": "regression",
                   "lambdarank": "lambdarank"}


class Model:
    """A tree ensemble with its model-text header fields."""

    def __init__(self, trees, max_feature_idx, objective="regression", feature_names=None,
                 feature_infos=None, num_class=1, num_tree_per_iteration=1, label_index=0,
                 parameters=None, sigmoid=1.0):
        self.trees = trees
        self.max_feature_idx = int(max_feature_idx)
        self.objective = objective
        nf = self.max_feature_idx + 1
        self.feature_names = list(feature_names) if feature_names is not None else \
            [f"Column_{i}" for i in range(nf)]
        self.feature_infos = list(feature_infos) if feature_infos is not None else ["none"] * nf
        self.num_class = int(num_class)
        self.num_tree_per_iteration = int(num_tree_per_iteration)
        self.label_index = int(label_index)
        self.parameters = parameters
        self.sigmoid = float(sigmoid)

    @property
    def objective_name(self):
        return (self.objective or "regression").split()[0]


def _ints(a):
    return " ".join(str(int(v)) for v in a)


def _g17(a):
    return " ".join("%.17g" % float(v) for v in a)


def _g6(a):
    return " ".join("%g" % float(v) for v in a)


def tree_to_string(t):
    """Tree::to_string (tree.rs:800-830): the block after the `Tree=i` line."""
    out = [f"num_leaves={int(t['num_leaves'])}", f"num_cat={int(t.get('num_cat', 0))}",
           f"split_feature={_ints(t['split_feature'])}",
           f"split_gain={_g6(np.asarray(t['split_gain'], np.float32))}",
           f"threshold={_g17(t['threshold'])}",
           f"decision_type={_ints(np.asarray(t['decision_type'], np.int8))}",
           f"left_child={_ints(t['left_child'])}", f"right_child={_ints(t['right_child'])}",
           f"leaf_value={_g17(t['leaf_value'])}", f"leaf_weight={_g17(t['leaf_weight'])}",
           f"leaf_count={_ints(t['leaf_count'])}",
           f"internal_value={_g6(t['internal_value'])}",
           f"internal_weight={_g6(t['internal_weight'])}",
           f"internal_count={_ints(t['internal_count'])}"]
    if int(t.get("num_cat", 0)) > 0:
        out.append(f"cat_boundaries={_ints(t['cat_boundaries'])}")
        out.append(f"cat_threshold={_ints(t['cat_threshold'])}")
    out.append("is_linear=0")
    out.append("shrinkage=%g" % float(t.get("shrinkage", 1.0)))
    return "\n".join(out) + "\n\n"


def _importances(model):
    """Split counts per feature over nodes with a positive gain (model_text.rs:290-306),
    stable-sorted by count, descending."""
    cnt = np.zeros(model.max_feature_idx + 1, dtype=np.int64)
    for t in model.trees:
        for f, g in zip(t["split_feature"], np.asarray(t["split_gain"], np.float32)):
            if g > 0:
                cnt[int(f)] += 1
    order = sorted((i for i in range(len(cnt)) if cnt[i] > 0), key=lambda i: -cnt[i])
    return [(model.feature_names[i], int(cnt[i])) for i in order]


def dump(model):
    """GBDT::SaveModelToString: the whole model text."""
    head = ["tree", "version=v4", f"num_class={model.num_class}",
            f"num_tree_per_iteration={model.num_tree_per_iteration}",
            f"label_index={model.label_index}", f"max_feature_idx={model.max_feature_idx}"]
    if model.objective:
        head.append(f"objective={model.objective}")
    head.append("feature_names=" + " ".join(model.feature_names))
    head.append("feature_infos=" + " ".join(model.feature_infos))
    blocks = [f"Tree={i}\n{tree_to_string(t)}\n" for i, t in enumerate(model.trees)]
    head.append("tree_sizes=" + " ".join(str(len(b.encode())) for b in blocks))
    text = "\n".join(head) + "\n\n" + "".join(blocks) + "end of trees\n"
    text += "\nfeature_importances:\n"
    text += "".join(f"{name}={c}\n" for name, c in _importances(model))
    params = model.parameters
    if params is None:
        params = "parameters:\n" + "".join(f"[{k}: {v}]\n" for k, v in
                                           [("objective", model.objective_name)]) + \
            "end of parameters\n\npandas_categorical:null\n"
    text += "\n" + params
    return text


def _num(s, dt):
    return np.array([dt(x) for x in s.split()] if s.strip() else [], dtype=dt)


def parse(text):
    """GBDT::LoadModelFromString (model_text.rs:53-196): header fields, the trees, and
    the `parameters:` tail kept verbatim."""
    header = {}
    lines = text.splitlines()
    i = 0
    while i < len(lines) and not lines[i].startswith("Tree="):
        ln = lines[i]
        if "=" in ln:
            k, v = ln.split("=", 1)
            header[k] = v
        i += 1
    trees = []
    cur = None
    while i < len(lines):
        ln = lines[i]
        if ln.startswith("Tree="):
            cur = {}
            trees.append(cur)
        elif ln == "end of trees":
            break
        elif "=" in ln and cur is not None:
            k, v = ln.split("=", 1)
            cur[k] = v
        i += 1
    tail = None
    pos = text.find("\nparameters:\n")
    if pos >= 0:
        tail = text[pos + 1:]
    out = []
    for raw in trees:
        nl = int(raw["num_leaves"])
        t = {"num_leaves": nl, "num_cat": int(raw.get("num_cat", "0"))}
        for k in ("split_feature", "left_child", "right_child", "leaf_count", "internal_count"):
            t[k] = _num(raw.get(k, ""), np.int32)
        t["decision_type"] = _num(raw.get("decision_type", ""), np.int8)
        for k in ("threshold", "leaf_value", "leaf_weight", "internal_value",
                  "internal_weight"):
            t[k] = _num(raw.get(k, ""), np.float64)
        t["split_gain"] = _num(raw.get("split_gain", ""), np.float32)
        t["cat_boundaries"] = _num(raw.get("cat_boundaries", ""), np.int32)
        t["cat_threshold"] = _num(raw.get("cat_threshold", ""), np.uint32)
        t["shrinkage"] = float(raw.get("shrinkage", "1"))
        if raw.get("is_linear", "0") != "0":
            raise ValueError("linear trees are not on this path")
        if len(t["leaf_value"]) != nl or len(t["split_feature"]) != max(nl - 1, 0):
            raise ValueError("tree arrays do not match num_leaves")
        out.append(t)
    obj = header.get("objective")
    sig = 1.0
    if obj and obj.startswith("binary"):
        for tok in obj.split()[1:]:
            if tok.startswith("sigmoid:"):
                sig = float(tok.split(":", 1)[1])
    m = Model(out, int(header["max_feature_idx"]), obj,
              header.get("feature_names", "").split() or None,
              header.get("feature_infos", "").split() or None,
              int(header.get("num_class", "1")),
              int(header.get("num_tree_per_iteration", header.get("num_class", "1"))),
              int(header.get("label_index", "0")), tail, sig)
    if m.num_class != 1:
        raise ValueError("multiclass models are not on this path")
    return m


def flatten(model):
    """The ensemble as lgbm_b200_model arrays: trees concatenated; a categorical node's
    threshold becomes its index into the concatenated cat_boundaries."""
    node_off, leaf_off = [0], [0]
    cols = {k: [] for k in ("split_feature", "threshold", "decision_type", "left_child",
                            "right_child", "leaf_value")}
    cat_b, cat_t = [0], []
    for t in model.trees:
        nn = len(t["split_feature"])
        thr = np.asarray(t["threshold"], np.float64).copy()
        dt = np.asarray(t["decision_type"], np.int8)
        cb = t["cat_boundaries"]
        base = len(cat_b) - 1
        for c in range(int(t.get("num_cat", 0))):
            cat_t.extend(int(w) for w in t["cat_threshold"][cb[c]:cb[c + 1]])
            cat_b.append(len(cat_t))
        for k in range(nn):
            if dt[k] & 1:
                thr[k] = thr[k] + base
        cols["split_feature"].append(np.asarray(t["split_feature"], np.int32))
        cols["threshold"].append(thr)
        cols["decision_type"].append(dt)
        cols["left_child"].append(np.asarray(t["left_child"], np.int32))
        cols["right_child"].append(np.asarray(t["right_child"], np.int32))
        cols["leaf_value"].append(np.asarray(t["leaf_value"], np.float64))
        node_off.append(node_off[-1] + nn)
        leaf_off.append(leaf_off[-1] + int(t["num_leaves"]))
    dts = {"split_feature": np.int32, "threshold": np.float64, "decision_type": np.int8,
           "left_child": np.int32, "right_child": np.int32, "leaf_value": np.float64}
    flat = {k: (np.concatenate(v).astype(dts[k]) if v else np.zeros(0, dts[k]))
            for k, v in cols.items()}
    flat.update(num_trees=len(model.trees), num_features=model.max_feature_idx + 1,
                node_offset=np.array(node_off, np.int32), leaf_offset=np.array(leaf_off, np.int32),
                cat_boundaries=np.array(cat_b, np.int32), cat_threshold=np.array(cat_t, np.uint32),
                num_cat=len(cat_b) - 1, transform=1 if model.objective_name == "binary" else 0,
                sigmoid=model.sigmoid)
    return flat


def _feature_info(m):
    """BinMapper::bin_info_string: `[min:max]` (17 significant digits) for numerical
    features, the categories of the bins joined by `:` for categorical ones, `none` for
    trivial features."""
    if m.get("is_trivial"):
        return "none"
    if m.get("bin_type", 0) == 1:
        return ":".join(str(int(c)) for c in m["bin_to_category"])
    return "[%.17g:%.17g]" % (m["min_val"], m["max_val"])


def _round_to_zero(v):
    return 0.0 if -1e-35 <= v <= 1e-35 else v


def _subtree_weights(t):
    nn = t["num_leaves"] - 1
    w = np.zeros(max(nn, 0), dtype=np.float64)

    def rec(n):
        if n < 0:
            return float(t["leaf_weight"][~n])
        w[n] = rec(int(t["left_child"][n])) + rec(int(t["right_child"][n]))
        return w[n]

    if nn > 0:
        rec(0)
    return w


def from_booster(booster):
    """The model of a trained lightgbm_rs_b200.Booster (trees after shrinkage)."""
    from . import categorical_bitsets

    mappers = booster.train_set.mappers
    if mappers is None:
        raise ValueError("the booster's dataset has no bin mappers")
    lr = float(booster.params["learning_rate"])
    init = booster.init_score()
    trees = []
    for it, bt in enumerate(booster.trees()):
        nl = int(bt["num_leaves"])
        t = {"num_leaves": nl}
        for k in ("split_feature", "left_child", "right_child", "leaf_count",
                  "internal_count"):
            t[k] = np.asarray(bt[k], np.int32)
        t["decision_type"] = np.asarray(bt["decision_type"], np.int8)
        t["split_gain"] = np.asarray(bt["split_gain"], np.float32)
        t["leaf_value"] = np.asarray(bt["leaf_value"], np.float64).copy()
        t["leaf_weight"] = np.asarray(bt["leaf_weight"], np.float64)
        t["internal_value"] = np.asarray(bt["internal_value"], np.float64).copy()
        thr = np.zeros(max(nl - 1, 0), dtype=np.float64)
        for n in range(nl - 1):
            m = mappers[int(t["split_feature"][n])]
            if t["decision_type"][n] & 1:
                thr[n] = float(bt["threshold_bin"][n])  # the categorical-node index
            else:
                thr[n] = float(m["upper"][int(bt["threshold_bin"][n])])
        t["threshold"] = thr
        bounds, words = categorical_bitsets(bt, mappers)
        t["num_cat"] = len(bounds) - 1
        t["cat_boundaries"] = np.array(bounds, np.int32)
        t["cat_threshold"] = np.array(words, np.uint32)
        t["internal_weight"] = _subtree_weights(t)
        t["shrinkage"] = lr if nl > 1 else 1.0
        if it == 0 and abs(init) > float(np.float32(1e-15)):
            t["leaf_value"] = np.array([_round_to_zero(v + init) for v in t["leaf_value"]])
            t["internal_value"] = np.array([_round_to_zero(v + init)
                                            for v in t["internal_value"]])
        trees.append(t)
    obj = booster.objective
    objective = _OBJECTIVE_TEXT.get(obj, obj).format(sigmoid=float(booster.params["sigmoid"]))
    return Model(trees, len(mappers) - 1, objective,
                 feature_infos=[_feature_info(m) for m in mappers],
                 sigmoid=float(booster.params["sigmoid"]))
