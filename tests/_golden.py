"""Parsers for the reference's golden vectors kept under tests/golden/.

Formats follow the reference's own parsers (crates/oracle-harness/tests/
kernel_parity.rs:100-160, :280-360; lgbm-dataset/tests/golden/mod.rs).
"""

import gzip
import os
import struct

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def read_text(name):
    path = os.path.join(GOLDEN, name)
    if os.path.exists(path + ".gz"):
        with gzip.open(path + ".gz", "rt") as f:
            return f.read()
    with open(path) as f:
        return f.read()


def f64_bits(s):
    return struct.unpack("<d", struct.pack("<Q", int(s)))[0]


def f32_bits(s):
    return struct.unpack("<f", struct.pack("<I", int(s)))[0]


def bits_of_f64(x):
    return struct.unpack("<Q", struct.pack("<d", float(x)))[0]


def f64_list(s, sep=";"):
    if not s:
        return np.zeros(0, dtype=np.float64)
    return np.array([int(t) for t in s.split(sep) if t != ""], dtype=np.uint64).view(np.float64)


def f32_list(s, sep=";"):
    if not s:
        return np.zeros(0, dtype=np.float32)
    return np.array([int(t) for t in s.split(sep) if t != ""], dtype=np.uint32).view(np.float32)


def u32_list(s, sep=";"):
    if not s:
        return np.zeros(0, dtype=np.uint32)
    return np.array([int(t) for t in s.split(sep) if t != ""], dtype=np.uint32)


def fields(tokens):
    out = {}
    for t in tokens:
        if "=" in t:
            k, v = t.split("=", 1)
            out[k] = v
    return out


def _records(text):
    for raw in text.splitlines():
        line = raw.strip()
        if not line or line.startswith("#"):
            continue
        yield line.split()


def histogram_cases():
    """kernels/histogram.txt: HCASE/BINS/GRAD/HESS/HIST records."""
    cases = []
    it = _records(read_text("histogram.txt"))
    for t in it:
        if t[0] != "HCASE":
            continue
        f = fields(t[1:])
        rec = {"name": f["name"], "num_bin": int(f["num_bin"])}
        for key in ("BINS", "GRAD", "HESS", "HIST"):
            r = next(it)
            assert r[0] == key
            rec[key] = r[1] if len(r) > 1 else ""
        rec["bins"] = u32_list(rec.pop("BINS"))
        rec["grad"] = f32_list(rec.pop("GRAD"))
        rec["hess"] = f32_list(rec.pop("HESS"))
        rec["hist"] = f64_list(rec.pop("HIST"))
        cases.append(rec)
    return cases


def split_cases():
    """kernels/split.txt: SCASE/SHIST/SCAND_REV/SCAND_FWD/SWIN records."""
    cases = []
    it = _records(read_text("split.txt"))
    for t in it:
        if t[0] != "SCASE":
            continue
        f = fields(t[1:])
        rec = {
            "name": f["name"],
            "num_bin": int(f["num_bin"]),
            "offset": int(f["offset"]),
            "default_bin": int(f["default_bin"]),
            "skip_default_bin": int(f["skip_default_bin"]) != 0,
            "na_as_missing": int(f["na_as_missing"]) != 0,
            "min_data_in_leaf": int(f["min_data_in_leaf"]),
            "min_sum_hessian_in_leaf": f64_bits(f["min_sum_hessian_in_leaf"]),
            "lambda_l1": f64_bits(f["lambda_l1"]),
            "lambda_l2": f64_bits(f["lambda_l2"]),
            "min_gain_to_split": f64_bits(f["min_gain_to_split"]),
            "sum_gradient": f64_bits(f["sum_gradient"]),
            "sum_hessian": f64_bits(f["sum_hessian"]),
            "num_data": int(f["num_data"]),
        }
        r = next(it)
        assert r[0] == "SHIST"
        rec["hist"] = f64_list(r[1] if len(r) > 1 else "")
        next(it)  # SCAND_REV
        next(it)  # SCAND_FWD
        w = next(it)
        assert w[0] == "SWIN"
        wf = fields(w[1:])
        rec["win"] = {
            "is_splittable": int(wf["is_splittable"]) != 0,
            "threshold": int(wf["threshold"]),
            "gain": int(wf["gain"]),
            "left_count": int(wf["left_count"]),
            "right_count": int(wf["right_count"]),
            "left_sum_gradient": int(wf["left_sum_gradient"]),
            "left_sum_hessian": int(wf["left_sum_hessian"]),
            "right_sum_gradient": int(wf["right_sum_gradient"]),
            "right_sum_hessian": int(wf["right_sum_hessian"]),
            "left_output": int(wf["left_output"]),
            "right_output": int(wf["right_output"]),
            "default_left": int(wf["default_left"]) != 0,
        }
        cases.append(rec)
    return cases


def subtract_cases():
    cases = []
    it = _records(read_text("subtract.txt"))
    for t in it:
        if t[0] != "SUBCASE":
            continue
        f = fields(t[1:])
        rec = {"name": f["name"]}
        for key in ("SUBPARENT", "SUBCHILD", "SUBDERIVED"):
            r = next(it)
            assert r[0] == key
            rec[key.lower()] = f64_list(r[1] if len(r) > 1 else "")
        cases.append(rec)
    return cases


def partition_cases():
    """kernels/partition.txt PCASE/PBINS/PORDER/PSPLIT (numeric routing only)."""
    cases = []
    it = _records(read_text("partition.txt"))
    for t in it:
        if t[0] != "PCASE":
            continue
        f = fields(t[1:])
        rec = {k: int(v) for k, v in f.items() if k not in ("name", "note")}
        rec["name"] = f["name"]
        r = next(it)
        assert r[0] == "PBINS"
        rec["bins"] = u32_list(r[1] if len(r) > 1 else "")
        r = next(it)
        assert r[0] == "PORDER"
        rec["order"] = u32_list(r[1] if len(r) > 1 else "")
        r = next(it)
        assert r[0] == "PSPLIT"
        rec["split"] = int(r[1])
        cases.append(rec)
    return cases


def parse_model_text(text):
    """Minimal LightGBM model-text reader: list of per-tree dicts of arrays."""
    trees = []
    cur = None
    for raw in text.splitlines():
        line = raw.strip()
        if line.startswith("Tree="):
            cur = {}
            trees.append(cur)
            continue
        if line == "end of trees":
            break
        if cur is None or "=" not in line:
            continue
        k, v = line.split("=", 1)
        cur[k] = v
    out = []
    for t in trees:
        d = {"num_leaves": int(t["num_leaves"])}
        for k in ("split_feature", "left_child", "right_child", "leaf_count", "internal_count",
                  "decision_type"):
            if k in t:
                d[k] = np.array([int(x) for x in t[k].split()], dtype=np.int64)
        for k in ("threshold", "leaf_value", "leaf_weight", "split_gain", "internal_value"):
            if k in t:
                d[k] = np.array([float(x) for x in t[k].split()], dtype=np.float64)
        d["shrinkage"] = float(t.get("shrinkage", "1"))
        out.append(d)
    return out


def g17(x):
    return "%.17g" % x


def binning_cases():
    """lgbm-dataset numeric_binning.txt (CASE/VALUES/GOLDEN/ASSIGN)."""
    cases = []
    it = _records(read_text("numeric_binning.txt"))
    for t in it:
        if t[0] != "CASE":
            continue
        f = fields(t[1:])
        rec = {
            "name": f["name"],
            "max_bin": int(f["max_bin"]),
            "min_data_in_bin": int(f["min_data_in_bin"]),
            "min_split_data": int(f["min_split_data"]),
            "pre_filter": int(f["pre_filter"]) != 0,
            "use_missing": int(f["use_missing"]) != 0,
            "zero_as_missing": int(f["zero_as_missing"]) != 0,
            "seed": int(f["seed"]),
            "sample_cnt": int(f["sample_cnt"]),
        }
        r = next(it)
        assert r[0] == "VALUES"
        rec["values"] = f64_list(r[1] if len(r) > 1 else "")
        r = next(it)
        assert r[0] == "GOLDEN"
        gf = fields(r[1:])
        rec["golden"] = {
            "num_bin": int(gf["num_bin"]),
            "bin_type": int(gf["bin_type"]),
            "missing_type": int(gf["missing_type"]),
            "default_bin": int(gf["default_bin"]),
            "most_freq_bin": int(gf["most_freq_bin"]),
            "is_trivial": int(gf["is_trivial"]) != 0,
            "upper": f64_list(gf.get("upper", "")),
        }
        r = next(it)
        assert r[0] == "ASSIGN"
        rec["assign"] = u32_list(r[1] if len(r) > 1 else "")
        cases.append(rec)
    return cases


def bits_line(line, kind="f64"):
    toks = [int(t) for t in line.split()]
    if kind == "f64":
        return np.array(toks, dtype=np.uint64).view(np.float64)
    return np.array(toks, dtype=np.uint32).view(np.float32)


def data_lines(name):
    return [l for l in read_text(name).splitlines() if l.strip() and not l.lstrip().startswith("#")]


def categorical_binning_cases():
    """lgbm-dataset categorical_folding.txt (CCASE/VALUES/MAPPER/C2B/B2C/ASSIGN)."""
    cases = []
    it = _records(read_text("categorical_folding.txt"))
    for t in it:
        if t[0] != "CCASE":
            continue
        f = fields(t[1:])
        rec = {k: int(f[k]) for k in ("max_bin", "min_data_in_bin", "use_missing",
                                       "zero_as_missing", "pre_filter", "min_split_data",
                                       "num_rows")}
        rec["name"] = f["name"]
        r = next(it)
        assert r[0] == "VALUES"
        rec["values"] = f64_list(r[1] if len(r) > 1 else "")
        r = next(it)
        assert r[0] == "MAPPER"
        rec["mapper"] = {k: int(v) for k, v in fields(r[1:]).items()}
        r = next(it)
        assert r[0] == "C2B"
        rec["c2b"] = {int(a): int(b) for a, b in (p.split(":") for p in r[1].split(";"))} \
            if len(r) > 1 else {}
        r = next(it)
        assert r[0] == "B2C"
        rec["b2c"] = [int(x) for x in r[1].split(";")] if len(r) > 1 else []
        r = next(it)
        assert r[0] == "ASSIGN"
        rec["assign"] = u32_list(r[1] if len(r) > 1 else "")
        cases.append(rec)
    return cases


def rank_case():
    """The lambdarank cells (oracle-harness rank/ fixtures, captured from lib_lightgbm
    4.6 by the reference's rank_oracle_capture.py): the 30-row, 6-query corpus. Its
    features and labels come from numpy's legacy RandomState(20240607) exactly as the
    capture drew them (randint(0, 8, (30, 3)), then randint(0, 4, 30)); the captured
    labels are checked against the regenerated ones. Returns X, labels (f32),
    query_boundaries, iteration-1 (g, h) and the final raw scores."""
    sc = {}
    for line in read_text("lambdarank_scores.txt").splitlines():
        if "=" in line and not line.startswith("#"):
            k, v = line.strip().split("=", 1)
            sc[k] = v.split(",")
    labels = np.array([int(x) for x in sc["labels"]], dtype=np.uint32).view(np.float32)
    qb = np.array([int(x) for x in sc["query_boundaries"]], dtype=np.int32)
    final = np.array([int(x) for x in sc["scores"]], dtype=np.uint64).view(np.float64)
    gh = {}
    for line in data_lines("lambdarank_gh_iter1.txt"):
        t = line.split()
        gh[t[0]] = np.array([int(x) for x in t[1:]], dtype=np.uint32).view(np.float32)
    rng = np.random.RandomState(20240607)
    X = rng.randint(0, 8, size=(30, 3)).astype(np.float64)
    regen = rng.randint(0, 4, size=30).astype(np.float32)
    assert np.array_equal(regen, labels), "rank corpus regeneration drifted"
    return X, labels, qb, gh["GRAD"], gh["HESS"], final


def bits_matrix(name):
    """`# rows=<n> cols=<m>` (or width=) header + rows of f64 bit patterns."""
    lines = read_text(name).splitlines()
    rows = [[int(t) for t in l.split()] for l in lines[1:] if l.strip() and not l.startswith("#")]
    return np.array(rows, dtype=np.uint64).view(np.float64)


def early_stop_cells(name):
    """`CELL freq=.. margin=.. rows=.. width=..` followed by one f64 bit pattern per row."""
    cells, cur = [], None
    for l in read_text(name).splitlines():
        if l.startswith("CELL"):
            f = dict(t.split("=") for t in l.split()[1:])
            cur = {k: int(v) for k, v in f.items()}
            cur["values"] = []
            cells.append(cur)
        elif l.strip() and not l.startswith("#") and cur is not None:
            cur["values"].append(int(l.split()[0]))
    for c in cells:
        c["values"] = np.array(c["values"], dtype=np.uint64).view(np.float64)
    return cells


MODEL_TEXTS = ["rank_lambdarank_byq0_es0_model.txt", "binary_spine_model.txt",
               "cat_onehot.txt", "cat_manyvsmany.txt", "predict_numeric_model.txt",
               "predict_categorical_model.txt", "na_missing_model.txt",
               "regression_3tree_model.txt"]
