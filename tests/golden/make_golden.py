"""Copy the reference's golden vectors for the hot path into tests/golden/.

The reference (BectorVoom/lightgbm_rs) keeps its golden vectors as text files
captured from LightGBM C++ 4.6.0.99 / lightgbm==4.6.0. The parity tests read
them from this directory so they also run where the reference tree is absent
(the GPU box). Large files are stored gzip-compressed; contents are unchanged.

Usage: python tests/golden/make_golden.py [REFERENCE_ROOT]
"""

import gzip
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))

# (path inside the reference project, compress?[, name under tests/golden/])
FILES = [
    ("crates/oracle-harness/tests/fixtures/kernels/histogram.txt", True),
    ("crates/oracle-harness/tests/fixtures/kernels/split.txt", False),
    ("crates/oracle-harness/tests/fixtures/kernels/subtract.txt", False),
    ("crates/oracle-harness/tests/fixtures/kernels/partition.txt", False),
    ("crates/oracle-harness/tests/fixtures/learner/spine_real.txt", False),
    ("crates/oracle-harness/tests/fixtures/learner/mfb_pos_real.txt", False),
    ("crates/oracle-harness/tests/fixtures/learner/real_gh.txt", False),
    ("crates/oracle-harness/tests/fixtures/boosting/binary_gh_iter1.txt", False),
    ("crates/oracle-harness/tests/fixtures/boosting/binary_gh_iterN.txt", False),
    ("crates/oracle-harness/tests/fixtures/boosting/binary_scores.txt", False),
    ("crates/oracle-harness/tests/fixtures/boosting/binary_spine_model.txt", False),
    ("crates/oracle-harness/tests/fixtures/boosting/regression_scores.txt", False),
    ("crates/oracle-harness/tests/fixtures/boosting/regression_gh_iter1.txt", False),
    ("crates/oracle-harness/tests/fixtures/quantized/quant_binary.xy.csv", True),
    ("crates/oracle-harness/tests/fixtures/quantized/quant_binary.pred", False),
    ("crates/oracle-harness/tests/fixtures/quantized/quant_binary.pred_exact", False),
    ("crates/oracle-harness/tests/fixtures/quantized/quant_binary.json", False),
    ("crates/lgbm-dataset/tests/fixtures/numeric_binning.txt", True),
    ("crates/lgbm-dataset/tests/fixtures/categorical_folding.txt", False),
    ("crates/oracle-harness/tests/fixtures/categorical/cat_onehot.txt", False),
    ("crates/oracle-harness/tests/fixtures/categorical/cat_onehot.bins.json", False),
    ("crates/oracle-harness/tests/fixtures/categorical/cat_manyvsmany.txt", False),
    ("crates/oracle-harness/tests/fixtures/categorical/cat_manyvsmany.bins.json", False),
    ("crates/oracle-harness/fixtures/rng_sequence.txt", True),
    ("crates/oracle-harness/tests/fixtures/rank/lambdarank_gh_iter1.txt", False),
    ("crates/oracle-harness/tests/fixtures/rank/lambdarank_scores.txt", False),
    ("crates/oracle-harness/tests/fixtures/rank/rank_lambdarank_byq0_es0_model.txt", False),
    ("crates/oracle-harness/tests/fixtures/boosting/binary_spine_pred.txt", False),
    ("crates/oracle-harness/tests/fixtures/predict_modes/numeric/model.txt", False,
     "predict_numeric_model.txt"),
    ("crates/oracle-harness/tests/fixtures/predict_modes/numeric/X.txt", False,
     "predict_numeric_X.txt"),
    ("crates/oracle-harness/tests/fixtures/predict_modes/numeric/early_stop.txt", False,
     "predict_numeric_early_stop.txt"),
    ("crates/oracle-harness/tests/fixtures/predict_modes/categorical/model.txt", False,
     "predict_categorical_model.txt"),
    ("crates/oracle-harness/tests/fixtures/predict_modes/categorical/X.txt", False,
     "predict_categorical_X.txt"),
    ("crates/oracle-harness/tests/fixtures/predict_modes/categorical/contrib.txt", False,
     "predict_categorical_contrib.txt"),
    ("crates/oracle-harness/tests/fixtures/predict_modes/numeric/contrib.txt", False,
     "predict_numeric_contrib.txt"),
    ("crates/oracle-harness/tests/fixtures/na_missing/model_real.txt", False,
     "na_missing_model.txt"),
    ("crates/oracle-harness/tests/fixtures/json_dump/regression_3tree/model.txt", False,
     "regression_3tree_model.txt"),
]


def main() -> None:
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LGBM_REF_ROOT")
    if not ref:
        sys.exit("usage: make_golden.py <reference checkout> (or set LGBM_REF_ROOT)")
    for entry in FILES:
        rel, compress = entry[0], entry[1]
        src = os.path.join(ref, rel)
        name = entry[2] if len(entry) > 2 else os.path.basename(rel)
        if not os.path.exists(src):
            print(f"missing: {src}")
            continue
        if compress:
            dst = os.path.join(HERE, name + ".gz")
            with open(src, "rb") as fi, gzip.GzipFile(dst, "wb", mtime=0) as fo:
                shutil.copyfileobj(fi, fo)
        else:
            dst = os.path.join(HERE, name)
            shutil.copyfile(src, dst)
        print(f"{rel} -> {os.path.relpath(dst, HERE)}")


if __name__ == "__main__":
    main()
