"""The bench's algorithmic byte model (no GPU): moving the main partitions' rows into the
control step only moves their bytes between the two kernels' entries."""

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def test_partition_bytes_split_between_kernels():
    import bench

    rows, F = 10_500_000, 28
    base = {"rows_parted": 100_813_140, "rows_built": 35_815_399, "fused": 1}
    whole = bench.kernel_bytes(base, rows, "quantized", F)
    assert whole["partition_ctl"] == 0
    # the root's partition (identity order, no index read) and some others inside control
    # steps: the two entries add up to the same bytes
    split = bench.kernel_bytes(dict(base, rows_parted_ctl=40_000_000, rows_built_ctl=9_000_000),
                               rows, "quantized", F)
    assert split["partition"] + split["partition_ctl"] == whole["partition"]
    assert split["child_hist_fused"] == whole["child_hist_fused"]
    assert split["build"] == whole["build"]
    # per parent row: 1 B bin + 4 B index written + 4 B index read, except the root's rows
    assert split["partition_ctl"] == (40_000_000 * 5 + (40_000_000 - rows) * 4 +
                                      9_000_000 * (F - 1 + 2))
