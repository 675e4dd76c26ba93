"""The collective sweep's markdown tables: one per (N, dtype, op), ratios NCCL / nexar."""
from nexar_b200.bench.sweep_table import tables


def _rec(op, impl, b, us, n=2):
    return {"op": op, "impl": impl, "dtype": "bf16", "bytes": b, "n_gpus": n, "us": us,
            "algbw_gbs": b / us / 1e3, "busbw_gbs": b / us / 1e3}


def test_tables_ratios_and_grouping():
    recs = [_rec("all_reduce", "nexar", 1024, 5.0), _rec("all_reduce", "nccl", 1024, 10.0),
            _rec("all_reduce", "nccl_group", 1024, 8.0), _rec("all_reduce", "nexar", 1 << 20, 20.0),
            _rec("all_reduce", "nccl", 1 << 20, 18.0), _rec("broadcast", "nexar", 1024, 4.0, n=4)]
    md = tables(recs)
    assert "### all_reduce, bf16, 2 GPUs" in md and "### broadcast, bf16, 4 GPUs" in md
    assert "| 1 KB | 5.0 | 10.0 | 8.0 |" in md
    assert "| 2.00 | 1.60 |" in md
    assert "lowest NCCL / nexar ratio: 0.90" in md
