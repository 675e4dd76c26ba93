"""Markdown tables from the collective sweep's JSONL records.

    python -m nexar_b200.bench.sweep_table sweep_bf16.jsonl [sweep_f32.jsonl ...]

One table per (GPU count, dtype, op): message size, device time of every arm
in microseconds, nexar's bus bandwidth, and the ratio NCCL time / nexar time
(above 1.0: nexar faster) against both NCCL arms (torch's NCCL backend and the
raw NcclGroup calls). ``nexar_sym`` runs on symmetric buffers; NCCL's arms run
on plain (unregistered) buffers, so only the ``nexar`` column is the
like-for-like comparison.
"""
from __future__ import annotations

import json
import sys
from collections import defaultdict

ARMS = ("nexar", "nexar_sym", "nccl", "nccl_group")


def _size(b: int) -> str:
    for unit, div in (("GB", 1 << 30), ("MB", 1 << 20), ("KB", 1 << 10)):
        if b >= div:
            v = b / div
            return f"{v:g} {unit}"
    return f"{b} B"


def tables(records) -> str:
    by = defaultdict(lambda: defaultdict(dict))
    for r in records:
        by[(r["n_gpus"], r["dtype"], r["op"])][r["bytes"]][r["impl"]] = r
    out = []
    for (n, dt, op) in sorted(by):
        rows = by[(n, dt, op)]
        arms = [a for a in ARMS if any(a in v for v in rows.values())]
        out.append(f"### {op}, {dt}, {n} GPUs\n")
        head = ["size"] + [f"{a} us" for a in arms] + ["nexar busbw GB/s", "nccl / nexar", "nccl_group / nexar"]
        out.append("| " + " | ".join(head) + " |")
        out.append("|" + "---|" * len(head))
        worst = None
        for b in sorted(rows):
            v = rows[b]
            cells = [_size(b)] + [f"{v[a]['us']:.1f}" if a in v else "-" for a in arms]
            nx = v.get("nexar")
            cells.append(f"{nx['busbw_gbs']:.1f}" if nx else "-")
            for ref in ("nccl", "nccl_group"):
                if nx and ref in v:
                    ratio = v[ref]["us"] / nx["us"]
                    cells.append(f"{ratio:.2f}")
                    worst = ratio if worst is None else min(worst, ratio)
                else:
                    cells.append("-")
            out.append("| " + " | ".join(cells) + " |")
        if worst is not None:
            out.append(f"\nlowest NCCL / nexar ratio: {worst:.2f}\n")
        else:
            out.append("")
    return "\n".join(out)


def main(argv=None) -> int:
    import argparse
    ap = argparse.ArgumentParser(description="markdown tables from collective sweep JSONL records")
    ap.add_argument("jsonl", nargs="+", help="files written by nexar_b200.bench.collectives --out")
    args = ap.parse_args(argv)
    recs = []
    for p in args.jsonl:
        with open(p) as f:
            recs.extend(json.loads(line) for line in f if line.strip())
    print(tables(recs))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
