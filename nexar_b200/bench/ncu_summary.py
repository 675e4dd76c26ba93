"""Summarise an Nsight Compute capture as roofline figures (one markdown row per launch).

    python -m nexar_b200.bench.ncu_summary prof.ncu-rep [--flops F] [--bytes B] [--peaks MEASURED_PEAKS.json]
    ncu -i prof.ncu-rep --page raw --csv > raw.csv && python -m nexar_b200.bench.ncu_summary raw.csv

Reads the raw page (``ncu -i <rep> --page raw --csv``; a ``.csv`` file is read
as that page directly) and prints, per captured launch: duration, DRAM bytes
read and written, tensor-pipe activity, active warps, registers per thread,
the achieved DRAM bandwidth and, given the launch's algorithmic ``--flops`` /
``--bytes``, the achieved rate as a fraction of the measured peaks
(``MEASURED_PEAKS.json``: ``hbm_gbs``, ``bf16_tflops``).
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import subprocess
import sys
from typing import Dict, List, Optional

# metric name prefixes -> column label
METRICS = [
    ("gpu__time_duration.sum", "duration"),
    ("dram__bytes_read.sum", "dram_read"),
    ("dram__bytes_write.sum", "dram_write"),
    ("sm__pipe_tensor_cycles_active", "tensor_active"),
    ("sm__warps_active", "warps_active"),
    ("launch__registers_per_thread", "regs"),
    ("gpu__dram_throughput", "dram_throughput"),
]

_TIME_SCALE = {"ns": 1e-9, "nsecond": 1e-9, "usecond": 1e-6, "us": 1e-6, "msecond": 1e-3, "ms": 1e-3,
               "second": 1.0, "s": 1.0}
_BYTE_SCALE = {"byte": 1, "kbyte": 1e3, "mbyte": 1e6, "gbyte": 1e9, "tbyte": 1e12,
               "kibyte": 1024, "mibyte": 1024 ** 2, "gibyte": 1024 ** 3}


def _num(s: str) -> Optional[float]:
    try:
        return float(str(s).replace(",", ""))
    except ValueError:
        return None


def parse_raw_csv(text: str) -> List[Dict[str, object]]:
    """Rows of the raw page: one dict per launch with the kernel name and the
    metrics above converted to seconds, bytes and plain numbers."""
    rows = list(csv.reader(io.StringIO(text)))
    start = next((i for i, r in enumerate(rows) if "Kernel Name" in r), None)
    if start is None:
        raise ValueError("not an ncu raw page: no 'Kernel Name' column")
    header, units = rows[start], rows[start + 1] if start + 1 < len(rows) else []
    has_units = bool(units) and "Kernel Name" not in units and not any(_num(u) is not None for u in units[-3:])
    body = rows[start + 2:] if has_units else rows[start + 1:]
    cols = {}
    for prefix, label in METRICS:
        for j, name in enumerate(header):
            if name.startswith(prefix):
                cols[label] = j
                break
    out = []
    ki = header.index("Kernel Name")
    for r in body:
        if len(r) <= ki or not r[ki]:
            continue
        rec: Dict[str, object] = {"kernel": r[ki]}
        for label, j in cols.items():
            v = _num(r[j]) if j < len(r) else None
            unit = (units[j].strip().lower() if has_units and j < len(units) else "")
            if v is not None and label == "duration":
                v *= _TIME_SCALE.get(unit, 1e-9)
            elif v is not None and label in ("dram_read", "dram_write"):
                v *= _BYTE_SCALE.get(unit, 1)
            rec[label] = v
        out.append(rec)
    return out


def load_peaks(path: Optional[str]) -> Dict[str, float]:
    """The measured denominators; the fallback figures when the file is absent."""
    if path and os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def summarise(recs: List[Dict[str, object]], peaks: Dict[str, float], flops: Optional[float] = None,
              algo_bytes: Optional[float] = None) -> str:
    src = peaks["source"]
    lines = [
        "| kernel | duration (us) | DRAM read / write (MB) | DRAM GB/s | tensor pipe % | warps active % | regs |"
        + (" TFLOP/s (of " + src + " peak) |" if flops else "")
        + (" algorithmic GB/s (of " + src + " HBM) |" if algo_bytes else ""),
        "|---|---|---|---|---|---|---|" + ("---|" if flops else "") + ("---|" if algo_bytes else ""),
    ]
    for r in recs:
        t = r.get("duration")
        rd, wr = r.get("dram_read") or 0.0, r.get("dram_write") or 0.0
        gbs = (rd + wr) / t / 1e9 if t else None

        def fmt(v, nd=1):
            return "-" if v is None else f"{v:.{nd}f}"

        row = (f"| `{r['kernel'][:60]}` | {fmt(t * 1e6 if t else None)} | {rd / 1e6:.1f} / {wr / 1e6:.1f} | "
               f"{fmt(gbs)} | {fmt(r.get('tensor_active'))} | {fmt(r.get('warps_active'))} | "
               f"{fmt(r.get('regs'), 0)} |")
        if flops:
            tf = flops / t / 1e12 if t else None
            row += f" {fmt(tf)} ({fmt(tf / peaks['bf16_tflops'] if tf else None, 2)}) |"
        if algo_bytes:
            ab = algo_bytes / t / 1e9 if t else None
            row += f" {fmt(ab)} ({fmt(ab / peaks['hbm_gbs'] if ab else None, 2)}) |"
        lines.append(row)
    return "\n".join(lines)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("report", help=".ncu-rep file, or a .csv of `ncu -i <rep> --page raw --csv`")
    ap.add_argument("--flops", type=float, default=None, help="algorithmic FLOPs of one launch")
    ap.add_argument("--bytes", type=float, default=None, help="algorithmic DRAM bytes of one launch")
    ap.add_argument("--peaks", default=os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json"))
    args = ap.parse_args(argv)
    if args.report.endswith(".csv"):
        with open(args.report) as f:
            text = f.read()
    else:
        text = subprocess.run(["ncu", "-i", args.report, "--page", "raw", "--csv"], check=True,
                              capture_output=True, text=True).stdout
    print(summarise(parse_raw_csv(text), load_peaks(args.peaks), args.flops, args.bytes))
    return 0


if __name__ == "__main__":
    sys.exit(main())
