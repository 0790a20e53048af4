"""Summarise ncu CSV output for the profiles/ notes.

    python -m linearard_b200.ncu_summary launches launches.csv
        per kernel: launches, total gpu__time_duration, share of the total
    python -m linearard_b200.ncu_summary raw report.csv
        selected raw metrics (``ncu -i x.ncu-rep --page raw --csv``) per kernel
"""
from __future__ import annotations

import collections
import csv
import io
import sys

SHORT = (("sm100_dq_kernel", "sm100_dq_kernel"),
         ("sm100_dk_kernel", "sm100_dk_kernel"),
         ("sm100_forward_kernel", "sm100_forward_kernel"),
         ("scale_lse_kernel", "scale_lse_kernel"),
         ("generic_backward_kernel", "generic_backward_kernel"),
         ("generic_forward_kernel", "generic_forward_kernel"),
         ("reduce_partials_kernel", "reduce_partials_kernel"),
         ("pack_mask_kernel", "pack_mask_kernel"))

RAW_KEYS = ("gpu__time_duration.sum", "dram__bytes_read.sum", "dram__bytes_write.sum",
            "dram__throughput.avg.pct_of_peak_sustained_elapsed",
            "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
            "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
            "sm__inst_executed_pipe_xu.avg.pct_of_peak_sustained_active",
            "sm__pipe_fma_cycles_active.avg.pct_of_peak_sustained_active",
            "sm__pipe_alu_cycles_active.avg.pct_of_peak_sustained_active",
            "lts__t_sectors_op_red.sum", "lts__t_sectors_op_atom.sum",
            "lts__throughput.avg.pct_of_peak_sustained_elapsed",
            "l1tex__throughput.avg.pct_of_peak_sustained_active",
            "sm__throughput.avg.pct_of_peak_sustained_elapsed",
            "launch__registers_per_thread", "sm__warps_active.avg.pct_of_peak_sustained_active")


def short_name(name: str) -> str:
    for key, s in SHORT:
        if key in name:
            return s
    return name.split("(")[0][-70:]


def _rows(path):
    text = open(path, errors="replace").read()
    start = text.find('"ID"')
    return list(csv.reader(io.StringIO(text[start:])))


_TIME_NS = {"nsecond": 1.0, "ns": 1.0, "usecond": 1e3, "us": 1e3, "msecond": 1e6, "ms": 1e6,
            "second": 1e9, "s": 1e9}


def launches(path):
    rows = _rows(path)
    hdr = rows[0]
    ki, vi, mi = hdr.index("Kernel Name"), hdr.index("Metric Value"), hdr.index("Metric Name")
    ui = hdr.index("Metric Unit") if "Metric Unit" in hdr else None
    agg = collections.OrderedDict()
    for r in rows[1:]:
        if len(r) < len(hdr) or r[mi] != "gpu__time_duration.sum":
            continue
        a = agg.setdefault(short_name(r[ki]), [0, 0.0])
        a[0] += 1
        scale = _TIME_NS.get(r[ui], 1.0) if ui is not None else 1.0
        a[1] += float(r[vi].replace(",", "")) * scale
    tot = sum(v[1] for v in agg.values())
    print(f"{'kernel':58s} {'launches':>8s} {'total ms':>10s} {'share':>7s}")
    for k, (n, t) in sorted(agg.items(), key=lambda x: -x[1][1]):
        print(f"{k:58s} {n:8d} {t / 1e6:10.3f} {100 * t / tot:6.2f}%")
    print(f"{'total':58s} {'':8s} {tot / 1e6:10.3f}")


def raw(path):
    rows = _rows(path)
    hdr = rows[0]
    units = rows[1] if len(rows) > 1 and not rows[1][0].strip().isdigit() else [""] * len(hdr)
    ki = hdr.index("Kernel Name")
    for r in rows[1:]:
        if len(r) < len(hdr) or not r[0].strip().isdigit():
            continue
        print(f"== {short_name(r[ki])} (ID {r[0]})")
        for key in RAW_KEYS:
            if key in hdr:
                i = hdr.index(key)
                print(f"   {key:70s} {r[i]:>14s} {units[i]}")


if __name__ == "__main__":
    {"launches": launches, "raw": raw}[sys.argv[1]](sys.argv[2])
