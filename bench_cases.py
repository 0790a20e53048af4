"""Measurement cases beside ``bench.py`` (not part of the library).

    python bench_cases.py profile [--heads 8] [--seq 32768] [--dim 128] [--reps 1]
        one forward + backward of one relation on cuda:0 (a small case for ncu
        captures; nothing is timed)
    python bench_cases.py strided [--seq 32768] [--iters 5]
        what strided inputs save on one LLaMA3-8B layer (contiguous copies, as
        the reference hook makes them, against the strided operator)
    python bench_cases.py grouped [--seq 4096] [--layers 32] [--iters 5]
        grouped calls against per-item calls over (relation x layer)
    python bench_cases.py ncu-launches launches.csv
        per kernel: launches, total gpu__time_duration, share of the total
    python bench_cases.py ncu-raw report.csv
        selected raw metrics (``ncu -i x.ncu-rep --page raw --csv``) per kernel

The timed cases print one JSON line; the ncu summaries print tables.
"""
from __future__ import annotations

import argparse
import collections
import csv
import io
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


# ------------------------------------------------------------------ profile
def profile(argv):
    import torch

    from linearard_b200.attention_KL import attn_kl_forward, kl_backward
    from linearard_b200.synth import relation_pair
    ap = argparse.ArgumentParser(prog="bench_cases.py profile")
    ap.add_argument("--heads", type=int, default=8)
    ap.add_argument("--seq", type=int, default=32768)
    ap.add_argument("--dim", type=int, default=128)
    ap.add_argument("--reps", type=int, default=1)
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "fp16"])
    ap.add_argument("--no-causal", action="store_true")
    a = ap.parse_args(argv)
    dt = torch.bfloat16 if a.dtype == "bf16" else torch.float16
    s, t = relation_pair((1, a.heads, a.seq, a.dim), seed_teacher=0, seed_student=1, theta=5e5,
                         apply_rope=True, dtype=dt, device="cuda")
    causal = not a.no_causal
    for _ in range(a.reps):
        loss, ls, lt = attn_kl_forward(s, s, t, t, None, causal)
        dS, _ = kl_backward(s, s, ls, t, t, lt, None, causal, fused=True)
    torch.cuda.synchronize()
    print(f"loss {float(loss):.6f}  |dS|max {float(dS.abs().max()):.4e}")


def _timed(arms, warmup, iters):
    import torch
    out = {}
    for name, fn in arms:
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            loss = fn()
        e1.record()
        torch.cuda.synchronize()
        out[name] = e0.elapsed_time(e1) / iters
        out[name.replace("_ms", "_loss")] = float(loss.detach())
    return out


# ------------------------------------------------------------------ strided
def strided(argv):
    """Both arms run the Q/Q (32 heads), K/K (8) and V/V (8) relations of one
    layer forward and backward; the reference hook copies each transposed
    projection with .contiguous() (train.py:133-142) before the operator."""
    import torch

    from linearard_b200.attention_KL import attn_kl_align, attn_kl_align_strided
    ap = argparse.ArgumentParser(prog="bench_cases.py strided")
    ap.add_argument("--seq", type=int, default=32768)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    T, D, H, Hkv = a.seq, 128, 32, 8
    g = torch.Generator(device="cuda").manual_seed(0)

    def proj(h):   # [B, T, h, D] projection output and its [B, h, T, D] view
        x = torch.randn(1, T, h, D, device="cuda", generator=g, dtype=torch.bfloat16)
        return x.transpose(1, 2)

    student = {"q": proj(H), "k": proj(Hkv), "v": proj(Hkv)}
    teacher = {r: (v + 0.1 * torch.randn(v.shape, device="cuda", generator=g,
                                         dtype=torch.bfloat16)).transpose(1, 2).contiguous()
               .transpose(1, 2) for r, v in student.items()}

    def copies_arm():
        total = None
        for r in student:
            s = student[r].contiguous().detach().requires_grad_(True)   # the hook's copies
            t = teacher[r].contiguous()
            l = attn_kl_align(s, s, t, t)
            total = l if total is None else total + l
        total.backward()
        return total

    def strided_arm():
        total = None
        for r in student:
            s = student[r].detach().requires_grad_(True)
            l = attn_kl_align_strided(s, s, teacher[r], teacher[r])
            total = l if total is None else total + l
        total.backward()
        return total

    out = {"workload": f"llama3_8b one layer, Q/Q x32 + K/K x8 + V/V x8, n={T}, d={D}, bf16"}
    out.update(_timed((("contiguous_copies_ms", copies_arm), ("strided_ms", strided_arm)),
                      a.warmup, a.iters))
    n_in = sum(v.numel() * v.element_size() for v in list(student.values()) +
               list(teacher.values()))
    out["copy_bytes_avoided"] = 2 * n_in   # each copy reads and writes its tensor
    print(json.dumps(out))


# ------------------------------------------------------------------ grouped
def grouped(argv):
    """The training loop issues the Q/Q, K/K and V/V relation losses of every
    layer (train.py:369-402): per-item attn_kl_align calls against one
    attn_kl_align_grouped call, LLaMA3-8B heads, symmetric calls."""
    import torch

    from linearard_b200.attention_KL import attn_kl_align, attn_kl_align_grouped
    ap = argparse.ArgumentParser(prog="bench_cases.py grouped")
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    T, D = a.seq, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    items = []
    for _ in range(a.layers):
        for H in (32, 8, 8):
            s = torch.randn(1, H, T, D, device="cuda", generator=g, dtype=torch.bfloat16)
            t = (s.float() + 0.1 * torch.randn(s.shape, device="cuda", generator=g)).bfloat16()
            items.append((s, t))

    def per_item():
        total = None
        for s, t in items:
            leaf = s.detach().requires_grad_(True)
            l = attn_kl_align(leaf, leaf, t, t)
            total = l if total is None else total + l
        total.backward()
        return total

    def grouped_arm():
        leaves = [(s.detach().requires_grad_(True), t) for s, t in items]
        total = attn_kl_align_grouped([(l, l, t, t) for l, t in leaves]).sum()
        total.backward()
        return total

    out = {"workload": f"llama3_8b heads, {a.layers} layers x (Q/Q 32 + K/K 8 + V/V 8), "
                       f"n={T}, d={D}, bf16, causal", "items": len(items)}
    out.update(_timed((("per_item_ms", per_item), ("grouped_ms", grouped_arm)), a.warmup,
                      a.iters))
    out["tokens_per_s_per_item_arm"] = T / (out["per_item_ms"] / 1e3)
    out["tokens_per_s_grouped_arm"] = T / (out["grouped_ms"] / 1e3)
    print(json.dumps(out))


# ------------------------------------------------------------------ ncu summaries
SHORT = (("sm100_dq_kernel", "sm100_dq_kernel"),
         ("sm100_dk_kernel", "sm100_dk_kernel"),
         ("sm100_forward_kernel", "sm100_forward_kernel"),
         ("scale_lse_kernel", "scale_lse_kernel"),
         ("generic_dq_kernel", "generic_dq_kernel"),
         ("generic_dk_kernel", "generic_dk_kernel"),
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


CASES = {"profile": profile, "strided": strided, "grouped": grouped,
         "ncu-launches": lambda argv: launches(argv[0]), "ncu-raw": lambda argv: raw(argv[0])}

if __name__ == "__main__":
    if len(sys.argv) < 2 or sys.argv[1] not in CASES:
        sys.exit(__doc__)
    CASES[sys.argv[1]](sys.argv[2:])
