"""Measure what strided inputs save: one LLaMA3-8B layer at 32K context.

An attention hook sees q, k, v as transposed projections ([B, T, H, D]
memory).  The reference path copies them with ``.contiguous()`` and then
calls the operator (``train.py:133-142``, ``:380-402``); the strided path
calls ``attn_kl_align_strided`` on the views.  Both run the Q/Q (32 heads),
K/K (8) and V/V (8) relations forward and backward; CUDA events time each
arm after warm-up.

    python -m linearard_b200.strided_case [--seq 32768] [--iters 5]

Prints one JSON line.
"""
from __future__ import annotations

import argparse
import json

import torch

from .attention_KL import attn_kl_align, attn_kl_align_strided


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=32768)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    T, D, H, Hkv = a.seq, 128, 32, 8
    g = torch.Generator(device="cuda").manual_seed(0)

    def proj(h):   # [B, T, h, D] projection output and its [B, h, T, D] view
        x = torch.randn(1, T, h, D, device="cuda", generator=g, dtype=torch.bfloat16)
        return x.transpose(1, 2)

    student = {"q": proj(H), "k": proj(Hkv), "v": proj(Hkv)}
    teacher = {r: v + 0.1 * torch.randn(v.shape, device="cuda", generator=g,
                                        dtype=torch.bfloat16).transpose(1, 2).transpose(1, 2)
               for r, v in student.items()}
    teacher = {r: v.transpose(1, 2).contiguous().transpose(1, 2) for r, v in teacher.items()}

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
    for name, fn in (("contiguous_copies_ms", copies_arm), ("strided_ms", strided_arm)):
        for _ in range(a.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.iters):
            loss = fn()
        e1.record()
        torch.cuda.synchronize()
        out[name] = e0.elapsed_time(e1) / a.iters
        out[name.replace("_ms", "_loss")] = float(loss)
    n_in = sum(v.numel() * v.element_size() for v in list(student.values()) +
               list(teacher.values()))
    out["copy_bytes_avoided"] = 2 * n_in   # each copy reads and writes its tensor
    print(json.dumps(out))


if __name__ == "__main__":
    main()
