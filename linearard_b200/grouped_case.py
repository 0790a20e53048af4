"""Measure grouped calls against per-item calls.

The training loop issues the Q/Q, K/K and V/V relation losses of every layer
(``train.py:369-402``).  Both arms compute them forward and backward for
LLaMA3-8B heads (Q 32, K 8, V 8, d = 128, bf16, causal, symmetric calls):
the per-item arm calls ``attn_kl_align`` once per (relation, layer), the
grouped arm calls ``attn_kl_align_grouped`` once.  CUDA events time each arm
after warm-up.

    python -m linearard_b200.grouped_case [--seq 4096] [--layers 32] [--iters 5]

Prints one JSON line.
"""
from __future__ import annotations

import argparse
import json

import torch

from .attention_KL import attn_kl_align, attn_kl_align_grouped


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
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

    def grouped():
        leaves = [(s.detach().requires_grad_(True), t) for s, t in items]
        losses = attn_kl_align_grouped([(l, l, t, t) for l, t in leaves])
        total = losses.sum()
        total.backward()
        return total

    out = {"workload": f"llama3_8b heads, {a.layers} layers x (Q/Q 32 + K/K 8 + V/V 8), "
                       f"n={T}, d={D}, bf16, causal", "items": len(items)}
    for name, fn in (("per_item_ms", per_item), ("grouped_ms", grouped)):
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
    out["tokens_per_s_per_item_arm"] = T / (out["per_item_ms"] / 1e3)
    out["tokens_per_s_grouped_arm"] = T / (out["grouped_ms"] / 1e3)
    print(json.dumps(out))


if __name__ == "__main__":
    main()
