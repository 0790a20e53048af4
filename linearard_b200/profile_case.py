"""Run one forward + backward of a single relation on cuda:0 (a small case for
ncu captures; nothing is timed here).

    python -m linearard_b200.profile_case --heads 8 --seq 32768 --dim 128 [--kv-heads 8]

Inputs come from the benchmark generator (Gaussian + RoPE, student at
positions/8), the call is the symmetric ``attn_kl_align(s, s, t, t)`` pattern:
``lkl_forward`` then ``lkl_backward`` with the fused dq+dk output.
"""
from __future__ import annotations

import argparse

import torch

from .attention_KL import attn_kl_forward, kl_backward
from .synth import relation_pair


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--heads", type=int, default=8)
    ap.add_argument("--seq", type=int, default=32768)
    ap.add_argument("--dim", type=int, default=128)
    ap.add_argument("--reps", type=int, default=1)
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "fp16"])
    ap.add_argument("--no-causal", action="store_true")
    a = ap.parse_args()
    dt = torch.bfloat16 if a.dtype == "bf16" else torch.float16
    s, t = relation_pair((1, a.heads, a.seq, a.dim), seed_teacher=0, seed_student=1, theta=5e5,
                         apply_rope=True, dtype=dt, device="cuda")
    causal = not a.no_causal
    for _ in range(a.reps):
        loss, ls, lt = attn_kl_forward(s, s, t, t, None, causal)
        dS, _ = kl_backward(s, s, ls, t, t, lt, None, causal, fused=True)
    torch.cuda.synchronize()
    print(f"loss {float(loss):.6f}  |dS|max {float(dS.abs().max()):.4e}")


if __name__ == "__main__":
    main()
