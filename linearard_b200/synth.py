"""Seeded synthetic relation tensors for the benchmark and parity configs.

LinearARD captures post-RoPE q/k/v from a frozen native-RoPE teacher and a
RoPE-scaled student (``train.py:116-143``).  There are no checkpoints or
datasets here, so the tensors are drawn instead:

* teacher ``X ~ N(0,1)`` (optionally times a per-channel scale ``U[0.5, 2]``),
* student ``X + 0.1 * N(0,1)``,
* HF-style rotate-half RoPE on the Q and K relations (not V), teacher at
  positions ``0..n-1`` and student at ``positions / factor`` (linear
  interpolation, as ``rope_scaling={"type": "linear"}`` does in ``train.py``).

Everything is generated with explicit ``torch.Generator`` objects so that a
(config, seed) pair always produces the same tensors on a given device type.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

__all__ = ["RelationConfig", "CONFIGS", "rope", "relation_pair", "make_relations"]


@dataclass(frozen=True)
class RelationConfig:
    """One of the workloads the benchmark and the parity tests run."""

    name: str
    batch: int
    q_heads: int
    kv_heads: int
    head_dim: int
    seq_len: int
    theta: float
    rope_factor: float = 8.0
    channel_scale: bool = False
    relations: tuple = ("q", "k", "v")
    dtype: torch.dtype = torch.bfloat16
    causal: bool = True

    def heads(self, rel: str) -> int:
        return self.q_heads if rel == "q" else self.kv_heads

    @property
    def rel_heads(self) -> int:
        """(relation, head) units per sequence."""
        return sum(self.heads(r) for r in self.relations)

    def algorithmic_flops(self) -> float:
        """Algorithmic FLOPs of one forward+backward over every rel-head.

        Six n x n x d contractions per rel-head (forward: ss, st; backward:
        ss, st recomputed, dq and dk) at 2*n^2*d FLOPs each; the causal
        triangle halves that to 6*n^2*d."""
        n, d = self.seq_len, self.head_dim
        per = 6.0 * n * n * d if self.causal else 12.0 * n * n * d
        return per * self.rel_heads * self.batch


CONFIGS = {
    # the CPU reference check: fp32, one Q/Q head
    "cfg1_cpu_check": RelationConfig("cfg1_cpu_check", 1, 1, 1, 64, 512, 1.0e4,
                                     relations=("q",), dtype=torch.float32),
    # LLaMA2-7B head shape
    "llama2_7b_8k": RelationConfig("llama2_7b_8k", 1, 32, 32, 128, 8192, 1.0e4,
                                   channel_scale=True),
    # LLaMA3-8B GQA head shape at 32K (the headline workload)
    "llama3_8b_32k": RelationConfig("llama3_8b_32k", 1, 32, 8, 128, 32768, 5.0e5),
    # Mistral-7B head shape, one sequence per GPU
    "mistral_7b_32k": RelationConfig("mistral_7b_32k", 1, 32, 8, 128, 32768, 1.0e4),
}


def rope(x: torch.Tensor, positions: torch.Tensor, theta: float) -> torch.Tensor:
    """Rotate-half rotary embedding on the last dim of ``x`` ``[..., T, D]``.

    ``inv_freq_i = theta^(-2i/D)``, angle = position * inv_freq, and the
    output is ``x*cos + rotate_half(x)*sin`` with ``rotate_half(x) =
    cat(-x2, x1)`` -- the HF LLaMA convention.  Computed in fp32.
    """
    D = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, device=x.device, dtype=torch.float64) / D))
    ang = positions.to(torch.float64)[:, None] * inv[None, :]
    emb = torch.cat([ang, ang], dim=-1)
    cos = emb.cos().to(torch.float32)
    sin = emb.sin().to(torch.float32)
    xf = x.to(torch.float32)
    x1, x2 = xf[..., : D // 2], xf[..., D // 2:]
    rot = torch.cat([-x2, x1], dim=-1)
    return xf * cos + rot * sin


def relation_pair(shape, *, seed_teacher: int, seed_student: int, theta: float,
                  apply_rope: bool, rope_factor: float = 8.0, channel_scale: bool = False,
                  dtype=torch.bfloat16, device="cpu", scale_seed: int | None = None):
    """(student, teacher) tensors of ``shape`` = [B, H, T, D].

    teacher = N(0,1) [* per-channel U[0.5,2]] then RoPE at positions 0..T-1;
    student = the same pre-RoPE X + 0.1*N(0,1) then RoPE at positions/factor.
    """
    B, H, T, D = shape
    dev = torch.device(device)
    g_t = torch.Generator(device=dev).manual_seed(seed_teacher)
    g_s = torch.Generator(device=dev).manual_seed(seed_student)
    x = torch.randn(shape, generator=g_t, device=dev, dtype=torch.float32)
    if channel_scale:
        g_c = torch.Generator(device=dev).manual_seed(
            scale_seed if scale_seed is not None else seed_teacher + 7919)
        sc = torch.rand((1, H, 1, D), generator=g_c, device=dev) * 1.5 + 0.5
        x = x * sc
    xs = x + 0.1 * torch.randn(shape, generator=g_s, device=dev, dtype=torch.float32)
    if apply_rope:
        pos = torch.arange(T, device=dev, dtype=torch.float64)
        teacher = rope(x, pos, theta)
        student = rope(xs, pos / rope_factor, theta)
    else:
        teacher, student = x, xs
    return student.to(dtype).contiguous(), teacher.to(dtype).contiguous()


def make_relations(cfg: RelationConfig, *, device="cpu", seed: int = 0, batch: int | None = None):
    """Dict rel -> (student, teacher) tensors for every relation of ``cfg``.

    Seeds: relation r of sequence batch uses teacher seed ``seed + 2*idx`` and
    student seed ``seed + 2*idx + 1`` (config 1: seeds 0 and 1, as named).
    """
    B = cfg.batch if batch is None else batch
    out = {}
    for idx, rel in enumerate(cfg.relations):
        shape = (B, cfg.heads(rel), cfg.seq_len, cfg.head_dim)
        out[rel] = relation_pair(
            shape, seed_teacher=seed + 2 * idx, seed_student=seed + 2 * idx + 1,
            theta=cfg.theta, apply_rope=(rel in ("q", "k")), rope_factor=cfg.rope_factor,
            channel_scale=cfg.channel_scale, dtype=cfg.dtype, device=device)
    return out


def padding_mask(B: int, T: int, ratio: float, *, seed: int, dtype=torch.int32, device="cpu"):
    """``(rand > ratio)`` with token 0 always valid -- the reference tests'
    mask recipe (``test_kernel_C.py:318-322``)."""
    g = torch.Generator(device=torch.device(device)).manual_seed(seed)
    m = (torch.rand((B, T), generator=g, device=device) > ratio).to(dtype)
    m[:, 0] = 1
    return m
