"""Parity case grid shared by the golden-fixture generator and the tests.

The grid mirrors LinearARD's own kernel test sweeps:

* LSE cases: ``kernels/attention_KL/test_kernel_A.py:208-235`` (every head dim
  x GQA {8/8, 8/4} x {causal, non-causal + 30% padding}, extra GQA/mask
  ratios, bf16, and T=127).
* KL / gradient cases: ``test_kernel_B.py:245-268`` and
  ``test_kernel_C.py:291-315`` (all 36 (Ds, Dt) pairs at T=16, mixed GQA with
  padding 0.3/0.7, non-causal, bf16 at D=64, T=127), plus the dk aggregation
  stress case ``test_kernel_C.py:255-286`` (B2 Hq16 Hkv_s4 Hkv_t8 T33).

Inputs are regenerated deterministically from a per-case seed with a CPU
``torch.Generator`` (fp32 normal draws cast to the case dtype) and the fixture
stores a SHA-256 of the input bytes so that a drift in the generator is caught.
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass

import numpy as np
import torch

DIMS = (8, 16, 32, 64, 128, 256)


@dataclass(frozen=True)
class LseCase:
    name: str
    dtype: str
    causal: bool
    mask_ratio: float | None
    B: int
    Hq: int
    Hkv: int
    T: int
    D: int
    seed: int


@dataclass(frozen=True)
class KlCase:
    name: str
    dtype: str
    causal: bool
    mask_ratio: float | None
    B: int
    Hq: int
    Hkv_s: int
    Hkv_t: int
    T: int
    Ds: int
    Dt: int
    seed: int


def _dt(name: str) -> torch.dtype:
    return {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[name]


def lse_cases() -> list[LseCase]:
    out = []
    s = 1000
    for D in DIMS:
        for Hq, Hkv in ((8, 8), (8, 4)):
            out.append(LseCase(f"lse_D{D}_g{Hq // Hkv}_causal", "fp16", True, None, 2, Hq, Hkv, 33, D, s)); s += 1
            out.append(LseCase(f"lse_D{D}_g{Hq // Hkv}_pad", "fp16", False, 0.3, 2, Hq, Hkv, 33, D, s)); s += 1
    out.append(LseCase("lse_gqa4_mask07", "fp16", True, 0.7, 2, 8, 2, 33, 8, s)); s += 1
    out.append(LseCase("lse_gqa4_H16", "fp16", False, 0.3, 2, 16, 4, 33, 16, s)); s += 1
    out.append(LseCase("lse_bf16_D8", "bf16", True, None, 2, 8, 8, 33, 8, s)); s += 1
    out.append(LseCase("lse_bf16_D256_pad", "bf16", False, 0.3, 2, 8, 4, 33, 256, s)); s += 1
    out.append(LseCase("lse_T127_causal", "fp16", True, None, 1, 8, 4, 127, 64, s)); s += 1
    out.append(LseCase("lse_T127_pad", "fp16", False, 0.3, 1, 8, 2, 127, 64, s)); s += 1
    return out


def kl_cases() -> list[KlCase]:
    out = []
    s = 2000
    for Ds in DIMS:
        for Dt in DIMS:
            out.append(KlCase(f"kl_Ds{Ds}_Dt{Dt}", "fp16", True, None, 1, 8, 8, 8, 16, Ds, Dt, s)); s += 1
    out.append(KlCase("kl_nc_pad03_gqa", "fp16", False, 0.3, 2, 8, 4, 2, 33, 8, 128, s)); s += 1
    out.append(KlCase("kl_causal_pad07_gqa", "fp16", True, 0.7, 2, 8, 2, 4, 33, 128, 8, s)); s += 1
    out.append(KlCase("kl_nc_pad03_H16", "fp16", False, 0.3, 2, 16, 4, 4, 33, 16, 32, s)); s += 1
    out.append(KlCase("kl_bf16_D64", "bf16", True, None, 2, 8, 8, 8, 33, 64, 64, s)); s += 1
    out.append(KlCase("kl_T127_nc_pad", "fp16", False, 0.3, 1, 8, 4, 2, 127, 64, 128, s)); s += 1
    for seed in (0, 1, 2):
        out.append(KlCase(f"kl_dk_stress_s{seed}", "fp16", True, 0.3, 2, 16, 4, 8, 33, 32, 64, 3000 + seed))
    # tile-boundary cases for the tensor-core path (128-row tiles)
    out.append(KlCase("kl_bf16_D128_T300_pad", "bf16", True, 0.2, 1, 4, 2, 2, 300, 128, 128, 3100))
    out.append(KlCase("kl_bf16_D64_T257_gqa", "bf16", True, None, 1, 4, 1, 2, 257, 64, 64, 3101))
    return out


def _randn(shape, g, dtype):
    return torch.randn(shape, generator=g, dtype=torch.float32).to(dtype)


def make_lse_inputs(c: LseCase):
    g = torch.Generator().manual_seed(c.seed)
    dt = _dt(c.dtype)
    q = _randn((c.B, c.Hq, c.T, c.D), g, dt)
    k = _randn((c.B, c.Hkv, c.T, c.D), g, dt)
    mask = None
    if c.mask_ratio is not None:
        mask = (torch.rand((c.B, c.T), generator=g) > c.mask_ratio).to(torch.int32)
        mask[:, 0] = 1
    return q, k, mask


def make_kl_inputs(c: KlCase):
    g = torch.Generator().manual_seed(c.seed)
    dt = _dt(c.dtype)
    qs = _randn((c.B, c.Hq, c.T, c.Ds), g, dt)
    ks = _randn((c.B, c.Hkv_s, c.T, c.Ds), g, dt)
    qt = _randn((c.B, c.Hq, c.T, c.Dt), g, dt)
    kt = _randn((c.B, c.Hkv_t, c.T, c.Dt), g, dt)
    mask = None
    if c.mask_ratio is not None:
        mask = (torch.rand((c.B, c.T), generator=g) > c.mask_ratio).to(torch.int32)
        mask[:, 0] = 1
    return qs, ks, qt, kt, mask


def digest(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        if t is None:
            h.update(b"none")
            continue
        a = t.detach().cpu().contiguous()
        if a.dtype in (torch.bfloat16, torch.float16):
            a = a.view(torch.int16)
        h.update(a.numpy().tobytes())
    return h.hexdigest()


def to_np(t):
    """Float tensor -> float64 numpy (exact for fp16/bf16/fp32 inputs)."""
    return None if t is None else t.detach().cpu().to(torch.float64).numpy()


def sm_scale(d: int) -> float:
    return 1.0 / (d ** 0.5)


FIXTURE = "reference_golden.npz"
