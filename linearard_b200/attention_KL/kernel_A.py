"""Row log-sum-exp operator (drop-in for LinearARD ``kernel_A.lse_stats_triton``,
``kernels/attention_KL/kernel_A.py:190-265``).

``lse[b,h,i] = log sum_{j valid} exp(sm_scale * q[b,h,i] . k[b,h//G,j])``;
rows removed by the padding mask get 0, rows with no valid column ``-inf``.
Computed by ``lkl_lse`` in ``liblinearard_b200.so``.
"""
from __future__ import annotations

import ctypes

import torch

from .. import _lib
from ._common import (SUPPORTED_HEAD_DIMS, check_pair, prepare_mask, problem, ptr, stream_of,
                      workspace)

__all__ = ["lse_stats", "lse_stats_triton", "SUPPORTED_HEAD_DIMS"]


def lse_stats(q, k, attn_mask=None, causal=True, sm_scale=None):
    """q: [B,Hq,T,D], k: [B,Hkv,T,D] fp16/bf16 CUDA -> lse [B,Hq,T] fp32."""
    check_pair(q, k)
    B, Hq, T, D = q.shape
    mask, mdt = prepare_mask(attn_mask, B, T, q.device)
    prob = problem(q, k, causal=causal, mask_dtype=mdt, sm_scale_s=sm_scale, sm_scale_t=sm_scale)
    lse = torch.empty((B, Hq, T), device=q.device, dtype=torch.float32)
    with torch.cuda.device(q.device):
        ws, n = workspace(prob, mask is not None, q.device)
        st = _lib.lib().lkl_lse(ptr(q), ptr(k), ptr(mask), ctypes.byref(prob), ptr(lse),
                                ptr(ws), n, stream_of(q.device))
    _lib.check(st, "lkl_lse")
    return lse


# name used by LinearARD's integration module, kept for drop-in imports
lse_stats_triton = lse_stats
