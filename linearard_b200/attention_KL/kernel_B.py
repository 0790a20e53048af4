"""KL forward operator given row LSEs (drop-in for LinearARD
``kernel_B.kl_forward_triton``, ``kernels/attention_KL/kernel_B.py:249-391``).

Returns the 0-d fp32 sum over valid rows of ``sum_j pt*(log pt - log ps)``,
reduced in a fixed order (the reference accumulates with float atomics,
``kernel_B.py:216-218``).  Computed by ``lkl_kl_forward``.
"""
from __future__ import annotations

import ctypes

import torch

from .. import _lib
from ._common import (SUPPORTED_HEAD_DIMS, check_lse, check_pair, prepare_mask, problem, ptr,
                      stream_of, workspace)

__all__ = ["kl_forward", "kl_forward_triton", "SUPPORTED_HEAD_DIMS"]


def kl_forward(qs, ks, lse_s, qt, kt, lse_t, attn_mask=None, causal=True,
               sm_scale_s=None, sm_scale_t=None):
    check_pair(qs, ks, "qs", "ks")
    check_pair(qt, kt, "qt", "kt")
    B, Hq, T, _ = qs.shape
    assert tuple(qt.shape[:3]) == (B, Hq, T), "student/teacher B/Hq/T must align"
    check_lse(lse_s, (B, Hq, T), "lse_s")
    check_lse(lse_t, (B, Hq, T), "lse_t")
    mask, mdt = prepare_mask(attn_mask, B, T, qs.device)
    prob = problem(qs, ks, qt, kt, causal, mdt, sm_scale_s, sm_scale_t)
    loss = torch.empty((), device=qs.device, dtype=torch.float32)
    with torch.cuda.device(qs.device):
        ws, n = workspace(prob, mask is not None, qs.device)
        st = _lib.lib().lkl_kl_forward(ptr(qs), ptr(ks), ptr(lse_s), ptr(qt), ptr(kt), ptr(lse_t),
                                       ptr(mask), ctypes.byref(prob), ptr(loss), ptr(ws), n,
                                       stream_of(qs.device))
    _lib.check(st, "lkl_kl_forward")
    return loss


kl_forward_triton = kl_forward
