"""KL backward operator (drop-in for LinearARD ``kernel_C.kl_backward_triton``,
``kernels/attention_KL/kernel_C.py:293-449``).

Returns fp32 ``dq [B,Hq,T,Ds]`` and ``dk [B,Hkv_s,T,Ds]`` of the KL sum with
respect to the student q and k (GQA heads summed into their kv head).
``dloss`` (optional 0-d fp32 CUDA tensor) multiplies both on the device, which
is the chain rule of ``AttnKLAlignFn.backward`` (``integration.py:62-64``).
``fused=True`` requires ``qs is ks`` and returns the single gradient
``dq + dk`` of the shared tensor (``train.py:380-402`` always passes the same
tensor twice).  Computed by ``lkl_backward``.
"""
from __future__ import annotations

import ctypes

import torch

from .. import _lib
from ._common import (SUPPORTED_HEAD_DIMS, check_lse, check_pair, prepare_mask, problem, ptr,
                      stream_of, workspace)

__all__ = ["kl_backward", "kl_backward_triton", "SUPPORTED_HEAD_DIMS"]


def kl_backward(qs, ks, lse_s, qt, kt, lse_t, attn_mask=None, causal=True,
                sm_scale_s=None, sm_scale_t=None, dloss=None, fused=False):
    check_pair(qs, ks, "qs", "ks")
    check_pair(qt, kt, "qt", "kt")
    B, Hq, T, Ds = qs.shape
    assert tuple(qt.shape[:3]) == (B, Hq, T), "student/teacher B/Hq/T must align"
    check_lse(lse_s, (B, Hq, T), "lse_s")
    check_lse(lse_t, (B, Hq, T), "lse_t")
    if fused:
        assert ks.data_ptr() == qs.data_ptr() and ks.shape == qs.shape, "fused needs qs is ks"
    mask, mdt = prepare_mask(attn_mask, B, T, qs.device)
    if dloss is not None:
        assert dloss.is_cuda and dloss.dtype == torch.float32 and dloss.numel() == 1, \
            "dloss must be a 1-element fp32 CUDA tensor"
        dloss = dloss.contiguous()
    prob = problem(qs, ks, qt, kt, causal, mdt, sm_scale_s, sm_scale_t)
    dq = torch.empty((B, Hq, T, Ds), device=qs.device, dtype=torch.float32)
    dk = dq if fused else torch.empty((B, ks.shape[1], T, Ds), device=qs.device,
                                      dtype=torch.float32)
    with torch.cuda.device(qs.device):
        ws, n = workspace(prob, mask is not None, qs.device, backward=True)
        st = _lib.lib().lkl_backward(ptr(qs), ptr(ks), ptr(lse_s), ptr(qt), ptr(kt), ptr(lse_t),
                                     ptr(mask), ctypes.byref(prob), ptr(dloss), ptr(dq), ptr(dk),
                                     ptr(ws), n, stream_of(qs.device))
    _lib.check(st, "lkl_backward")
    return (dq, None) if fused else (dq, dk)


kl_backward_triton = kl_backward
