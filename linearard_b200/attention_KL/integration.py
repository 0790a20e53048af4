"""Autograd operator (drop-in for LinearARD ``kernels/attention_KL/integration.py``).

``attn_kl_align(qs, ks, qt, kt, attn_mask=None, causal=True, sm_scale_s=None,
sm_scale_t=None)`` returns the 0-d fp32 **sum** over rows of
``KL(softmax(qt kt^T sc_t) || softmax(qs ks^T sc_s))`` -- the same value and
call signature as the reference (``integration.py:70-73``).

Differences in mechanism, not in results:

* forward is one fused pass (``lkl_forward``) that produces both row LSEs and
  the loss, instead of the reference's three launches (kernel A twice, then
  kernel B, ``integration.py:18-27``);
* backward multiplies by ``dloss`` on the device, and when ``qs is ks`` (the
  call pattern of ``train.py:380-402``) it returns one fused ``dq + dk``
  gradient for the shared tensor instead of two fp32 tensors that autograd
  would add.
"""
from __future__ import annotations

import ctypes

import torch

from .. import _lib
from ._common import check_pair, prepare_mask, problem, ptr, stream_of, workspace
from .kernel_C import kl_backward

__all__ = ["AttnKLAlignFn", "attn_kl_align", "attn_kl_forward"]


def attn_kl_forward(qs, ks, qt, kt, attn_mask=None, causal=True, sm_scale_s=None,
                    sm_scale_t=None):
    """Fused forward: (loss_sum 0-d fp32, lse_s [B,Hq,T], lse_t [B,Hq,T])."""
    check_pair(qs, ks, "qs", "ks")
    check_pair(qt, kt, "qt", "kt")
    B, Hq, T, _ = qs.shape
    assert tuple(qt.shape[:3]) == (B, Hq, T), "student/teacher B/Hq/T must align"
    assert qs.device == qt.device, "student/teacher must be on the same device"
    mask, mdt = prepare_mask(attn_mask, B, T, qs.device)
    prob = problem(qs, ks, qt, kt, causal, mdt, sm_scale_s, sm_scale_t)
    lse_s = torch.empty((B, Hq, T), device=qs.device, dtype=torch.float32)
    lse_t = torch.empty((B, Hq, T), device=qs.device, dtype=torch.float32)
    loss = torch.empty((), device=qs.device, dtype=torch.float32)
    with torch.cuda.device(qs.device):
        ws, n = workspace(prob, mask is not None, qs.device)
        st = _lib.lib().lkl_forward(ptr(qs), ptr(ks), ptr(qt), ptr(kt), ptr(mask),
                                    ctypes.byref(prob), ptr(lse_s), ptr(lse_t), ptr(loss),
                                    ptr(ws), n, stream_of(qs.device))
    _lib.check(st, "lkl_forward")
    return loss, lse_s, lse_t


class AttnKLAlignFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qs, ks, qt, kt, attn_mask, causal: bool, sm_scale_s, sm_scale_t):
        """qs, ks, qt, kt: [B, H, T, D]; attn_mask: [B, T] (1 = valid) or None.
        Returns the scalar loss (sum over rows)."""
        kl, lse_s, lse_t = attn_kl_forward(qs, ks, qt, kt, attn_mask, causal, sm_scale_s,
                                           sm_scale_t)
        if attn_mask is None:
            mask_saved = torch.empty(0, device=qs.device)
            ctx.has_mask = False
        else:
            mask_saved = attn_mask
            ctx.has_mask = True
        ctx.shared_student = qs is ks
        ctx.save_for_backward(qs, ks, lse_s, qt, kt, lse_t, mask_saved)
        ctx.causal = causal
        ctx.sm_scale_s = sm_scale_s
        ctx.sm_scale_t = sm_scale_t
        return kl

    @staticmethod
    def backward(ctx, dloss):
        qs, ks, lse_s, qt, kt, lse_t, mask_or_empty = ctx.saved_tensors
        attn_mask = mask_or_empty if ctx.has_mask else None
        dloss = dloss.detach().to(torch.float32).reshape(1)
        dqs, dks = kl_backward(qs, ks, lse_s, qt, kt, lse_t, attn_mask=attn_mask,
                               causal=ctx.causal, sm_scale_s=ctx.sm_scale_s,
                               sm_scale_t=ctx.sm_scale_t, dloss=dloss,
                               fused=ctx.shared_student)
        # the teacher, mask, causal flag and scales get no gradient
        return dqs, dks, None, None, None, None, None, None


def attn_kl_align(qs, ks, qt, kt, attn_mask=None, causal=True, sm_scale_s=None, sm_scale_t=None):
    return AttnKLAlignFn.apply(qs, ks, qt, kt, attn_mask, causal, sm_scale_s, sm_scale_t)
