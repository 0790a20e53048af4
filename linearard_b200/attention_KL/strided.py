"""``attn_kl_align_strided``: the operator on [B, H, T, D] views, no copies.

LinearARD's attention hook makes every captured q/k/v contiguous before the
loss sees it (``train.py:133-142``), because the reference wrappers require
contiguous inputs (``kernel_B.py:289-290``, ``kernel_C.py:334-335``).  In a
HF attention layer those tensors are transposed views of the projections
([B, T, H, D] memory, [B, H, T, D] shape), so each ``.contiguous()`` is a
full copy of q, k and v per layer.  This operator takes the views as they
are: the tensor-core kernels read them in place through 4-D TMA maps
(``lkl_forward_strided`` / ``lkl_backward_strided``).

Same value, gradients and call signature as ``attn_kl_align``.  Inputs need a
last-dim stride of 1, the other strides multiples of 8 elements and 16-byte
aligned storage; shapes the tensor-core path does not cover (Ds or Dt not in
{8, 16, 32, 64, 128}, other strides) go through ``attn_kl_align`` on contiguous copies,
i.e. the same GPU kernels the reference-shaped call uses.
"""
from __future__ import annotations

import ctypes

import torch

from .. import _lib
from ._common import TC_HEAD_DIMS, prepare_mask, problem, ptr, stream_of, workspace
from .integration import attn_kl_align

__all__ = ["attn_kl_align_strided", "AttnKLAlignStridedFn", "strided_ok"]


def _strides(t: torch.Tensor) -> _lib.LKLStrides:
    return _lib.LKLStrides(b=t.stride(0), h=t.stride(1), t=t.stride(2))


def strided_ok(qs, ks, qt, kt) -> bool:
    """True when the tensor-core path reads these views in place."""
    for t in (qs, ks, qt, kt):
        if not (t.is_cuda and t.ndim == 4 and t.stride(-1) == 1 and t.data_ptr() % 16 == 0
                and all(s > 0 and s % 8 == 0 for s in t.stride()[:3])):
            return False
    if qs.dtype != ks.dtype or qt.dtype != kt.dtype:
        return False
    if qs.dtype not in (torch.float16, torch.bfloat16) or qt.dtype not in (torch.float16,
                                                                            torch.bfloat16):
        return False
    return (qs.shape[3] in TC_HEAD_DIMS and qt.shape[3] in TC_HEAD_DIMS
            and qs.shape[1] % ks.shape[1] == 0 and qs.shape[1] % kt.shape[1] == 0)


def _array(*ts):
    return (_lib.LKLStrides * 4)(*[_strides(t) for t in ts])


class AttnKLAlignStridedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qs, ks, qt, kt, attn_mask, causal: bool, sm_scale_s, sm_scale_t):
        B, Hq, T, Ds = qs.shape
        assert tuple(qt.shape[:3]) == (B, Hq, T), "student/teacher B/Hq/T must align"
        assert (ks.shape[0], ks.shape[2], ks.shape[3]) == (B, T, Ds), "qs/ks B/T/D must match"
        assert (kt.shape[0], kt.shape[2], kt.shape[3]) == (B, T, qt.shape[3]), \
            "qt/kt B/T/D must match"
        assert Hq % ks.shape[1] == 0 and Hq % kt.shape[1] == 0, "Hq must be divisible by Hkv"
        mask, mdt = prepare_mask(attn_mask, B, T, qs.device)
        prob = problem(qs, ks, qt, kt, causal, mdt, sm_scale_s, sm_scale_t)
        strides = _array(qs, ks, qt, kt)
        lse_s = torch.empty((B, Hq, T), device=qs.device, dtype=torch.float32)
        lse_t = torch.empty((B, Hq, T), device=qs.device, dtype=torch.float32)
        loss = torch.empty((), device=qs.device, dtype=torch.float32)
        with torch.cuda.device(qs.device):
            ws, n = workspace(prob, mask is not None, qs.device)
            st = _lib.lib().lkl_forward_strided(ptr(qs), ptr(ks), ptr(qt), ptr(kt), strides,
                                                ptr(mask), ctypes.byref(prob), ptr(lse_s),
                                                ptr(lse_t), ptr(loss), ptr(ws), n,
                                                stream_of(qs.device))
        _lib.check(st, "lkl_forward_strided")
        ctx.shared_student = qs is ks
        ctx.has_mask = mask is not None
        ctx.save_for_backward(qs, ks, lse_s, qt, kt, lse_t,
                              mask if mask is not None else torch.empty(0, device=qs.device))
        ctx.mdt, ctx.causal = mdt, causal
        ctx.sm_scale_s, ctx.sm_scale_t = sm_scale_s, sm_scale_t
        return loss

    @staticmethod
    def backward(ctx, dloss):
        qs, ks, lse_s, qt, kt, lse_t, mask = ctx.saved_tensors
        mask = mask if ctx.has_mask else None
        B, Hq, T, Ds = qs.shape
        prob = problem(qs, ks, qt, kt, ctx.causal, ctx.mdt, ctx.sm_scale_s, ctx.sm_scale_t)
        dloss = dloss.detach().to(torch.float32).reshape(1).contiguous()
        fused = ctx.shared_student
        dq = torch.empty((B, Hq, T, Ds), device=qs.device, dtype=torch.float32)
        dk = dq if fused else torch.empty((B, ks.shape[1], T, Ds), device=qs.device,
                                          dtype=torch.float32)
        with torch.cuda.device(qs.device):
            ws, n = workspace(prob, mask is not None, qs.device, backward=True)
            st = _lib.lib().lkl_backward_strided(ptr(qs), ptr(ks), ptr(lse_s), ptr(qt), ptr(kt),
                                                 ptr(lse_t), _array(qs, ks, qt, kt), ptr(mask),
                                                 ctypes.byref(prob), ptr(dloss), ptr(dq),
                                                 ptr(dk), ptr(ws), n, stream_of(qs.device))
        _lib.check(st, "lkl_backward_strided")
        return dq, (None if fused else dk), None, None, None, None, None, None


def attn_kl_align_strided(qs, ks, qt, kt, attn_mask=None, causal=True, sm_scale_s=None,
                          sm_scale_t=None):
    """``attn_kl_align`` on [B, H, T, D] tensors of any layout with a unit last
    stride; returns the 0-d fp32 sum of row KLs."""
    for name, t in (("qs", qs), ("ks", ks), ("qt", qt), ("kt", kt)):
        assert isinstance(t, torch.Tensor), f"{name} must be a torch.Tensor"
        assert t.is_cuda, "Q/K must be on CUDA"
        assert t.ndim == 4, f"{name} shape must be [B,H,T,D]"
        assert t.stride(-1) == 1, f"{name} last-dim stride must be 1"
    if strided_ok(qs, ks, qt, kt):
        return AttnKLAlignStridedFn.apply(qs, ks, qt, kt, attn_mask, causal, sm_scale_s,
                                          sm_scale_t)
    # the shapes the tensor-core path does not cover: the contiguous operator
    cs = qs.contiguous()
    ck = cs if ks is qs else ks.contiguous()
    ct = qt.contiguous()
    ckt = ct if kt is qt else kt.contiguous()
    return attn_kl_align(cs, ck, ct, ckt, attn_mask, causal, sm_scale_s, sm_scale_t)
