"""``attn_kl_align_grouped``: many (relation, layer) losses of one sequence in
one call.

The training loop computes the Q/Q, K/K and V/V relation losses of every
selected layer for each micro-batch (``train.py:369-402``), i.e. 3·L calls
of ``attn_kl_align``.  This operator takes them all at once and returns the
per-item losses as one fp32 tensor ``[n]``; its forward is a single launch over
every item's row tiles (``lkl_forward_grouped``) and its backward one dq and
one dk launch per chunk of kv groups across items (``lkl_backward_grouped``).
Loss values, LSEs and gradients are those of the per-item calls.

Items share B, T, the head dims, dtypes, scales, causal flag and mask; each
has its own head counts.  Inputs may be [B, H, T, D] views with any strides
that are multiples of 8 elements (the transposed projections an attention
hook sees): they are read in place, as by ``attn_kl_align_strided``.  When an
item is outside the tensor-core path (16-byte-aligned inputs, Ds and Dt in
{8, 16, 32, 64, 128}) the call falls back to per-item
``attn_kl_align_strided`` calls.
"""
from __future__ import annotations

import ctypes

import torch

from .. import _lib
from ._common import prepare_mask, problem, ptr, stream_of
from .strided import attn_kl_align_strided, strided_ok

__all__ = ["attn_kl_align_grouped", "AttnKLAlignGroupedFn", "grouped_ok"]


def grouped_ok(items) -> bool:
    """True when every item runs on the tensor-core path."""
    return all(strided_ok(*it) for it in items)


def _table(items, lse, grads=None):
    arr = (_lib.LKLGroupItem * len(items))()
    for i, (qs, ks, qt, kt) in enumerate(items):
        e = arr[i]
        e.qs, e.ks, e.qt, e.kt = qs.data_ptr(), ks.data_ptr(), qt.data_ptr(), kt.data_ptr()
        e.Hq, e.Hkv_s, e.Hkv_t = qs.shape[1], ks.shape[1], kt.shape[1]
        e.strided = 0 if all(t.is_contiguous() for t in (qs, ks, qt, kt)) else 1
        if e.strided:
            for k, t in enumerate((qs, ks, qt, kt)):
                e.strides[k] = _lib.LKLStrides(b=t.stride(0), h=t.stride(1), t=t.stride(2))
        e.lse_s, e.lse_t = lse[i][0].data_ptr(), lse[i][1].data_ptr()
        if grads is not None:
            e.dq, e.dk = grads[i][0].data_ptr(), grads[i][1].data_ptr()
    return arr


def _workspace(n, table, prob, has_mask, backward, device):
    size = int(_lib.lib().lkl_grouped_workspace_size(n, table, ctypes.byref(prob),
                                                     1 if has_mask else 0,
                                                     1 if backward else 0))
    return torch.empty(max(size, 256), dtype=torch.uint8, device=device), size


class AttnKLAlignGroupedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, n, attn_mask, causal, sm_scale_s, sm_scale_t, *flat):
        items = [tuple(flat[4 * i:4 * i + 4]) for i in range(n)]
        qs0 = items[0][0]
        B, _, T, _ = qs0.shape
        mask, mdt = prepare_mask(attn_mask, B, T, qs0.device)
        prob = problem(qs0, items[0][1], items[0][2], items[0][3], causal, mdt, sm_scale_s,
                       sm_scale_t)
        lse = [(torch.empty((B, qs.shape[1], T), device=qs.device, dtype=torch.float32),
                torch.empty((B, qs.shape[1], T), device=qs.device, dtype=torch.float32))
               for qs, _, _, _ in items]
        losses = torch.empty(n, device=qs0.device, dtype=torch.float32)
        table = _table(items, lse)
        with torch.cuda.device(qs0.device):
            ws, size = _workspace(n, table, prob, mask is not None, False, qs0.device)
            st = _lib.lib().lkl_forward_grouped(n, table, ptr(mask), ctypes.byref(prob),
                                                ptr(losses), ptr(ws), size,
                                                stream_of(qs0.device))
        _lib.check(st, "lkl_forward_grouped")
        ctx.n, ctx.causal, ctx.mdt = n, causal, mdt
        ctx.sm_scale_s, ctx.sm_scale_t = sm_scale_s, sm_scale_t
        ctx.fused = [qs is ks for qs, ks, _, _ in items]
        ctx.has_mask = mask is not None
        saved = list(flat) + [t for pair in lse for t in pair]
        saved.append(mask if mask is not None else torch.empty(0, device=qs0.device))
        ctx.save_for_backward(*saved)
        return losses

    @staticmethod
    def backward(ctx, dlosses):
        n = ctx.n
        saved = ctx.saved_tensors
        items = [tuple(saved[4 * i:4 * i + 4]) for i in range(n)]
        lse = [(saved[4 * n + 2 * i], saved[4 * n + 2 * i + 1]) for i in range(n)]
        mask = saved[6 * n] if ctx.has_mask else None
        qs0 = items[0][0]
        prob = problem(qs0, items[0][1], items[0][2], items[0][3], ctx.causal, ctx.mdt,
                       ctx.sm_scale_s, ctx.sm_scale_t)
        grads = []
        for (qs, ks, _, _), fused in zip(items, ctx.fused):
            dq = torch.empty(qs.shape, device=qs.device, dtype=torch.float32)
            dk = dq if fused else torch.empty(ks.shape, device=qs.device, dtype=torch.float32)
            grads.append((dq, dk))
        dl = dlosses.detach().to(torch.float32).contiguous()
        table = _table(items, lse, grads)
        with torch.cuda.device(qs0.device):
            ws, size = _workspace(n, table, prob, mask is not None, True, qs0.device)
            st = _lib.lib().lkl_backward_grouped(n, table, ptr(mask), ctypes.byref(prob),
                                                 ptr(dl), ptr(ws), size, stream_of(qs0.device))
        _lib.check(st, "lkl_backward_grouped")
        out = []
        for (dq, dk), fused in zip(grads, ctx.fused):
            out += [dq, None if fused else dk, None, None]
        return (None, None, None, None, None, *out)


def attn_kl_align_grouped(items, attn_mask=None, causal=True, sm_scale_s=None,
                          sm_scale_t=None):
    """items: sequence of (qs, ks, qt, kt) for one sequence (same B and T).
    Returns fp32 ``[n]``: entry i is ``attn_kl_align(*items[i], ...)``."""
    items = [tuple(it) for it in items]
    assert len(items) > 0, "items must not be empty"
    B, T = items[0][0].shape[0], items[0][0].shape[2]
    for qs, ks, qt, kt in items:
        for name, t in (("qs", qs), ("ks", ks), ("qt", qt), ("kt", kt)):
            assert isinstance(t, torch.Tensor), f"{name} must be a torch.Tensor"
            assert t.is_cuda, "Q/K must be on CUDA"
            assert t.ndim == 4, f"{name} shape must be [B,H,T,D]"
            assert t.stride(-1) == 1, f"{name} last-dim stride must be 1"
        assert qs.dtype in (torch.float16, torch.bfloat16), "qs dtype supports only fp16/bf16"
        assert qt.dtype in (torch.float16, torch.bfloat16), "qt dtype supports only fp16/bf16"
        assert qs.dtype == ks.dtype and qt.dtype == kt.dtype, "q/k dtypes must match"
        assert tuple(qt.shape[:3]) == tuple(qs.shape[:3]), "student/teacher B/Hq/T must align"
        assert (ks.shape[0], ks.shape[2], ks.shape[3]) == (qs.shape[0], qs.shape[2],
                                                            qs.shape[3]), "qs/ks B/T/D must match"
        assert qs.shape[1] % ks.shape[1] == 0 and qs.shape[1] % kt.shape[1] == 0, \
            "Hq must be divisible by Hkv"
        assert (qs.shape[0], qs.shape[2]) == (B, T), "grouped items must share B and T"
        assert qs.shape[3] == items[0][0].shape[3] and qt.shape[3] == items[0][2].shape[3], \
            "grouped items must share the head dims"
        assert qs.dtype == items[0][0].dtype and qt.dtype == items[0][2].dtype, \
            "grouped items must share dtypes"
    if not grouped_ok(items):
        return torch.stack([attn_kl_align_strided(*it, attn_mask, causal, sm_scale_s,
                                                  sm_scale_t) for it in items])
    flat = [t for it in items for t in it]
    return AttnKLAlignGroupedFn.apply(len(items), attn_mask, causal, sm_scale_s, sm_scale_t,
                                      *flat)
