"""Grouped calls (``attn_kl_align_grouped``, ``lkl_forward_grouped`` /
``lkl_backward_grouped``) on a B200.

Several (relation, layer) items of one sequence go through one forward launch
and one dq + one dk launch per chunk of kv groups.  The per-CTA work and the
summation orders are those of the per-item calls, so losses, LSEs and
gradients must be bitwise equal to ``attn_kl_align`` item by item -- also when
a small D buffer splits the backward into chunks that cross items.
"""
import ctypes

import pytest
import torch

from gpu_util import check_device_status, path_is_tensor_core
from linearard_b200 import _lib
from linearard_b200.attention_KL import attn_kl_align, attn_kl_align_grouped
from linearard_b200.attention_KL._common import problem

pytestmark = pytest.mark.gpu


def _t(g, *shape, dtype=torch.bfloat16):
    return torch.randn(*shape, generator=g).to(dtype).cuda()


def _items(seed, B, T, D, specs, dtype=torch.bfloat16):
    """specs: (Hq, Hkv, fused) per item -> list of (qs, ks, qt, kt) leaves."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for Hq, Hkv, fused in specs:
        qs = _t(g, B, Hq, T, D, dtype=dtype)
        qt = (qs.float() + 0.3 * _t(g, B, Hq, T, D, dtype=torch.float32)).to(dtype)
        if fused:
            out.append((qs, qs, qt, qt))
        else:
            out.append((qs, _t(g, B, Hkv, T, D, dtype=dtype), qt, _t(g, B, Hkv, T, D, dtype=dtype)))
    return out


def _leaves(items):
    res = []
    for qs, ks, qt, kt in items:
        q = qs.detach().clone().requires_grad_(True)
        k = q if ks is qs else ks.detach().clone().requires_grad_(True)
        res.append((q, k, qt, kt))
    return res


def _grads(items):
    return [(q.grad, None if k is q else k.grad) for q, k, _, _ in items]


def _check(items, mask=None, causal=True, weights=None):
    a = _leaves(items)
    losses = attn_kl_align_grouped(a, attn_mask=mask, causal=causal)
    assert path_is_tensor_core()
    w = torch.ones(len(items), device="cuda") if weights is None else weights
    (losses * w).sum().backward()
    b = _leaves(items)
    ref = torch.stack([attn_kl_align(*it, attn_mask=mask, causal=causal) for it in b])
    (ref * w).sum().backward()
    torch.cuda.synchronize()
    check_device_status()
    assert torch.equal(losses.detach(), ref.detach()), (losses, ref)
    for (ga, gb) in zip(_grads(a), _grads(b)):
        assert torch.equal(ga[0], gb[0])
        if gb[1] is not None:
            assert torch.equal(ga[1], gb[1])


def test_relations_of_two_layers_causal():
    # Q/Q (4 heads), K/K and V/V (2 heads each), for two layers, plus a GQA item
    specs = [(4, 4, True), (2, 2, True), (2, 2, True)] * 2 + [(4, 2, False)]
    _check(_items(1, 1, 700, 128, specs), weights=torch.linspace(0.5, 2.0, 7, device="cuda"))


def test_masked_noncausal_d64_fp16():
    B, T = 2, 300
    mask = (torch.rand(B, T, generator=torch.Generator().manual_seed(3)) > 0.3).to(torch.int32)
    mask[:, 0] = 1
    specs = [(2, 2, True), (4, 1, False), (2, 2, True)]
    _check(_items(2, B, T, 64, specs, torch.float16), mask=mask.cuda(), causal=False)


def test_strided_items_transposed_projections():
    """Items given as [B, H, T, D] views of [B, T, H, D] projections (what an
    attention hook sees) are read in place: same results as contiguous items."""
    B, T, D = 1, 520, 128
    g = torch.Generator().manual_seed(6)
    items = []
    for H in (4, 2, 2):
        xs = _t(g, B, T, H, D)
        xt = (xs.float() + 0.3 * _t(g, B, T, H, D, dtype=torch.float32)).to(torch.bfloat16)
        items.append((xs.transpose(1, 2), xs.transpose(1, 2), xt.transpose(1, 2),
                      xt.transpose(1, 2)))
    a = []
    for qs, _, qt, _ in items:
        leaf = qs.detach().transpose(1, 2).clone().transpose(1, 2).requires_grad_(True)
        assert not leaf.is_contiguous()
        a.append((leaf, leaf, qt, qt))
    losses = attn_kl_align_grouped(a)
    losses.sum().backward()
    b = [(qs.detach().contiguous().requires_grad_(True), qt.contiguous()) for qs, _, qt, _ in items]
    ref = attn_kl_align_grouped([(q, q, t, t) for q, t in b])
    ref.sum().backward()
    torch.cuda.synchronize()
    check_device_status()
    assert torch.equal(losses.detach(), ref.detach())
    for (q, _, _, _), (qr, _) in zip(a, b):
        assert torch.equal(q.grad, qr.grad)


def test_items_outside_the_tensor_core_path_fall_back_per_item():
    specs = [(2, 2, True)]
    items = _items(4, 1, 200, 32, specs)
    a = _leaves(items)
    got = attn_kl_align_grouped(a)
    ref = attn_kl_align(*_leaves(items)[0])
    assert torch.equal(got[0], ref)


def test_small_d_buffer_chunks_across_items():
    """Call the C ABI with room for only a few kv groups of D tiles."""
    L = _lib.lib()
    B, T, D = 1, 640, 128
    items = _items(5, B, T, D, [(4, 4, True), (2, 2, True), (4, 2, False), (2, 2, True)])
    n = len(items)
    prob = problem(items[0][0], items[0][1], items[0][2], items[0][3], True,
                   _lib.LKL_MASK_U8, None, None)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    lse = [(torch.empty(B, qs.shape[1], T, device="cuda"), torch.empty(B, qs.shape[1], T,
                                                                       device="cuda"))
           for qs, _, _, _ in items]
    grads = []
    for qs, ks, _, _ in items:
        dq = torch.full(qs.shape, float("nan"), device="cuda")
        grads.append((dq, dq if ks is qs else torch.full(ks.shape, float("nan"), device="cuda")))
    table = (_lib.LKLGroupItem * n)()
    for i, (qs, ks, qt, kt) in enumerate(items):
        table[i] = _lib.LKLGroupItem(qs.data_ptr(), ks.data_ptr(), qt.data_ptr(), kt.data_ptr(),
                                     qs.shape[1], ks.shape[1], kt.shape[1], 0,
                                     lse[i][0].data_ptr(), lse[i][1].data_ptr(),
                                     grads[i][0].data_ptr(), grads[i][1].data_ptr())
    losses = torch.empty(n, device="cuda")
    nf = L.lkl_grouped_workspace_size(n, table, ctypes.byref(prob), 0, 0)
    ws = torch.empty(nf, dtype=torch.uint8, device="cuda")
    assert L.lkl_forward_grouped(n, table, None, ctypes.byref(prob), ctypes.c_void_p(
        losses.data_ptr()), ctypes.c_void_p(ws.data_ptr()), nf, st) == 0
    full = L.lkl_grouped_workspace_size(n, table, ctypes.byref(prob), 0, 1)
    n_t = (T + 127) // 128
    tiles_head = n_t * (n_t + 1) // 2
    assert full - nf > 0
    outs = []
    for groups in (None, 3, 2):   # D tiles for all, 3 and 2 query heads' groups
        size = full if groups is None else full - (full - nf) + groups * tiles_head * 32768 + 4096
        wsb = torch.empty(size, dtype=torch.uint8, device="cuda")
        for dq, dk in grads:
            dq.fill_(float("nan"))
            dk.fill_(float("nan"))
        rc = L.lkl_backward_grouped(n, table, None, ctypes.byref(prob), None,
                                    ctypes.c_void_p(wsb.data_ptr()), size, st)
        assert rc == 0, _lib.STATUS.get(rc)
        torch.cuda.synchronize()
        check_device_status()
        outs.append([(dq.clone(), dk.clone()) for dq, dk in grads])
    for o in outs:
        for (a, b), (ra, rb) in zip(o, outs[0]):
            assert torch.isfinite(a).all() and torch.isfinite(b).all()
            assert torch.equal(a, ra) and torch.equal(b, rb)
    # and the per-item reference
    for i, (qs, ks, qt, kt) in enumerate(items):
        q = qs.detach().clone().requires_grad_(True)
        k = q if ks is qs else ks.detach().clone().requires_grad_(True)
        loss = attn_kl_align(q, k, qt, kt)
        loss.backward()
        assert torch.equal(loss.detach(), losses[i])
        if k is q:
            assert torch.equal(q.grad.float(), outs[0][i][0].to(q.grad.dtype).float())
        else:
            assert torch.equal(q.grad.float(), outs[0][i][0].to(q.grad.dtype).float())
            assert torch.equal(k.grad.float(), outs[0][i][1].to(k.grad.dtype).float())


def test_grouped_mixed_items_masked_noncausal():
    """Contiguous and strided items together, different student / teacher kv
    heads, a padding mask, non-causal: bitwise the per-item calls."""
    B, T, D = 2, 400, 128
    g = torch.Generator().manual_seed(41)
    mask = (torch.rand(B, T, generator=g) > 0.25).to(torch.bool)
    mask[:, 0] = True
    items = _items(42, B, T, D, [(4, 4, True), (4, 2, False)])
    # a strided item: [B, T, H, D] memory
    xs = _t(g, B, T, 4, D)
    xt = (xs.float() + 0.3 * _t(g, B, T, 4, D, dtype=torch.float32)).to(torch.bfloat16)
    ks = _t(g, B, T, 2, D)
    kt = _t(g, B, T, 1, D)
    items.append((xs.transpose(1, 2), ks.transpose(1, 2), xt.transpose(1, 2), kt.transpose(1, 2)))
    a = _leaves(items)
    losses = attn_kl_align_grouped(a, attn_mask=mask.cuda(), causal=False)
    assert path_is_tensor_core()
    losses.sum().backward()
    b = _leaves(items)
    from linearard_b200.attention_KL import attn_kl_align_strided
    ref = torch.stack([attn_kl_align_strided(*it, attn_mask=mask.cuda(), causal=False)
                       for it in b])
    ref.sum().backward()
    torch.cuda.synchronize()
    check_device_status()
    assert torch.equal(losses.detach(), ref.detach())
    for ga, gb in zip(_grads(a), _grads(b)):
        assert torch.equal(ga[0], gb[0])
        if gb[1] is not None:
            assert torch.equal(ga[1], gb[1])
