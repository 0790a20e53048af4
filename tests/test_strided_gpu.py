"""Strided inputs (``attn_kl_align_strided``, ``lkl_forward_strided`` /
``lkl_backward_strided``) on a B200.

The tensor-core kernels read [B, H, T, D] views in place through 4-D TMA
maps.  Each case builds the views an attention hook sees -- transposed
[B, T, H, D] projections, heads sliced out of a fused QKV projection, a
padded head dim -- and checks that the loss and the gradients are exactly
those of ``attn_kl_align`` on contiguous copies (same kernels, same values),
and, for one case, those of the numpy oracle.
"""
import math

import numpy as np
import pytest
import torch

from gpu_util import assert_grad_close, assert_loss_close, check_device_status, path_is_tensor_core
from linearard_b200.attention_KL import attn_kl_align, attn_kl_align_strided
from oracle import attn_kl_oracle as O

pytestmark = pytest.mark.gpu


def _proj(seed, B, T, H, D, dtype=torch.bfloat16, extra_heads=0, d_pad=0):
    """A [B, T, H + extra, D + pad] projection and its [B, H, T, D] view."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, H + extra_heads, D + d_pad, generator=g).to(dtype).cuda()
    return x, x[:, :, :H, :D].transpose(1, 2)


def _run(fn, s, t, ks=None, kt=None, mask=None, causal=True):
    """loss and the student gradient(s) of fn(qs, ks, qt, kt)."""
    leaf = s.detach().requires_grad_(True)
    leaf_k = None if ks is None else ks.detach().requires_grad_(True)
    qs, ksv = leaf, (leaf if leaf_k is None else leaf_k)
    qt, ktv = t, (t if kt is None else kt)
    loss = fn(qs, ksv, qt, ktv, mask, causal)
    loss.backward()
    torch.cuda.synchronize()
    check_device_status()
    return float(loss), leaf.grad, (None if leaf_k is None else leaf_k.grad)


def _compare(s, t, ks=None, kt=None, mask=None, causal=True):
    got = _run(attn_kl_align_strided, s, t, ks, kt, mask, causal)
    assert path_is_tensor_core()
    c = lambda x: None if x is None else x.contiguous()
    ref = _run(attn_kl_align, c(s), c(t), c(ks), c(kt), mask, causal)
    assert got[0] == ref[0], (got[0], ref[0])
    for a, b in zip(got[1:], ref[1:]):
        if b is not None:
            assert torch.equal(a, b)
    return got


@pytest.mark.parametrize("D", [16, 64, 128])
def test_transposed_projection_symmetric(D):
    # HF layout: q = proj(x).view(B, T, H, D).transpose(1, 2); symmetric call qs is ks
    _, s = _proj(1, 2, 700, 4, D)
    _, t = _proj(2, 2, 700, 4, D)
    assert not s.is_contiguous()
    loss, g, _ = _compare(s, t)
    sc = 1.0 / math.sqrt(D)
    S = s.float().cpu().numpy().astype(np.float64)
    Tt = t.float().cpu().numpy().astype(np.float64)
    ref_loss = O.oracle_attn_kl_align(S, S, Tt, Tt, None, True, sc, sc)[0]
    assert_loss_close(loss, ref_loss)
    dq, dk = O.oracle_attn_kl_align_backward(S, S, Tt, Tt, None, True, sc, sc)
    assert_grad_close(g.float().cpu().numpy(), dq + dk, "dS")


def test_heads_of_a_fused_qkv_projection_gqa_masked():
    # q: 8 heads and k: 2 heads sliced out of one [B, T, 12, 128] projection
    B, T, D = 1, 520, 128
    xs, _ = _proj(3, B, T, 12, D)
    xt, _ = _proj(4, B, T, 12, D)
    qs, ks = xs[:, :, :8].transpose(1, 2), xs[:, :, 8:10].transpose(1, 2)
    qt, kt = xt[:, :, :8].transpose(1, 2), xt[:, :, 8:10].transpose(1, 2)
    mask = (torch.rand(B, T, generator=torch.Generator().manual_seed(5)) > 0.3).to(torch.int32)
    mask[:, 0] = 1
    _compare(qs, qt, ks, kt, mask.cuda())


def test_padded_head_dim_noncausal_fp16():
    # a [B, H, T, 136] buffer read as D = 128 (t stride 136, a multiple of 8)
    _, s = _proj(6, 1, 300, 2, 128, torch.float16, d_pad=8)
    _, t = _proj(7, 1, 300, 2, 128, torch.float16, d_pad=8)
    s, t = s.transpose(1, 2).contiguous().transpose(1, 2), t
    _compare(s, t, causal=False)


def test_shapes_outside_the_tensor_core_path_use_contiguous_copies():
    _, s = _proj(8, 1, 200, 2, 256)
    _, t = _proj(9, 1, 200, 2, 256)
    got = _run(attn_kl_align_strided, s, t)
    ref = _run(attn_kl_align, s.contiguous(), t.contiguous())
    # the CUDA-core backward writes every gradient row once: bitwise equal
    assert got[0] == ref[0]
    torch.testing.assert_close(got[1], ref[1], rtol=0, atol=0)


def test_strided_asymmetric_kv_heads_masked_noncausal_fp16():
    """Student kv heads 2, teacher kv heads 4, padding mask, non-causal, fp16,
    every input a transposed projection: bitwise the contiguous call."""
    B, T, D = 2, 330, 64
    g = torch.Generator().manual_seed(31)
    def view(h):
        return torch.randn(B, T, h, D, generator=g).half().cuda().transpose(1, 2)
    qs, ks, qt, kt = view(8), view(2), view(8), view(4)
    mask = (torch.rand(B, T, generator=g) > 0.3).to(torch.int64)
    mask[:, 0] = 1
    _compare(qs, qt, ks, kt, mask.cuda(), causal=False)
