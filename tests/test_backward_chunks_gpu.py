"""Chunked tensor-core backward on a B200.

The backward stores the rounded D tiles of the dq launch in the workspace and
the dk launch streams them back.  When the workspace holds fewer D tiles than
the problem has, the work is split into chunks (whole kv groups, or ranges of
query tiles of one group), each a dq launch and a dk launch.  These tests pass
workspaces of several sizes through the C ABI and check that every plan gives
the gradients of the one-chunk plan and of the numpy oracle, including the
fused dq + dk output (qs is ks) and the non-causal case whose fused output is
cleared and accumulated.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from gpu_util import assert_grad_close, check_device_status
from linearard_b200 import _lib
from oracle import attn_kl_oracle as O

pytestmark = pytest.mark.gpu

TILE_BYTES = 128 * 128 * 2


def _vp(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _inputs(seed, B, Hq, Hkv, T, D, fused):
    g = torch.Generator().manual_seed(seed)
    qs = torch.randn(B, Hq, T, D, generator=g).bfloat16()
    ks = qs if fused else torch.randn(B, Hkv, T, D, generator=g).bfloat16()
    qt = (qs.float() + 0.3 * torch.randn(B, Hq, T, D, generator=g)).bfloat16()
    kt = qt if fused else torch.randn(B, Hkv, T, D, generator=g).bfloat16()
    return qs, ks, qt, kt


def _run(args, prob, d_tiles, fused, mask=None):
    """lkl_forward, then lkl_backward with room for `d_tiles` D tiles (None = the
    size lkl_backward_workspace_size asks for)."""
    L = _lib.lib()
    qs, qt = args[0].cuda(), args[2].cuda()
    ks = qs if fused else args[1].cuda()
    kt = qt if fused else args[3].cuda()
    B, Hq, T, D = qs.shape
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    has_mask = 1 if mask is not None else 0
    lse_s = torch.empty(B, Hq, T, device="cuda")
    lse_t = torch.empty(B, Hq, T, device="cuda")
    loss = torch.empty((), device="cuda")
    n_f = L.lkl_workspace_size(ctypes.byref(prob), has_mask)
    ws = torch.empty(max(n_f, 256), dtype=torch.uint8, device="cuda")
    assert L.lkl_forward(_vp(qs), _vp(ks), _vp(qt), _vp(kt), _vp(mask), ctypes.byref(prob),
                         _vp(lse_s), _vp(lse_t), _vp(loss), _vp(ws), n_f, st) == 0
    n_b = L.lkl_backward_workspace_size(ctypes.byref(prob), has_mask)
    if d_tiles is not None:
        n_b = n_f + d_tiles * TILE_BYTES
    wsb = torch.empty(n_b, dtype=torch.uint8, device="cuda")
    dq = torch.full((B, Hq, T, D), float("nan"), device="cuda")
    dk = dq if fused else torch.full((B, ks.shape[1], T, D), float("nan"), device="cuda")
    rc = L.lkl_backward(_vp(qs), _vp(ks), _vp(lse_s), _vp(qt), _vp(kt), _vp(lse_t), _vp(mask),
                        ctypes.byref(prob), None, _vp(dq), _vp(dk), _vp(wsb), n_b, st)
    assert rc == 0, _lib.STATUS.get(rc)
    assert L.lkl_last_path() == 1, "expected the tensor-core backward"
    torch.cuda.synchronize()
    check_device_status()
    return dq.cpu(), (None if fused else dk.cpu()), lse_s.cpu(), lse_t.cpu()


def _problem(B, Hq, Hkv, T, D, causal, mask_dtype=_lib.LKL_MASK_I32):
    return _lib.LKLProblem(B=B, Hq=Hq, Hkv_s=Hkv, Hkv_t=Hkv, T=T, Ds=D, Dt=D,
                           dtype_s=_lib.LKL_BF16, dtype_t=_lib.LKL_BF16,
                           causal=1 if causal else 0, mask_dtype=mask_dtype,
                           sm_scale_s=0.0, sm_scale_t=0.0)


def _tiles(T, causal):
    n = math.ceil(T / 128)
    return n * (n + 1) // 2 if causal else n * n


# (name, B, Hq, Hkv, T, D, causal, fused, D-tile budgets)
CASES = [
    # GQA, causal: whole groups per chunk, then query-tile ranges (rows split)
    ("gqa_causal", 1, 4, 2, 1300, 128, True, False, (132, 60, 22)),
    # fused output, causal: dk adds into rows that earlier dq launches wrote
    ("fused_causal", 2, 2, 2, 1000, 64, True, True, (36, 16, 8)),
    # non-causal, separate outputs: later chunks add into dk
    ("gqa_noncausal", 1, 4, 2, 700, 128, False, False, (72, 30, 12)),
    # non-causal fused: the output is cleared first and every launch adds
    ("fused_noncausal", 1, 2, 2, 600, 64, False, True, (25, 10, 5)),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: c[0])
def test_chunked_backward_matches_one_chunk(case):
    name, B, Hq, Hkv, T, D, causal, fused, budgets = case
    args = _inputs(len(name), B, Hq, Hkv, T, D, fused)
    prob = _problem(B, Hq, Hkv, T, D, causal)
    G = Hq // Hkv
    full_tiles = B * Hq * _tiles(T, causal)
    n_f = _lib.lib().lkl_workspace_size(ctypes.byref(prob), 0)
    assert _lib.lib().lkl_backward_workspace_size(ctypes.byref(prob), 0) == \
        n_f + full_tiles * TILE_BYTES
    ref_dq, ref_dk, lse_s, lse_t = _run(args, prob, None, fused)
    assert torch.isfinite(ref_dq).all()
    for tiles in budgets:
        assert tiles >= G * math.ceil(T / 128)   # the smallest budget the ABI accepts
        dq, dk, _, _ = _run(args, prob, tiles, fused)
        # dq rows are computed the same way in every plan; dk sums chunk
        # partials in a different order
        torch.testing.assert_close(dq, ref_dq, rtol=1e-5, atol=1e-6)
        if not fused:
            torch.testing.assert_close(dk, ref_dk, rtol=1e-5, atol=1e-6)
    # and the one-chunk plan against the numpy oracle
    qs, ks, qt, kt = (C.float().numpy().astype(np.float64) for C in args)
    sc = 1.0 / math.sqrt(D)
    dq_o, dk_o = O.oracle_grad(qs, ks, lse_s.numpy(), qt, kt, lse_t.numpy(), None, causal, sc, sc)
    if fused:
        assert_grad_close(ref_dq.numpy(), dq_o + dk_o, "dq+dk")
    else:
        assert_grad_close(ref_dq.numpy(), dq_o, "dq")
        assert_grad_close(ref_dk.numpy(), dk_o, "dk")


def test_chunked_backward_gqa4_with_padding_mask():
    """Four query heads per kv head and a padding mask, with workspaces from
    the whole D buffer down to one query-tile row of a kv group."""
    B, Hq, Hkv, T, D = 2, 8, 2, 520, 128
    args = _inputs(11, B, Hq, Hkv, T, D, False)
    g = torch.Generator().manual_seed(12)
    mask = (torch.rand(B, T, generator=g) > 0.25).to(torch.int32)
    mask[:, 0] = 1
    mask = mask.cuda()
    prob = _problem(B, Hq, Hkv, T, D, True)
    n_t = math.ceil(T / 128)
    ref_dq, ref_dk, lse_s, lse_t = _run(args, prob, None, False, mask)
    for tiles in (2 * 4 * _tiles(T, True), 4 * _tiles(T, True), 4 * n_t):
        dq, dk, _, _ = _run(args, prob, tiles, False, mask)
        torch.testing.assert_close(dq, ref_dq, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(dk, ref_dk, rtol=1e-5, atol=1e-6)
    qs, ks, qt, kt = (C.float().numpy().astype(np.float64) for C in args)
    sc = 1.0 / math.sqrt(D)
    dq_o, dk_o = O.oracle_grad(qs, ks, lse_s.numpy(), qt, kt, lse_t.numpy(), mask.cpu().numpy(),
                               True, sc, sc)
    assert_grad_close(ref_dq.numpy(), dq_o, "dq")
    assert_grad_close(ref_dk.numpy(), dk_o, "dk")


def test_tensor_core_backward_with_different_kv_head_counts():
    """Student kv heads 2, teacher kv heads 4 (Hq 8): the tensor-core backward
    (the teacher grouping enters only the dq launch's teacher scores), whole
    and chunked, against the oracle."""
    L = _lib.lib()
    B, Hq, Hkv_s, Hkv_t, T, D = 1, 8, 2, 4, 400, 64
    g = torch.Generator().manual_seed(21)
    qs = torch.randn(B, Hq, T, D, generator=g).bfloat16()
    ks = torch.randn(B, Hkv_s, T, D, generator=g).bfloat16()
    qt = (qs.float() + 0.3 * torch.randn(B, Hq, T, D, generator=g)).bfloat16()
    kt = torch.randn(B, Hkv_t, T, D, generator=g).bfloat16()
    prob = _lib.LKLProblem(B=B, Hq=Hq, Hkv_s=Hkv_s, Hkv_t=Hkv_t, T=T, Ds=D, Dt=D,
                           dtype_s=_lib.LKL_BF16, dtype_t=_lib.LKL_BF16, causal=1,
                           mask_dtype=_lib.LKL_MASK_I32, sm_scale_s=0.0, sm_scale_t=0.0)
    args = (qs, ks, qt, kt)
    ref_dq, ref_dk, lse_s, lse_t = _run(args, prob, None, False)
    dq, dk, _, _ = _run(args, prob, (Hq // Hkv_s) * math.ceil(T / 128), False)
    torch.testing.assert_close(dq, ref_dq, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(dk, ref_dk, rtol=1e-5, atol=1e-6)
    a = [x.float().numpy().astype(np.float64) for x in args]
    sc = 1.0 / math.sqrt(D)
    dq_o, dk_o = O.oracle_grad(a[0], a[1], lse_s.numpy(), a[2], a[3], lse_t.numpy(), None, True,
                               sc, sc)
    assert_grad_close(ref_dq.numpy(), dq_o, "dq")
    assert_grad_close(ref_dk.numpy(), dk_o, "dk")


def test_backward_refuses_less_than_one_row_of_tiles():
    L = _lib.lib()
    B, Hq, Hkv, T, D = 1, 4, 2, 1300, 128
    prob = _problem(B, Hq, Hkv, T, D, True)
    qs, ks, qt, kt = (x.cuda() for x in _inputs(7, B, Hq, Hkv, T, D, False))
    lse = torch.zeros(B, Hq, T, device="cuda")
    dq = torch.empty(B, Hq, T, D, device="cuda")
    dk = torch.empty(B, Hkv, T, D, device="cuda")
    n_f = L.lkl_workspace_size(ctypes.byref(prob), 0)
    row = (Hq // Hkv) * math.ceil(T / 128)
    ws = torch.empty(n_f + row * TILE_BYTES, dtype=torch.uint8, device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.lkl_backward(_vp(qs), _vp(ks), _vp(lse), _vp(qt), _vp(kt), _vp(lse), None,
                        ctypes.byref(prob), None, _vp(dq), _vp(dk), _vp(ws),
                        n_f + row * TILE_BYTES - 256, st)
    assert rc == 6, _lib.STATUS.get(rc)
