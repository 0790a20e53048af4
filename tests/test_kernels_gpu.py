"""Kernel-level parity on a B200: every case of LinearARD's own kernel test
grids (tests/golden/cases.py), checked against fixtures produced by the
reference's oracles and against the numpy oracle, through both the sm_100a
tensor-core kernels and the generic CUDA-core kernels."""
import numpy as np
import pytest
import torch

import cases as C
from gpu_util import (REF_TOL, assert_grad_close, assert_loss_close, check_device_status, cuda,
                      force_generic, path_is_tensor_core)
from oracle import attn_kl_oracle as O

pytestmark = pytest.mark.gpu

TC_DIMS = (8, 16, 32, 64, 128)   # head dims on the tensor cores


@pytest.mark.parametrize("generic", [False, True], ids=["auto", "generic"])
@pytest.mark.parametrize("case", C.lse_cases(), ids=lambda c: c.name)
def test_lse_matches_reference(case, generic, golden):
    """kernel_A level: the tensor-core LSE-only launch for head dims 64 and
    128, the CUDA-core kernel for the others (and when forced)."""
    from linearard_b200.attention_KL import lse_stats
    q, k, mask = C.make_lse_inputs(case)
    with force_generic(generic):
        out = lse_stats(cuda(q), cuda(k), attn_mask=cuda(mask), causal=case.causal,
                        sm_scale=C.sm_scale(case.D))
        used_tc = path_is_tensor_core()
    torch.cuda.synchronize()
    check_device_status()
    assert used_tc == ((not generic) and case.D in TC_DIMS)
    rtol, atol = REF_TOL[case.dtype]
    ref = torch.from_numpy(golden[f"{case.name}/lse"])
    torch.testing.assert_close(out.cpu(), ref, rtol=rtol, atol=atol)
    orc = O.oracle_lse(C.to_np(q), C.to_np(k), C.to_np(mask), case.causal, C.sm_scale(case.D))
    np.testing.assert_allclose(out.cpu().numpy(), orc, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("generic", [False, True], ids=["auto", "generic"])
@pytest.mark.parametrize("case", C.kl_cases(), ids=lambda c: c.name)
def test_forward_backward_match_reference(case, generic, golden):
    from linearard_b200.attention_KL import attn_kl_forward, kl_backward, kl_forward
    qs, ks, qt, kt, mask = C.make_kl_inputs(case)
    sc_s, sc_t = C.sm_scale(case.Ds), C.sm_scale(case.Dt)
    g = {k: golden[f"{case.name}/{k}"] for k in ("lse_s", "lse_t", "kl", "dq", "dk")}
    Q = [cuda(x) for x in (qs, ks, qt, kt)]
    m = cuda(mask)
    rtol, atol = REF_TOL[case.dtype]
    with force_generic(generic):
        loss, lse_s, lse_t = attn_kl_forward(*Q, attn_mask=m, causal=case.causal,
                                             sm_scale_s=sc_s, sm_scale_t=sc_t)
        used_tc = path_is_tensor_core()
        dq, dk = kl_backward(Q[0], Q[1], lse_s, Q[2], Q[3], lse_t, attn_mask=m,
                             causal=case.causal, sm_scale_s=sc_s, sm_scale_t=sc_t)
        used_tc_b = path_is_tensor_core()
    torch.cuda.synchronize()
    check_device_status()
    expect_tc = (not generic) and case.Ds in TC_DIMS and case.Dt in TC_DIMS
    # the tensor-core backward covers different student / teacher kv-head counts too
    assert used_tc == expect_tc and used_tc_b == expect_tc
    torch.testing.assert_close(lse_s.cpu(), torch.from_numpy(g["lse_s"]), rtol=rtol, atol=atol)
    torch.testing.assert_close(lse_t.cpu(), torch.from_numpy(g["lse_t"]), rtol=rtol, atol=atol)
    assert_loss_close(float(loss), float(g["kl"]))
    torch.testing.assert_close(dq.cpu(), torch.from_numpy(g["dq"]), rtol=rtol, atol=atol)
    torch.testing.assert_close(dk.cpu(), torch.from_numpy(g["dk"]), rtol=rtol, atol=atol)
    assert_grad_close(dq.cpu().numpy(), g["dq"], "dq")
    assert_grad_close(dk.cpu().numpy(), g["dk"], "dk")
    # kernel-B level: KL from the reference's own LSEs
    lse_ref_s = torch.from_numpy(g["lse_s"]).cuda()
    lse_ref_t = torch.from_numpy(g["lse_t"]).cuda()
    with force_generic(generic):
        kl_b = kl_forward(*Q[:2], lse_ref_s, *Q[2:], lse_ref_t, attn_mask=m, causal=case.causal,
                          sm_scale_s=sc_s, sm_scale_t=sc_t)
        assert path_is_tensor_core() == expect_tc
    assert_loss_close(float(kl_b), float(g["kl"]))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", (32, 64, 128))
@pytest.mark.parametrize("T", [1, 127, 128, 129, 383, 640])
@pytest.mark.parametrize("causal", [True, False])
def test_tensor_core_vs_oracle_tile_edges(D, T, causal, dtype):
    """Ragged T around the 128-row tile, both dtypes, GQA, against the oracle."""
    from linearard_b200.attention_KL import attn_kl_forward, kl_backward
    gen = torch.Generator().manual_seed(T * 7 + D)
    B, Hq, Hkv = 1, 4, 2
    qs = torch.randn(B, Hq, T, D, generator=gen).to(dtype)
    ks = torch.randn(B, Hkv, T, D, generator=gen).to(dtype)
    qt = (qs.float() + 0.3 * torch.randn(B, Hq, T, D, generator=gen)).to(dtype)
    kt = torch.randn(B, Hkv, T, D, generator=gen).to(dtype)
    Q = [x.cuda() for x in (qs, ks, qt, kt)]
    loss, lse_s, lse_t = attn_kl_forward(*Q, causal=causal)
    assert path_is_tensor_core()
    dq, dk = kl_backward(Q[0], Q[1], lse_s, Q[2], Q[3], lse_t, causal=causal)
    torch.cuda.synchronize()
    check_device_status()
    a = [C.to_np(x) for x in (qs, ks, qt, kt)]
    ref_loss, rls, rlt = O.oracle_attn_kl_align(*a, None, causal)
    np.testing.assert_allclose(lse_s.cpu().numpy(), rls, rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(lse_t.cpu().numpy(), rlt, rtol=1e-4, atol=1e-4)
    assert_loss_close(float(loss), ref_loss)
    rdq, rdk = O.oracle_grad(*a[:2], rls, *a[2:], rlt, None, causal)
    assert_grad_close(dq.cpu().numpy(), rdq, "dq")
    assert_grad_close(dk.cpu().numpy(), rdk, "dk")


@pytest.mark.parametrize("mdtype", [torch.bool, torch.uint8, torch.int32, torch.int64])
def test_mask_dtypes_and_cpu_mask(mdtype):
    """Every mask dtype the reference accepts, passed on the CPU (moved to the
    device like kernel_A.py:210-213), with rows that are entirely padding."""
    from linearard_b200.attention_KL import attn_kl_forward, kl_backward
    gen = torch.Generator().manual_seed(5)
    B, H, T, D = 2, 2, 300, 128
    qs = torch.randn(B, H, T, D, generator=gen).bfloat16()
    qt = torch.randn(B, H, T, D, generator=gen).bfloat16()
    mask = (torch.rand(B, T, generator=gen) > 0.4)
    mask[:, 0] = True
    mask[1, 150:] = False  # a padded tail
    mask = mask.to(mdtype)
    Q = [qs.cuda(), qt.cuda()]
    loss, ls, lt = attn_kl_forward(Q[0], Q[0], Q[1], Q[1], attn_mask=mask)
    assert path_is_tensor_core()
    dq, dk = kl_backward(Q[0], Q[0], ls, Q[1], Q[1], lt, attn_mask=mask)
    torch.cuda.synchronize()
    a, t = C.to_np(qs), C.to_np(qt)
    m = mask.to(torch.int32).numpy()
    ref_loss, rls, rlt = O.oracle_attn_kl_align(a, a, t, t, m, True)
    np.testing.assert_allclose(ls.cpu().numpy(), rls, rtol=1e-4, atol=1e-4)
    assert np.all(ls.cpu().numpy()[1, :, 150:] == 0.0)
    assert_loss_close(float(loss), ref_loss)
    rdq, rdk = O.oracle_grad(a, a, rls, t, t, rlt, m, True)
    assert_grad_close(dq.cpu().numpy(), rdq, "dq")
    assert_grad_close(dk.cpu().numpy(), rdk, "dk")
    assert np.all(dq.cpu().numpy()[1, :, 150:] == 0.0)


@pytest.mark.parametrize("D", TC_DIMS)
@pytest.mark.parametrize("T", [1, 129, 383, 1000])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("masked", [False, True])
def test_tensor_core_lse_and_kl_given_lse_vs_oracle(D, T, causal, masked):
    """The kernel-A / kernel-B level entry points on the tensor cores: ragged
    T, GQA, padding masks (including a padded first token, whose row has no
    valid column under the causal mask), against the oracle."""
    from linearard_b200.attention_KL import kl_forward, lse_stats
    gen = torch.Generator().manual_seed(T * 13 + D + (7 if masked else 0))
    B, Hq, Hkv = 2, 4, 2
    qs = torch.randn(B, Hq, T, D, generator=gen).bfloat16()
    ks = torch.randn(B, Hkv, T, D, generator=gen).bfloat16()
    qt = (qs.float() + 0.2 * torch.randn(B, Hq, T, D, generator=gen)).bfloat16()
    kt = torch.randn(B, Hq, T, D, generator=gen).bfloat16()
    mask = None
    if masked:
        mask = (torch.rand(B, T, generator=gen) > 0.25).to(torch.int32)
        mask[:, 0] = 0
    a = [C.to_np(x) for x in (qs, ks, qt, kt)]
    m_np = None if mask is None else C.to_np(mask)
    ref_ls = O.oracle_lse(a[0], a[1], m_np, causal)
    ref_lt = O.oracle_lse(a[2], a[3], m_np, causal)
    ls = lse_stats(qs.cuda(), ks.cuda(), attn_mask=cuda(mask), causal=causal)
    assert path_is_tensor_core()
    lt = lse_stats(qt.cuda(), kt.cuda(), attn_mask=cuda(mask), causal=causal)
    torch.cuda.synchronize()
    check_device_status()
    np.testing.assert_allclose(ls.cpu().numpy(), ref_ls, rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(lt.cpu().numpy(), ref_lt, rtol=1e-4, atol=1e-4)
    # KL given the oracle's LSEs (-inf rows included)
    kl = kl_forward(qs.cuda(), ks.cuda(), torch.from_numpy(ref_ls).float().cuda(), qt.cuda(),
                    kt.cuda(), torch.from_numpy(ref_lt).float().cuda(), attn_mask=cuda(mask),
                    causal=causal)
    assert path_is_tensor_core()
    ref_kl = O.oracle_kl(a[0], a[1], ref_ls, a[2], a[3], ref_lt, m_np, causal)
    assert_loss_close(float(kl), ref_kl)


@pytest.mark.parametrize("D", [256])
def test_cuda_core_backward_is_bit_reproducible(D):
    """Head dims outside the tensor-core kernels: the CUDA-core backward writes
    each dq and dk row once (a dq launch, then a column-stationary dk launch),
    so repeated calls agree bit for bit; GQA and the fused dq + dk buffer."""
    from linearard_b200.attention_KL import attn_kl_forward, kl_backward
    g = torch.Generator().manual_seed(D)
    B, Hq, Hkv, T = 1, 4, 2, 300
    qs = torch.randn(B, Hq, T, D, generator=g).bfloat16().cuda()
    ks = torch.randn(B, Hkv, T, D, generator=g).bfloat16().cuda()
    qt = (qs.float() + 0.2 * torch.randn(B, Hq, T, D, generator=g).cuda()).bfloat16()
    kt = torch.randn(B, Hkv, T, D, generator=g).bfloat16().cuda()
    loss, ls, lt = attn_kl_forward(qs, ks, qt, kt)
    outs = [kl_backward(qs, ks, ls, qt, kt, lt) for _ in range(3)]
    assert not path_is_tensor_core()
    fused = [kl_backward(qs, qs, ls, qt, qt, lt, fused=True)[0] for _ in range(2)]
    torch.cuda.synchronize()
    for dq, dk in outs[1:]:
        assert torch.equal(dq, outs[0][0]) and torch.equal(dk, outs[0][1])
    assert torch.equal(fused[0], fused[1])
    a = [C.to_np(x.cpu()) for x in (qs, ks, qt, kt)]
    _, rls, rlt = O.oracle_attn_kl_align(*a)
    rdq, rdk = O.oracle_grad(a[0], a[1], rls, a[2], a[3], rlt)
    assert_grad_close(outs[0][0].cpu().numpy(), rdq, "dq")
    assert_grad_close(outs[0][1].cpu().numpy(), rdk, "dk")
