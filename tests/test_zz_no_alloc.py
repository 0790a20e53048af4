"""lkl_forward_noalloc: the fused forward for callers that cannot allocate.

Some callers of this library cannot allocate device memory -- a C/Go/Java
binding that only receives pointers from a framework owning the memory pool,
or code that must not call cudaMalloc mid-step because it can synchronise the
device.  lkl_forward_noalloc takes no workspace and uses a fixed scratch array
inside the library instead.  These tests call it through the C ABI and check
that it returns what lkl_forward (with a caller-provided workspace) returns, on
two calls in a row, and that it refuses problems beyond its scratch size.

The file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

from linearard_b200 import _lib

LOSS_REL = 1e-3   # loss tolerance used by every parity test
LSE_TOL = 1e-4


def _problem(B, Hq, Hkv, T, D, mask_dtype=_lib.LKL_MASK_I32):
    return _lib.LKLProblem(B=B, Hq=Hq, Hkv_s=Hkv, Hkv_t=Hkv, T=T, Ds=D, Dt=D,
                           dtype_s=_lib.LKL_BF16, dtype_t=_lib.LKL_BF16, causal=1,
                           mask_dtype=mask_dtype, sm_scale_s=0.0, sm_scale_t=0.0)


def _vp(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _inputs(seed, B, Hq, Hkv, T, D, with_mask):
    g = torch.Generator().manual_seed(seed)
    qs = torch.randn(B, Hq, T, D, generator=g).bfloat16().cuda()
    ks = torch.randn(B, Hkv, T, D, generator=g).bfloat16().cuda()
    qt = (qs.float().cpu() + 0.2 * torch.randn(B, Hq, T, D, generator=g)).bfloat16().cuda()
    kt = torch.randn(B, Hkv, T, D, generator=g).bfloat16().cuda()
    mask = None
    if with_mask:
        mask = (torch.rand(B, T, generator=g) > 0.3).to(torch.int32)
        mask[:, 0] = 1
        mask = mask.cuda()
    return qs, ks, qt, kt, mask


def _run(fn_name, args, prob, B, Hq, T):
    L = _lib.lib()
    lse_s = torch.empty(B, Hq, T, device="cuda")
    lse_t = torch.empty(B, Hq, T, device="cuda")
    loss = torch.empty((), device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    qs, ks, qt, kt, mask = args
    if fn_name == "lkl_forward":
        n = L.lkl_forward_workspace_size(ctypes.byref(prob), 1 if mask is not None else 0)
        ws = torch.empty(max(n, 256), dtype=torch.uint8, device="cuda")
        st = L.lkl_forward(_vp(qs), _vp(ks), _vp(qt), _vp(kt), _vp(mask), ctypes.byref(prob),
                           _vp(lse_s), _vp(lse_t), _vp(loss), _vp(ws), n, stream)
    else:
        st = L.lkl_forward_noalloc(_vp(qs), _vp(ks), _vp(qt), _vp(kt), _vp(mask),
                                   ctypes.byref(prob), _vp(lse_s), _vp(lse_t), _vp(loss), stream)
    assert st == 0, _lib.STATUS.get(st)
    torch.cuda.synchronize()
    return float(loss), lse_s, lse_t


@pytest.mark.gpu
def test_noalloc_matches_workspace_forward_two_calls():
    # two different problems back to back: the second (with a padding mask and
    # more tiles) must not see anything the first left in the shared scratch
    cases = [(1, (1, 4, 2, 700, 128), False), (2, (2, 4, 4, 1300, 64), True)]
    for seed, (B, Hq, Hkv, T, D), with_mask in cases:
        args = _inputs(seed, B, Hq, Hkv, T, D, with_mask)
        prob = _problem(B, Hq, Hkv, T, D)
        ref_loss, ref_ls, ref_lt = _run("lkl_forward", args, prob, B, Hq, T)
        loss, ls, lt = _run("lkl_forward_noalloc", args, prob, B, Hq, T)
        assert abs(loss - ref_loss) <= LOSS_REL * abs(ref_loss), (loss, ref_loss)
        torch.testing.assert_close(ls, ref_ls, rtol=LSE_TOL, atol=LSE_TOL)
        torch.testing.assert_close(lt, ref_lt, rtol=LSE_TOL, atol=LSE_TOL)
    assert _lib.lib().lkl_device_status() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,with_mask", [(1, 32768, True), (8, 32768, False)])
def test_noalloc_headline_relation_and_the_size_limit(B, T, with_mask):
    """One LLaMA3-8B Q/Q relation (32 heads x 32K tokens, with a padding mask),
    and 8 of them without a mask, whose scratch is exactly the 1 MiB limit."""
    Hq, Hkv, D = 32, 8, 128
    prob = _problem(B, Hq, Hkv, T, D)
    need = _lib.lib().lkl_forward_workspace_size(ctypes.byref(prob), 1 if with_mask else 0)
    assert need <= NOALLOC_BYTES
    if not with_mask:
        assert need == NOALLOC_BYTES
    g = torch.Generator(device="cuda").manual_seed(7)
    qs = torch.randn(B, Hq, T, D, device="cuda", generator=g).bfloat16()
    ks = torch.randn(B, Hkv, T, D, device="cuda", generator=g).bfloat16()
    qt = (qs.float() + 0.1 * torch.randn(B, Hq, T, D, device="cuda", generator=g)).bfloat16()
    kt = (ks.float() + 0.1 * torch.randn(B, Hkv, T, D, device="cuda", generator=g)).bfloat16()
    mask = None
    if with_mask:
        mask = (torch.rand(B, T, device="cuda", generator=g) > 0.1).to(torch.int32)
        mask[:, 0] = 1
    args = (qs, ks, qt, kt, mask)
    ref_loss, ref_ls, ref_lt = _run("lkl_forward", args, prob, B, Hq, T)
    loss, ls, lt = _run("lkl_forward_noalloc", args, prob, B, Hq, T)
    assert abs(loss - ref_loss) <= LOSS_REL * abs(ref_loss), (loss, ref_loss)
    torch.testing.assert_close(ls, ref_ls, rtol=LSE_TOL, atol=LSE_TOL)
    torch.testing.assert_close(lt, ref_lt, rtol=LSE_TOL, atol=LSE_TOL)
    assert _lib.lib().lkl_device_status() == 0


NOALLOC_BYTES = 1 << 20   # LKL_NOALLOC_SCRATCH_BYTES


@pytest.mark.parametrize("B,Hq,T,with_mask", [
    (8, 32, 32769, False),      # one 32-row block more than the exact fit
    (8, 32, 32768, True),       # the exact fit plus the packed mask
    (1, 32, 254145, True),      # one token past the largest masked sequence (254144)
    (8, 64, 1 << 20, False),    # far beyond (64 MiB of partials)
])
def test_noalloc_refuses_problems_beyond_its_scratch(B, Hq, T, with_mask):
    """Refused with LKL_ERR_TOO_LARGE before any device work (no GPU needed),
    exactly when the forward's scratch would exceed the fixed array."""
    L = _lib.lib()
    prob = _problem(B, Hq, 8, T, 128)
    assert L.lkl_forward_workspace_size(ctypes.byref(prob), int(with_mask)) > NOALLOC_BYTES
    fake = ctypes.c_void_p(0x10000)
    st = L.lkl_forward_noalloc(fake, fake, fake, fake, fake if with_mask else None,
                               ctypes.byref(prob), fake, fake, fake, None)
    assert st == 11, _lib.STATUS.get(st)


def test_noalloc_largest_masked_sequence_fits():
    """32 heads x 248K tokens with a mask is the largest masked one-sequence
    problem in the array (exactly 1 MiB; host-side size check only)."""
    L = _lib.lib()
    assert L.lkl_forward_workspace_size(ctypes.byref(_problem(1, 32, 8, 254144, 128)), 1) == \
        NOALLOC_BYTES
