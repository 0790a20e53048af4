"""C-ABI checks that need no GPU: the library loads, exports every function
that include/linearard_b200.h declares, and rejects bad arguments with the
documented status codes before touching the device."""
import ctypes
import os
import re

import pytest
import torch

from linearard_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "linearard_b200.h")


def header_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(lkl_\w+)\s*\(", src, re.M)))


def test_library_loads_and_exports_header_symbols():
    L = _lib.lib()
    names = header_functions()
    assert len(names) >= 10
    assert set(names) == set(_lib.EXPORTS)
    for n in names:
        assert hasattr(L, n), n
    # the version build() checks: the header's LKL_ABI_VERSION
    want = int(re.search(r"#define LKL_ABI_VERSION (\d+)", open(HEADER).read()).group(1))
    assert L.lkl_abi_version() == want


def test_status_strings():
    L = _lib.lib()
    for code in range(13):
        assert L.lkl_status_string(code)
    assert L.lkl_status_string(0) == b"ok"


def _prob(**kw):
    d = dict(B=1, Hq=4, Hkv_s=2, Hkv_t=4, T=300, Ds=128, Dt=128, dtype_s=1, dtype_t=1,
             causal=1, mask_dtype=2, sm_scale_s=0.0, sm_scale_t=0.0)
    d.update(kw)
    return _lib.LKLProblem(**d)


def test_workspace_size():
    L = _lib.lib()
    p = _prob()
    n0 = L.lkl_workspace_size(ctypes.byref(p), 0)
    n1 = L.lkl_workspace_size(ctypes.byref(p), 1)
    assert n0 % 256 == 0 and n1 % 256 == 0
    # one fp32 partial per 32-row block of each (batch, head)
    assert n0 >= 4 * 1 * 4 * ((300 + 31) // 32)
    assert n1 - n0 >= 1 * ((300 + 31) // 32) * 4
    assert L.lkl_workspace_size(ctypes.byref(_prob(T=0)), 1) == 0
    # the forward entry points need only the partials and the mask bits; the
    # common size adds the backward's 8 bytes per (batch, head, row)
    f0 = L.lkl_forward_workspace_size(ctypes.byref(p), 0)
    f1 = L.lkl_forward_workspace_size(ctypes.byref(p), 1)
    assert f0 == 256 * ((4 * 4 * ((300 + 31) // 32) + 255) // 256)
    assert f1 == f0 + 256
    assert n0 == f0 + 256 * ((8 * 4 * 300 + 255) // 256)
    assert n1 == f1 + (n0 - f0)
    assert L.lkl_forward_workspace_size(ctypes.byref(_prob(T=0)), 1) == 0


def test_backward_workspace_holds_the_d_tiles():
    """Tensor-core shapes add one 32 KB D tile per (query head, tile pair);
    beyond 8 GiB the buffer is capped and the backward runs in chunks."""
    L = _lib.lib()
    for mask in (0, 1):
        p = _prob(Hkv_t=2)                      # tensor-core backward
        base = L.lkl_workspace_size(ctypes.byref(p), mask)
        n_t = (300 + 127) // 128
        tiles = 1 * 4 * n_t * (n_t + 1) // 2    # causal: tiles j <= i per head
        assert L.lkl_backward_workspace_size(ctypes.byref(p), mask) == base + tiles * 32768
        nc = _prob(Hkv_t=2, causal=0)
        assert (L.lkl_backward_workspace_size(ctypes.byref(nc), mask)
                == L.lkl_workspace_size(ctypes.byref(nc), mask) + 4 * n_t * n_t * 32768)
    # shapes served by the CUDA-core kernels need nothing extra
    for kw in (dict(Ds=256, Dt=256, Hkv_t=2), dict(Ds=256, Dt=128)):   # head dim 256
        p = _prob(**kw)
        assert (L.lkl_backward_workspace_size(ctypes.byref(p), 0)
                == L.lkl_workspace_size(ctypes.byref(p), 0))
    # different student / teacher kv-head counts: tensor-core backward as well
    asym = _prob()                                      # Hkv_s 2, Hkv_t 4
    assert (L.lkl_backward_workspace_size(ctypes.byref(asym), 0)
            == L.lkl_workspace_size(ctypes.byref(asym), 0) + 4 * n_t * (n_t + 1) // 2 * 32768)
    # LLaMA3-8B Q/Q relation at 32K: 32 heads x 32896 tiles -> capped at 8 GiB
    big = _prob(B=1, Hq=32, Hkv_s=32, Hkv_t=32, T=32768)
    extra = (L.lkl_backward_workspace_size(ctypes.byref(big), 0)
             - L.lkl_workspace_size(ctypes.byref(big), 0))
    assert extra == 8 << 30
    assert L.lkl_backward_workspace_size(ctypes.byref(_prob(T=0)), 0) == 0


def test_backward_rejects_a_forward_sized_workspace():
    L = _lib.lib()
    p = _prob(Hkv_t=2)
    fake = ctypes.c_void_p(0x10000)
    n = L.lkl_workspace_size(ctypes.byref(p), 0)
    st = L.lkl_backward(fake, fake, fake, fake, fake, fake, None, ctypes.byref(p), None,
                        fake, ctypes.c_void_p(0x20000), fake, n, None)
    assert st == 6, _lib.STATUS.get(st)


@pytest.mark.parametrize("kw,code", [
    (dict(Hq=6, Hkv_s=4), 2),       # Hq % Hkv_s
    (dict(Hkv_t=3), 2),             # Hq % Hkv_t
    (dict(Ds=96), 3),               # head dim
    (dict(Dt=512), 3),
    (dict(dtype_s=7), 4),
    (dict(mask_dtype=9), 4),
    (dict(B=-1), 2),
])
def test_bad_problem_rejected_before_device(kw, code):
    L = _lib.lib()
    p = _prob(**kw)
    fake = ctypes.c_void_p(0x10000)
    st = L.lkl_forward(fake, fake, fake, fake, None, ctypes.byref(p), fake, fake, fake,
                       fake, 1 << 20, None)
    assert st == code, _lib.STATUS.get(st)


def test_null_pointers_and_alias_rules():
    L = _lib.lib()
    p = _prob(Hkv_s=4)
    fake = ctypes.c_void_p(0x10000)
    other = ctypes.c_void_p(0x20000)
    assert L.lkl_forward(None, fake, fake, fake, None, ctypes.byref(p), fake, fake, fake,
                         fake, 1 << 20, None) == 1
    # dq == dk but qs != ks -> bad alias
    assert L.lkl_backward(fake, other, fake, fake, fake, fake, None, ctypes.byref(p), None,
                          fake, fake, fake, 1 << 20, None) == 10
    # misaligned gradient buffer
    odd = ctypes.c_void_p(0x10004)
    assert L.lkl_backward(fake, fake, fake, fake, fake, fake, None, ctypes.byref(p), None,
                          odd, fake, fake, 1 << 20, None) == 5


def test_workspace_too_small_rejected():
    L = _lib.lib()
    p = _prob()
    fake = ctypes.c_void_p(0x10000)
    st = L.lkl_forward(fake, fake, fake, fake, None, ctypes.byref(p), fake, fake, fake,
                       fake, 16, None)
    assert st == 6


def test_empty_sequence_is_not_an_error_for_lse():
    L = _lib.lib()
    p = _prob(T=0)
    fake = ctypes.c_void_p(0x10000)
    assert L.lkl_lse(fake, fake, None, ctypes.byref(p), fake, None, 0, None) == 0


def test_python_wrappers_assert_like_reference():
    """Same failure mode as the reference wrappers (AssertionError) on CPU tensors."""
    from linearard_b200.attention_KL import attn_kl_align, lse_stats
    q = torch.randn(1, 2, 8, 16, dtype=torch.float16)
    with pytest.raises(AssertionError, match="must be on CUDA"):
        lse_stats(q, q)
    with pytest.raises(AssertionError):
        attn_kl_align(q, q, q, q)


def test_wrapper_has_no_tensor_math():
    """The reference's static audit (test_kernel_A.py:102-119): wrapper sources
    contain no torch math calls -- everything is computed by the library."""
    import inspect
    from linearard_b200.attention_KL import kernel_A, kernel_B, kernel_C, integration
    banned = ["matmul", "einsum", "softmax", "logsumexp", "exp(", "log(", "sum(", "max(",
              "mean(", "transpose"]
    for fn in (kernel_A.lse_stats, kernel_B.kl_forward, kernel_C.kl_backward,
               integration.attn_kl_forward, integration.AttnKLAlignFn.forward,
               integration.AttnKLAlignFn.backward):
        src = inspect.getsource(fn).lower()
        for key in banned:
            assert key not in src, f"{fn.__qualname__} contains {key}"


def test_strided_entry_points_validate_before_device():
    L = _lib.lib()
    p = _prob(Hkv_t=2)
    fake = ctypes.c_void_p(0x10000)
    good = (_lib.LKLStrides * 4)(*[_lib.LKLStrides(b=300 * 4 * 128, h=128, t=4 * 128)] * 4)
    odd = (_lib.LKLStrides * 4)(*[_lib.LKLStrides(b=300 * 4 * 128, h=128, t=4 * 128 + 4)] * 4)
    zero = (_lib.LKLStrides * 4)(*[_lib.LKLStrides(b=0, h=128, t=512)] * 4)
    n = 1 << 20
    f = L.lkl_forward_strided
    assert f(fake, fake, fake, fake, None, None, ctypes.byref(p), fake, fake, fake, fake, n,
             None) == 1
    assert f(fake, fake, fake, fake, odd, None, ctypes.byref(p), fake, fake, fake, fake, n,
             None) == 5
    assert f(fake, fake, fake, fake, zero, None, ctypes.byref(p), fake, fake, fake, fake, n,
             None) == 2
    assert f(ctypes.c_void_p(0x10008), fake, fake, fake, good, None, ctypes.byref(p), fake,
             fake, fake, fake, n, None) == 5     # base pointer not 16-byte aligned
    b = L.lkl_backward_strided
    other = ctypes.c_void_p(0x20000)
    # dq == dk with qs != ks -> bad alias
    assert b(fake, other, fake, fake, fake, fake, good, None, ctypes.byref(p), None, fake, fake,
             fake, n, None) == 10
    assert L.lkl_status_string(12)


def test_grouped_entry_points_validate_before_device():
    L = _lib.lib()
    shared = _prob(Hkv_t=2)
    fake = 0x10000

    def item(Hq=4, Hkv_s=2, Hkv_t=2, dq=fake, dk=fake + 0x1000, qs=fake, ks=fake + 0x2000):
        return _lib.LKLGroupItem(qs, ks, fake, fake, Hq, Hkv_s, Hkv_t, 0, fake, fake, dq, dk)

    one = (_lib.LKLGroupItem * 1)(item())
    n_f = L.lkl_grouped_workspace_size(1, one, ctypes.byref(shared), 0, 0)
    n_b = L.lkl_grouped_workspace_size(1, one, ctypes.byref(shared), 0, 1)
    assert n_f > 0 and n_f % 256 == 0
    n_t = (300 + 127) // 128
    assert n_b - n_f >= 4 * n_t * (n_t + 1) // 2 * 32768   # every D tile fits (< 8 GiB)
    # head dim 256 is outside the tensor-core path
    small = _prob(Ds=256, Dt=256, Hkv_t=2)
    assert L.lkl_grouped_workspace_size(1, one, ctypes.byref(small), 0, 0) == 0
    c = ctypes.c_void_p
    assert L.lkl_forward_grouped(1, one, None, ctypes.byref(small), c(fake), c(fake), 1 << 20,
                                 None) == 12
    # dq == dk with qs != ks
    bad = (_lib.LKLGroupItem * 1)(item(dq=fake, dk=fake))
    assert L.lkl_backward_grouped(1, bad, None, ctypes.byref(shared), None, c(fake), 1 << 20,
                                  None) == 10
    # Hkv_s != Hkv_t is on the tensor-core path: this one fails later, on the
    # workspace (16 bytes)
    mixed = (_lib.LKLGroupItem * 1)(item(Hkv_t=4))
    assert L.lkl_backward_grouped(1, mixed, None, ctypes.byref(shared), None, c(fake), 16,
                                  None) == 6
    assert L.lkl_forward_grouped(0, one, None, ctypes.byref(shared), c(fake), c(fake), 1 << 20,
                                 None) == 2
    assert L.lkl_forward_grouped(1, one, None, ctypes.byref(shared), c(fake), c(fake), 16,
                                 None) == 6


def _plan(p, ws=None, fused=1, mask=0):
    L = _lib.lib()
    if ws is None:
        ws = L.lkl_backward_workspace_size(ctypes.byref(p), mask)
    n = ctypes.c_int32(-1)
    st = L.lkl_backward_plan(ctypes.byref(p), mask, ws, fused, ctypes.byref(n))
    return st, n.value


def test_backward_plan_chunks():
    """The chunk planner of the tensor-core backward, host-only."""
    L = _lib.lib()
    # everything fits: one chunk
    assert _plan(_prob(Hkv_t=2)) == (0, 1)
    # LLaMA3-8B at 32K with the default workspace: Q/Q 32 heads -> 5 chunks, K/K 8 -> 2
    qq = _prob(B=1, Hq=32, Hkv_s=32, Hkv_t=32, T=32768)
    kk = _prob(B=1, Hq=8, Hkv_s=8, Hkv_t=8, T=32768)
    assert _plan(qq) == (0, 5) and _plan(kk) == (0, 2)
    # a workspace for two kv groups' tiles: ceil(4 groups / 2) chunks (Hq 4, Hkv 4)
    p = _prob(Hq=4, Hkv_s=4, Hkv_t=4, T=1300)
    n_t = (1300 + 127) // 128
    base = L.lkl_workspace_size(ctypes.byref(p), 0)
    per_head = n_t * (n_t + 1) // 2 * 32768
    assert _plan(p, base + 2 * per_head) == (0, 2)
    # less than one group: query-tile ranges of one group at a time (more chunks)
    st, n = _plan(p, base + per_head // 3)
    assert st == 0 and n > 4
    # below one query-tile row of tiles: refused
    assert _plan(p, base + (n_t - 1) * 32768)[0] == 6
    # the CUDA-core shapes have no D buffer and no chunks
    assert _plan(_prob(Ds=256, Dt=256)) == (0, 0)
