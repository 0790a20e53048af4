"""AttnKLAlignFn / attn_kl_align end to end on a B200 (autograd included),
against the numpy oracle and LinearARD's golden CPU-check values, plus
size-independent properties at the benchmark sizes."""
import numpy as np
import pytest
import torch

import cases as C
from gpu_util import (assert_grad_close, assert_loss_close, check_device_status, force_generic,
                      path_is_tensor_core)
from oracle import attn_kl_oracle as O

pytestmark = pytest.mark.gpu


def _rand(shape, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g).to(dtype)


@pytest.mark.parametrize("shared", [True, False], ids=["qs_is_ks", "separate"])
@pytest.mark.parametrize("D", [64, 128, 32])
def test_attn_kl_align_autograd_vs_oracle(shared, D):
    from linearard_b200 import attn_kl_align
    B, H, T = 1, 2, 200
    qs = _rand((B, H, T, D), 1).cuda().requires_grad_(True)
    ks = qs if shared else _rand((B, H, T, D), 2).cuda().requires_grad_(True)
    qt = _rand((B, H, T, D), 3).cuda()
    kt = qt if shared else _rand((B, H, T, D), 4).cuda()
    loss = attn_kl_align(qs, ks, qt, kt)
    (2.5 * loss).backward()
    torch.cuda.synchronize()
    check_device_status()
    a = [C.to_np(x.detach()) for x in (qs, ks, qt, kt)]
    ref_loss, _, _ = O.oracle_attn_kl_align(*a)
    assert_loss_close(float(loss), ref_loss)
    dq, dk = O.oracle_attn_kl_align_backward(*a, dloss=2.5)
    if shared:
        assert_grad_close(qs.grad.float().cpu().numpy(), dq + dk, "dS")
    else:
        assert_grad_close(qs.grad.float().cpu().numpy(), dq, "dqs")
        assert_grad_close(ks.grad.float().cpu().numpy(), dk, "dks")
    assert qt.grad is None


def test_cfg1_against_reference_golden(golden):
    """The CPU-check configuration (one Q/Q head, n=512, d=64, RoPE, student at pos/8).
    The reference computes it in fp32; the kernels take fp16 inputs, so the
    comparison is tight against the oracle on the rounded inputs and loose
    against the fp32 golden."""
    from linearard_b200 import attn_kl_align
    from linearard_b200.synth import CONFIGS, make_relations
    cfg = CONFIGS["cfg1_cpu_check"]
    student, teacher = make_relations(cfg)["q"]
    s16, t16 = student.half(), teacher.half()
    s = s16.cuda().requires_grad_(True)
    t = t16.cuda()
    loss = attn_kl_align(s, s, t, t)
    loss.backward()
    torch.cuda.synchronize()
    a, b = C.to_np(s16), C.to_np(t16)
    ref, _, _ = O.oracle_attn_kl_align(a, a, b, b)
    assert_loss_close(float(loss), ref)
    dq, dk = O.oracle_attn_kl_align_backward(a, a, b, b)
    assert_grad_close(s.grad.float().cpu().numpy(), dq + dk, "dS")
    assert abs(float(loss) - float(golden["cfg1/kl"])) < 0.02 * float(golden["cfg1/kl"])
    assert_grad_close(s.grad.float().cpu().numpy(), golden["cfg1/grad_autograd"], "dS-golden",
                      cos_min=0.99, rel_max=0.1)


def test_attn_mask_and_dloss_chain_rule():
    from linearard_b200 import attn_kl_align
    B, H, T, D = 2, 4, 257, 128
    qs = _rand((B, H, T, D), 11).cuda().requires_grad_(True)
    qt = _rand((B, H, T, D), 12).cuda()
    mask = torch.ones(B, T, dtype=torch.int64)
    mask[0, 200:] = 0
    mask[1, ::3] = 0
    mask[1, 0] = 1
    loss = attn_kl_align(qs, qs, qt, qt, attn_mask=mask)
    g = torch.autograd.grad(loss * -0.75, qs)[0]
    a, b = C.to_np(qs.detach()), C.to_np(qt)
    m = mask.numpy()
    ref, _, _ = O.oracle_attn_kl_align(a, a, b, b, m)
    assert_loss_close(float(loss), ref)
    dq, dk = O.oracle_attn_kl_align_backward(a, a, b, b, m, dloss=-0.75)
    assert_grad_close(g.float().cpu().numpy(), dq + dk, "dS")


def test_identical_student_teacher_gives_zero():
    """KL(p||p) = 0 and zero gradient, at a multi-tile length."""
    from linearard_b200 import attn_kl_align
    x = _rand((1, 4, 1000, 128), 21).cuda()
    s = x.clone().requires_grad_(True)
    loss = attn_kl_align(s, s, x, x)
    loss.backward()
    assert abs(float(loss)) < 1e-2
    assert float(s.grad.abs().max()) < 1e-3


def test_backward_from_a_fresh_host_thread():
    """PyTorch runs backward on its own worker thread, which may have no
    current CUDA context; every entry point binds the device of its inputs
    itself (the tensor-map encoder needs a current context)."""
    import threading
    from linearard_b200.attention_KL import attn_kl_forward, kl_backward
    s = _rand((1, 4, 300, 128), 31).cuda()
    t = _rand((1, 4, 300, 128), 32).cuda()
    loss, ls, lt = attn_kl_forward(s, s, t, t)
    ref, _ = kl_backward(s, s, ls, t, t, lt, fused=True)
    out = {}

    def worker():
        try:
            out["dS"], _ = kl_backward(s, s, ls, t, t, lt, fused=True)
            out["path"] = path_is_tensor_core()
            torch.cuda.synchronize()
        except Exception as e:  # noqa: BLE001
            out["err"] = e

    th = threading.Thread(target=worker)
    th.start()
    th.join()
    assert "err" not in out, out.get("err")
    assert out["path"]
    torch.testing.assert_close(out["dS"], ref, rtol=0, atol=0)
