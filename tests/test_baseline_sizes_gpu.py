"""Parity at the sizes the benchmark configurations are quoted on.

The CUDA kernels against the row-blocked float64 oracle (``oracle/
attn_kl_blocked.py``, the materialised formulation of LinearARD's
``test_kernel_A/B/C.py`` reference functions evaluated one row block at a
time) on the seeded synthetic inputs of:

* the LLaMA3-8B GQA relations at n = 32768 (Q/Q, K/K and V/V, RoPE theta 5e5,
  student at positions / 8) -- the headline workload;
* the LLaMA2-7B relations at n = 8192 (per-channel teacher scale, theta 1e4);
* the Mistral-7B Q/Q relation at n = 32768 (theta 1e4);
* a grouped call over items with different head counts and a padding mask.

Each relation runs whole on the GPU (every head, the default chunked backward
plan); selected heads are compared with the oracle: row LSEs, the per-head
loss (a single-head forward call) and the fused gradient dS = dq + dk of the
shared student tensor.  Tolerances: loss relative error <= 1e-3, gradient
cosine >= 0.999 and max|dS - ref| / max|ref| <= 2e-2; LSE abs <= 2e-3.
"""
import numpy as np
import pytest
import torch

from gpu_util import assert_grad_close, assert_loss_close, check_device_status, grad_metrics
from gpu_util import path_is_tensor_core
from oracle import attn_kl_oracle as O
from oracle.attn_kl_blocked import blocked_attn_kl

pytestmark = pytest.mark.gpu

LSE_ATOL = 2e-3


def _np(t):
    return t.detach().float().cpu().numpy()


def _relation_vs_oracle(s, t, heads, label, causal=True):
    """s, t: one relation's student / teacher [1, H, T, D] on the GPU."""
    from linearard_b200.attention_KL import attn_kl_forward, kl_backward
    loss, ls, lt = attn_kl_forward(s, s, t, t, None, causal)
    assert path_is_tensor_core()
    dS, _ = kl_backward(s, s, ls, t, t, lt, None, causal, fused=True)
    torch.cuda.synchronize()
    check_device_status()
    assert np.isfinite(float(loss)) and float(loss) > 0
    for h in heads:
        sh, th = s[:, h:h + 1].contiguous(), t[:, h:h + 1].contiguous()
        loss_h, _, _ = attn_kl_forward(sh, sh, th, th, None, causal)
        a, b = _np(sh), _np(th)
        ref = blocked_attn_kl(a, a, b, b, causal=causal)
        np.testing.assert_allclose(_np(ls[:, h:h + 1]), ref["lse_s"], rtol=0, atol=LSE_ATOL)
        np.testing.assert_allclose(_np(lt[:, h:h + 1]), ref["lse_t"], rtol=0, atol=LSE_ATOL)
        assert_loss_close(float(loss_h), ref["loss"], name=f"{label} head {h} loss")
        g_ref = ref["dq"] + ref["dk"]
        got = _np(dS[:, h:h + 1])
        cos, rel = grad_metrics(got, g_ref)
        print(f"{label} head {h}: loss {float(loss_h):.6f} vs {ref['loss']:.6f} "
              f"(rel {abs(float(loss_h) - ref['loss']) / abs(ref['loss']):.2e}); "
              f"dS cosine {cos:.7f}, max rel {rel:.2e}")
        assert_grad_close(got, g_ref, f"{label} head {h} dS")


@pytest.mark.parametrize("rel,heads", [("q", (0, 31)), ("k", (7,)), ("v", (0,))])
def test_llama3_8b_32k_vs_blocked_oracle(rel, heads):
    """BASELINE config 3 (the bench workload): each relation whole, heads
    compared with the oracle at n = 32768."""
    from linearard_b200.synth import CONFIGS, make_relations
    cfg = CONFIGS["llama3_8b_32k"]
    s, t = make_relations(cfg, device="cuda", seed=0)[rel]
    _relation_vs_oracle(s, t, heads, f"llama3 32K {rel.upper()}/{rel.upper()}")


def test_llama2_7b_8k_vs_blocked_oracle():
    """per-channel teacher scale, theta 1e4, n = 8192."""
    from linearard_b200.synth import CONFIGS, make_relations
    cfg = CONFIGS["llama2_7b_8k"]
    rels = make_relations(cfg, device="cuda", seed=0)
    _relation_vs_oracle(*rels["q"], (0, 17), "llama2 8K Q/Q")
    _relation_vs_oracle(*rels["v"], (5,), "llama2 8K V/V")


def test_mistral_7b_32k_vs_blocked_oracle():
    """BASELINE config 4's inputs (theta 1e4) at n = 32768, Q/Q relation."""
    from linearard_b200.synth import CONFIGS, make_relations
    cfg = CONFIGS["mistral_7b_32k"]
    s, t = make_relations(cfg, device="cuda", seed=3)["q"]
    _relation_vs_oracle(s, t, (12,), "mistral 32K Q/Q")


def test_grouped_call_vs_oracle():
    """One grouped call over three items with different head counts (a
    symmetric Q/Q item, an asymmetric GQA item with a separate student key
    tensor, and a small K/K item), a shared padding mask and dloss != 1,
    each item against the dense oracle."""
    from linearard_b200.attention_KL import attn_kl_align_grouped
    from linearard_b200.attention_KL.grouped import grouped_ok
    from linearard_b200.synth import padding_mask, relation_pair
    T, D = 700, 128
    mask = padding_mask(2, T, 0.2, seed=5, device="cuda")
    mask[:, -37:] = 0
    s1, t1 = relation_pair((2, 8, T, D), seed_teacher=11, seed_student=12, theta=1e4,
                           apply_rope=True, device="cuda")
    s2, t2 = relation_pair((2, 4, T, D), seed_teacher=13, seed_student=14, theta=1e4,
                           apply_rope=True, device="cuda")
    k2, kt2 = relation_pair((2, 2, T, D), seed_teacher=15, seed_student=16, theta=1e4,
                            apply_rope=True, device="cuda")
    s3, t3 = relation_pair((2, 2, T, D), seed_teacher=17, seed_student=18, theta=1e4,
                           apply_rope=False, device="cuda")
    a1 = s1.clone().requires_grad_(True)
    a2 = s2.clone().requires_grad_(True)
    b2 = k2.clone().requires_grad_(True)
    a3 = s3.clone().requires_grad_(True)
    items = [(a1, a1, t1, t1), (a2, b2, t2, kt2), (a3, a3, t3, t3)]
    assert grouped_ok(items)   # one grouped launch, not the per-item fallback
    losses = attn_kl_align_grouped(items, attn_mask=mask, causal=True)
    dl = torch.tensor([0.5, 2.0, -1.5], device="cuda")
    (losses * dl).sum().backward()
    torch.cuda.synchronize()
    check_device_status()
    m = _np(mask)
    refs = [
        (s1, s1, t1, t1, [a1.grad], 0.5),
        (s2, k2, t2, kt2, [a2.grad, b2.grad], 2.0),
        (s3, s3, t3, t3, [a3.grad], -1.5),
    ]
    for n, (qs, ks, qt, kt, grads, w) in enumerate(refs):
        args = [_np(x) for x in (qs, ks, qt, kt)]
        loss, lse_s, lse_t = O.oracle_attn_kl_align(*args, m, True)
        assert_loss_close(float(losses[n].detach()), loss, name=f"item {n} loss")
        dq, dk = O.oracle_grad(args[0], args[1], lse_s, args[2], args[3], lse_t, m, True)
        if len(grads) == 1:
            assert_grad_close(_np(grads[0]), w * (dq + dk), f"item {n} dS")
        else:
            assert_grad_close(_np(grads[0]), w * dq, f"item {n} dq")
            assert_grad_close(_np(grads[1]), w * dk, f"item {n} dk")
