"""The distillation step of ``linearard_b200.distill`` on a B200, at a tiny
LLaMA size: its loss and LoRA gradients against the reference's materialised
PyTorch formulation of the same loss (``integration.py:102-127``, fp32) on
the same captured q/k/v, normalised as ``train.py:380-410``."""

import pytest
import torch

from gpu_util import assert_grad_close, assert_loss_close, check_device_status
from linearard_b200 import distill

pytestmark = pytest.mark.gpu


def _args(**kw):
    a = distill.parse([])
    a.layers, a.hidden, a.heads, a.intermediate, a.vocab, a.seq = 2, 512, 4, 1024, 1000, 520
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def _materialised(qs, qt, scale):
    """Sum of row KL(softmax(qt qt^T) || softmax(qs qs^T)), causal, fp32."""
    T = qs.shape[2]
    s = torch.matmul(qs.float(), qs.float().transpose(-1, -2)) * scale
    t = torch.matmul(qt.float(), qt.float().transpose(-1, -2)) * scale
    tri = torch.tril(torch.ones(T, T, dtype=torch.bool, device=qs.device))
    neg = torch.finfo(torch.float32).min
    lps = torch.log_softmax(s.masked_fill(~tri, neg), -1)
    lpt = torch.log_softmax(t.masked_fill(~tri, neg), -1)
    return (lpt.exp() * (lpt - lps)).sum()


def test_step_loss_and_lora_grads_match_materialised_reference():
    a = _args()
    dev = torch.device("cuda", 0)
    teacher, student, lora = distill.build_models(a, dev, seed=3)
    g = torch.Generator(device=dev).manual_seed(4)
    for m in student.modules():            # non-zero B so that every LoRA factor gets a gradient
        if isinstance(m, distill.LoRALinear):
            m.lora_B.data.normal_(0, 0.02, generator=g)
    ids = torch.randint(0, a.vocab, (1, a.seq), device=dev, generator=g)
    layers = list(range(a.layers))
    with torch.no_grad(), distill.Capture() as ct:
        teacher(input_ids=ids, use_cache=False)
    assert sorted(ct.q) == layers and not ct.q[0].is_contiguous()

    with distill.Capture() as cs:
        student(input_ids=ids, use_cache=False)
    loss = distill.relation_loss(cs, ct, layers)
    loss.backward()
    ours = [p.grad.float().clone() for p in lora]
    for p in lora:
        p.grad = None

    with distill.Capture() as cs2:
        student(input_ids=ids, use_cache=False)
    scale = (a.hidden // a.heads) ** -0.5
    ref = 0.0
    for l in layers:
        for s, t in ((cs2.q[l], ct.q[l]), (cs2.k[l], ct.k[l]), (cs2.v[l], ct.v[l])):
            ref = ref + _materialised(s, t, scale)
    qs = cs2.q[0]
    ref = ref / (qs.shape[0] * qs.shape[1] * qs.shape[2]) / len(layers)
    ref.backward()
    torch.cuda.synchronize()
    check_device_status()
    assert_loss_close(float(loss), float(ref))
    for i, p in enumerate(lora):
        assert_grad_close(ours[i].cpu().numpy(), p.grad.float().cpu().numpy(), f"lora[{i}]")
