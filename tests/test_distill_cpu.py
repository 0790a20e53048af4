"""The distillation driver's plumbing without a GPU: the registered attention
function records every layer's q/k/v as the (non-contiguous) views the
attention layer produced, and LoRA wraps exactly q/k/v with a zero B."""
import pytest
import torch

transformers = pytest.importorskip("transformers")

from linearard_b200 import distill  # noqa: E402


def test_capture_and_lora_on_a_tiny_model():
    a = distill.parse([])
    a.layers, a.hidden, a.heads, a.intermediate, a.vocab, a.seq = 2, 64, 2, 128, 100, 32
    teacher, student, lora = distill.build_models(a, torch.device("cpu"), seed=0)
    assert len(lora) == a.layers * 3 * 2            # A and B of q, k, v per layer
    assert all(p.requires_grad for p in lora)
    assert sum(p.requires_grad for p in student.parameters()) == len(lora)
    assert not any(p.requires_grad for p in teacher.parameters())
    for m in student.modules():
        if isinstance(m, distill.LoRALinear):
            assert torch.count_nonzero(m.lora_B) == 0 and m.scale == a.lora_alpha / a.lora_r
    ids = torch.randint(0, a.vocab, (1, a.seq))
    with torch.no_grad(), distill.Capture() as c:
        student(input_ids=ids, use_cache=False)
    assert sorted(c.q) == [0, 1]
    q = c.q[0]
    assert q.shape == (1, a.heads, a.seq, a.hidden // a.heads)
    assert not q.is_contiguous() and q.stride(-1) == 1      # the hook keeps the views
    assert distill._ACTIVE is None
    # teacher and student share base weights but not the RoPE scaling
    assert student.rotary_emb.config.rope_parameters["rope_type"] == "linear"
    assert teacher.rotary_emb.config.rope_parameters["rope_type"] == "default"
