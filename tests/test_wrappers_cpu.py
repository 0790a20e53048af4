"""The strided and grouped operators reject bad inputs with AssertionError
before any device work, as the reference wrappers do (no GPU needed)."""
import pytest
import torch

from linearard_b200.attention_KL import attn_kl_align_grouped, attn_kl_align_strided


def _t(*shape, dtype=torch.bfloat16):
    return torch.randn(*shape).to(dtype)


def test_strided_requires_tensors_on_cuda():
    q = _t(1, 2, 64, 64)
    with pytest.raises(AssertionError, match="CUDA"):
        attn_kl_align_strided(q, q, q, q)
    with pytest.raises(AssertionError, match="torch.Tensor"):
        attn_kl_align_strided(q.float().numpy(), q, q, q)


def test_grouped_requires_items_and_cuda():
    with pytest.raises(AssertionError, match="must not be empty"):
        attn_kl_align_grouped([])
    q = _t(1, 2, 64, 64)
    with pytest.raises(AssertionError, match="CUDA"):
        attn_kl_align_grouped([(q, q, q, q)])
    with pytest.raises(AssertionError, match="torch.Tensor"):
        attn_kl_align_grouped([(q.float().numpy(), q, q, q)])
