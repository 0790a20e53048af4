"""Drop-in replacement for LinearARD's ``kernels.attention_KL`` package.

``from linearard_b200.attention_KL.integration import attn_kl_align`` replaces
``from kernels.attention_KL.integration import attn_kl_align``.
"""
from .integration import AttnKLAlignFn, attn_kl_align, attn_kl_forward
from .kernel_A import lse_stats, lse_stats_triton
from .kernel_B import kl_forward, kl_forward_triton
from .kernel_C import kl_backward, kl_backward_triton
from ._common import SUPPORTED_HEAD_DIMS
from .strided import attn_kl_align_strided
from .grouped import attn_kl_align_grouped

__all__ = ["AttnKLAlignFn", "attn_kl_align", "attn_kl_forward", "lse_stats", "kl_forward",
           "kl_backward", "lse_stats_triton", "kl_forward_triton", "kl_backward_triton",
           "SUPPORTED_HEAD_DIMS", "attn_kl_align_strided", "attn_kl_align_grouped"]
