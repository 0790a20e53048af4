"""B200 (sm_100a) attention-relation KL loss of LinearARD.

The compute lives in ``liblinearard_b200.so`` (C ABI, ``include/linearard_b200.h``);
this package is the PyTorch-facing mirror of LinearARD's ``kernels/attention_KL``.
"""
from .attention_KL import (AttnKLAlignFn, attn_kl_align, attn_kl_forward, kl_backward,
                           kl_forward, lse_stats)

__all__ = ["AttnKLAlignFn", "attn_kl_align", "attn_kl_forward", "lse_stats", "kl_forward",
           "kl_backward"]
__version__ = "0.1.0"
