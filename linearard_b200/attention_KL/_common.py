"""Argument checks and C-ABI marshalling shared by the operator wrappers.

The checks and their messages follow the assertions of LinearARD's Triton
wrappers (``kernels/attention_KL/kernel_A.py:192-227``,
``kernel_B.py:262-331``, ``kernel_C.py:306-375``), so the same bad inputs fail
the same way (``AssertionError``).  No tensor math happens here: every
number is computed by ``liblinearard_b200.so``.
"""
from __future__ import annotations

import ctypes
import math

import torch

from .. import _lib

SUPPORTED_HEAD_DIMS = (8, 16, 32, 64, 128, 256)
# head dims of the sm_100a tensor-core kernels (8..32 run zero-padded to 64)
TC_HEAD_DIMS = (8, 16, 32, 64, 128)

_DT = {torch.float16: _lib.LKL_F16, torch.bfloat16: _lib.LKL_BF16}
_MASK_DT = {torch.bool: _lib.LKL_MASK_BOOL, torch.uint8: _lib.LKL_MASK_U8,
            torch.int32: _lib.LKL_MASK_I32, torch.int64: _lib.LKL_MASK_I64}


def check_pair(q, k, qn="q", kn="k"):
    assert isinstance(q, torch.Tensor), f"{qn} must be a torch.Tensor"
    assert isinstance(k, torch.Tensor), f"{kn} must be a torch.Tensor"
    assert q.is_cuda and k.is_cuda, f"{qn}/{kn} must be on CUDA"
    assert q.dtype in (torch.float16, torch.bfloat16), f"{qn} dtype supports only fp16/bf16"
    assert k.dtype in (torch.float16, torch.bfloat16), f"{kn} dtype supports only fp16/bf16"
    assert q.dtype == k.dtype, f"{qn}/{kn} dtype must match"
    assert q.ndim == 4 and k.ndim == 4, f"{qn}/{kn} shape must be [B,H,T,D]"
    assert q.shape[0] == k.shape[0], f"{qn}/{kn} B must match"
    assert q.shape[2] == k.shape[2], f"{qn}/{kn} T must match"
    assert q.shape[3] == k.shape[3], f"{qn}/{kn} D must match"
    assert q.is_contiguous() and k.is_contiguous(), f"{qn}/{kn} must be contiguous"
    assert q.stride(-1) == 1 and k.stride(-1) == 1, f"{qn}/{kn} last-dim stride must be 1"
    assert q.device == k.device, f"{qn}/{kn} must be on the same device"
    Hq, Hkv = q.shape[1], k.shape[1]
    assert Hq % Hkv == 0, "Hq must be divisible by Hkv"
    assert q.shape[3] in SUPPORTED_HEAD_DIMS, "head_dim is not in the supported set"


def check_lse(lse, shape, name="lse"):
    assert isinstance(lse, torch.Tensor), f"{name} must be a torch.Tensor"
    assert lse.is_cuda, "lse must be on CUDA"
    assert lse.ndim == 3, "lse shape must be [B,H,T]"
    assert lse.dtype == torch.float32, "lse must be float32"
    assert lse.is_contiguous(), "lse must be contiguous"
    assert tuple(lse.shape) == tuple(shape), f"{name} shape must match [B,Hq,T]"


def prepare_mask(attn_mask, B, T, device):
    """CPU masks are moved to the device (kernel_A.py:210-219); returns
    (mask tensor or None, lkl mask dtype)."""
    if attn_mask is None:
        return None, _lib.LKL_MASK_U8
    assert isinstance(attn_mask, torch.Tensor), "attn_mask must be a torch.Tensor"
    if attn_mask.device.type == "cpu":
        assert attn_mask.is_contiguous(), "attn_mask must be contiguous"
        attn_mask = attn_mask.to(device=device)
    assert attn_mask.is_cuda, "attn_mask must be on CUDA"
    assert attn_mask.ndim == 2, "attn_mask shape must be [B,T]"
    assert attn_mask.shape[0] == B and attn_mask.shape[1] == T, "attn_mask shape must be [B,T]"
    assert attn_mask.dtype in _MASK_DT, "attn_mask dtype is invalid"
    assert attn_mask.is_contiguous(), "attn_mask must be contiguous"
    assert attn_mask.stride(-1) == 1, "attn_mask last-dim stride must be 1"
    return attn_mask, _MASK_DT[attn_mask.dtype]


def scale_of(s, D, name):
    if s is None:
        s = 1.0 / math.sqrt(D)
    assert isinstance(s, (float, int)), f"{name} must be a scalar"
    return float(s)


def problem(qs, ks, qt=None, kt=None, causal=True, mask_dtype=_lib.LKL_MASK_U8,
            sm_scale_s=None, sm_scale_t=None) -> _lib.LKLProblem:
    B, Hq, T, Ds = qs.shape
    qt = qs if qt is None else qt
    kt = ks if kt is None else kt
    return _lib.LKLProblem(
        B=B, Hq=Hq, Hkv_s=ks.shape[1], Hkv_t=kt.shape[1], T=T, Ds=Ds, Dt=qt.shape[3],
        dtype_s=_DT[qs.dtype], dtype_t=_DT[qt.dtype], causal=1 if causal else 0,
        mask_dtype=mask_dtype, sm_scale_s=scale_of(sm_scale_s, Ds, "sm_scale_s"),
        sm_scale_t=scale_of(sm_scale_t, qt.shape[3], "sm_scale_t"))


def workspace(prob: _lib.LKLProblem, has_mask: bool, device, backward: bool = False):
    L = _lib.lib()
    size_fn = L.lkl_backward_workspace_size if backward else L.lkl_forward_workspace_size
    n = int(size_fn(ctypes.byref(prob), 1 if has_mask else 0))
    ws = torch.empty(max(n, 256), dtype=torch.uint8, device=device)
    return ws, n


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
