"""Generate ``reference_golden.npz`` by running LinearARD's own oracles.

Run once, in a container where the LinearARD sources are present (they are not
shipped with this repository and are not needed at test time):

    LINEARARD_REF=/path/to/LinearARD PYTHONDONTWRITEBYTECODE=1 \
        python tests/golden/make_golden.py

It imports ``kernels/attention_KL/test_kernel_{A,B,C}.py`` from the reference
checkout and calls their materialised PyTorch oracles on CPU tensors:

* ``reference_lse``  (test_kernel_A.py:62-98)
* ``reference_kl``   (test_kernel_B.py:63-106), fed with ``reference_lse``
* ``reference_grad`` (test_kernel_C.py:64-117), fed with ``reference_lse``

and, for the CPU-check configuration (one Q/Q head, n=512, d=64, fp32, RoPE theta=1e4,
student at positions/8), the loss and its autograd gradient through the
materialised softmax formulation of ``kernels/attention_KL/integration.py:102-127``.

Gradients are stored as float32 with the low 8 mantissa bits cleared
(relative error <= 2^-15, far below every tolerance used); everything else is
stored exactly.  Each case carries a SHA-256 digest of the
inputs, which the tests regenerate from the case seeds in ``cases.py``.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import cases as C  # noqa: E402
from linearard_b200.synth import CONFIGS, make_relations  # noqa: E402


def _import_reference(root: str):
    sys.dont_write_bytecode = True
    sys.path.insert(0, root)
    from kernels.attention_KL import test_kernel_A, test_kernel_B, test_kernel_C  # noqa
    return test_kernel_A.reference_lse, test_kernel_B.reference_kl, test_kernel_C.reference_grad


def _materialised_loss(qs, ks, qt, kt, mask, causal, sc_s, sc_t):
    """integration.py:102-127: full log-softmax formulation (fp32)."""
    T = qs.shape[2]
    logits_s = torch.matmul(qs, ks.transpose(-1, -2)) * sc_s
    logits_t = torch.matmul(qt, kt.transpose(-1, -2)) * sc_t
    if mask is None:
        mask = torch.ones((qs.shape[0], T), dtype=torch.int32)
    row_mask = mask[:, None, :, None].bool()
    col_mask = mask[:, None, None, :].bool()
    tri = torch.tril(torch.ones(T, T, dtype=torch.bool))[None, None]
    valid = row_mask & col_mask & (tri if causal else torch.ones_like(tri))
    neg = torch.finfo(logits_s.dtype).min
    logits_s = logits_s.masked_fill(~valid, neg)
    logits_t = logits_t.masked_fill(~valid, neg)
    rows = valid.any(dim=-1).unsqueeze(-1)
    lps = torch.where(rows, torch.log_softmax(logits_s, -1), torch.zeros_like(logits_s))
    lpt = torch.where(rows, torch.log_softmax(logits_t, -1), torch.zeros_like(logits_t))
    pt = torch.where(rows, torch.softmax(logits_t, -1), torch.zeros_like(logits_t))
    return (pt * (lpt - lps)).sum()


def _compact(a: np.ndarray) -> np.ndarray:
    """float32 with the low 8 mantissa bits cleared (relative error <= 2^-15),
    which lets the gradient arrays compress about 2x."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    return (a.view(np.uint32) & np.uint32(0xFFFFFF00)).view(np.float32)


def main():
    root = os.environ.get("LINEARARD_REF")
    if not root:
        raise SystemExit("set LINEARARD_REF to a LinearARD checkout (see the module docstring)")
    reference_lse, reference_kl, reference_grad = _import_reference(root)
    out = {}
    torch.set_num_threads(max(1, os.cpu_count() or 1))

    for c in C.lse_cases():
        q, k, mask = C.make_lse_inputs(c)
        lse = reference_lse(q, k, mask, c.causal, C.sm_scale(c.D))
        out[f"{c.name}/digest"] = np.array(C.digest(q, k, mask))
        out[f"{c.name}/lse"] = lse.float().numpy()

    for c in C.kl_cases():
        qs, ks, qt, kt, mask = C.make_kl_inputs(c)
        sc_s, sc_t = C.sm_scale(c.Ds), C.sm_scale(c.Dt)
        lse_s = reference_lse(qs, ks, mask, c.causal, sc_s)
        lse_t = reference_lse(qt, kt, mask, c.causal, sc_t)
        kl = reference_kl(qs, ks, lse_s, qt, kt, lse_t, mask, c.causal, sc_s, sc_t)
        dq, dk = reference_grad(qs, ks, lse_s, qt, kt, lse_t, mask, c.causal, sc_s, sc_t)
        out[f"{c.name}/digest"] = np.array(C.digest(qs, ks, qt, kt, mask))
        out[f"{c.name}/lse_s"] = lse_s.float().numpy()
        out[f"{c.name}/lse_t"] = lse_t.float().numpy()
        out[f"{c.name}/kl"] = np.array(float(kl), dtype=np.float64)
        out[f"{c.name}/dq"] = _compact(dq.float().numpy())
        out[f"{c.name}/dk"] = _compact(dk.float().numpy())

    # the CPU-check configuration: Q/Q relation, fp32, n=512, d=64, causal, RoPE.
    cfg = CONFIGS["cfg1_cpu_check"]
    student, teacher = make_relations(cfg, device="cpu")["q"]
    sc = C.sm_scale(cfg.head_dim)
    lse_s = reference_lse(student, student, None, True, sc)
    lse_t = reference_lse(teacher, teacher, None, True, sc)
    kl = reference_kl(student, student, lse_s, teacher, teacher, lse_t, None, True, sc, sc)
    dq, dk = reference_grad(student, student, lse_s, teacher, teacher, lse_t, None, True, sc, sc)
    s_leaf = student.clone().requires_grad_(True)
    loss = _materialised_loss(s_leaf, s_leaf, teacher, teacher, None, True, sc, sc)
    loss.backward()
    out["cfg1/digest"] = np.array(C.digest(student, teacher))
    out["cfg1/lse_s"] = lse_s.numpy()
    out["cfg1/lse_t"] = lse_t.numpy()
    out["cfg1/kl"] = np.array(float(kl), dtype=np.float64)
    out["cfg1/loss_autograd"] = np.array(float(loss), dtype=np.float64)
    out["cfg1/grad_autograd"] = s_leaf.grad.numpy()
    out["cfg1/dq_plus_dk"] = (dq + dk).numpy()

    path = os.path.join(HERE, C.FIXTURE)
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path) / 1e6:.2f} MB; "
          f"cfg1 loss sum {float(kl):.6f} (autograd {float(loss):.6f}), mean/row {float(kl) / cfg.seq_len:.6f}")


if __name__ == "__main__":
    main()
