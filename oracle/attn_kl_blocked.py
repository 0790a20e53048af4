"""Row-blocked float64 oracle for the attention-relation KL loss at full length.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this module:
only ``tests/`` use it, as the checker of the CUDA kernels at the sequence
lengths the benchmark configurations are quoted on (n = 8192 and 32768), where
the dense oracle in ``attn_kl_oracle.py`` would need several n x n float64
maps (8 GiB each at n = 32768).

It is the same materialised formulation, evaluated one block of query rows at
a time so that only a [rows, n] slice of each map exists (paths are inside the
LinearARD project):

* scores ``s = scale * q . k`` with the kv head of query head h being
  ``h // (Hq / Hkv)`` (``kernels/attention_KL/test_kernel_A.py:69-72``);
* valid (i, j): row and column unmasked and, when causal, ``j <= i``
  (``test_kernel_A.py:74-86``);
* ``lse_i = log sum_j e^{s_ij}`` over valid j, ``-inf`` for rows with no valid
  column, 0 for rows the padding mask removes (``test_kernel_A.py:88-98``,
  ``kernel_A.py:146-158``);
* ``KL_i = sum_j pt_ij (log pt_ij - log ps_ij)`` with ``log p = s - lse``
  (``test_kernel_B.py:93-104``);
* ``D = ps - pt`` on valid entries of rows with finite LSEs, ``dq = scale D
  ks`` and ``dk = scale D^T qs`` summed over the query heads of each kv head
  (``test_kernel_C.py:64-117``).

A row block needs only the key columns up to its last row when causal, and its
LSEs are complete within the block (every column of a row is in its slice), so
one pass per block yields LSEs, row KLs, dq rows and that block's share of dk.
Blocks run on a thread pool (numpy releases the GIL inside matmul and ufuncs),
with one BLAS thread per worker.

``tests/test_oracle.py`` checks this module against the dense oracle and the
reference-generated golden fixtures at small sizes.
"""
from __future__ import annotations

import os
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np

__all__ = ["blocked_attn_kl"]


def _kv_of(hq: int, hkv: int, h: int) -> int:
    return h // (hq // hkv)


def blocked_attn_kl(qs, ks, qt, kt, mask=None, causal=True, sm_scale_s=None,
                    sm_scale_t=None, grad=True, block=256, threads=None):
    """Loss, LSEs, row KLs and (optionally) gradients of the KL sum.

    Inputs are ``[B, H, T, D]`` arrays of any float dtype (converted to
    float64 one block at a time); ``mask`` is ``[B, T]`` (nonzero = valid) or
    None.  Returns a dict with ``loss`` (float), ``lse_s``, ``lse_t``,
    ``kl_rows`` (``[B, Hq, T]``) and, when ``grad``, ``dq`` ``[B, Hq, T, Ds]``
    and ``dk`` ``[B, Hkv_s, T, Ds]`` (float64)."""
    qs, ks, qt, kt = (np.asarray(a) for a in (qs, ks, qt, kt))
    B, Hq, T, Ds = qs.shape
    Hkv_s, Hkv_t, Dt = ks.shape[1], kt.shape[1], qt.shape[3]
    sc_s = 1.0 / np.sqrt(Ds) if sm_scale_s is None else float(sm_scale_s)
    sc_t = 1.0 / np.sqrt(Dt) if sm_scale_t is None else float(sm_scale_t)
    mvalid = None if mask is None else (np.asarray(mask) != 0)

    lse_s = np.zeros((B, Hq, T))
    lse_t = np.zeros((B, Hq, T))
    kl_rows = np.zeros((B, Hq, T))
    dq = np.zeros((B, Hq, T, Ds)) if grad else None
    dk = np.zeros((B, Hkv_s, T, Ds)) if grad else None
    dk_locks = [[threading.Lock() for _ in range(Hkv_s)] for _ in range(B)]

    def run(b, h, r0):
        r1 = min(r0 + block, T)
        c1 = r1 if causal else T
        hs, ht = _kv_of(Hq, Hkv_s, h), _kv_of(Hq, Hkv_t, h)
        q_s = qs[b, h, r0:r1].astype(np.float64)
        k_s = ks[b, hs, :c1].astype(np.float64)
        ss = (q_s @ k_s.T) * sc_s
        st = (qt[b, h, r0:r1].astype(np.float64) @ kt[b, ht, :c1].astype(np.float64).T) * sc_t
        valid = np.ones((r1 - r0, c1), dtype=bool)
        if causal:
            valid &= np.arange(c1)[None, :] <= np.arange(r0, r1)[:, None]
        if mvalid is not None:
            valid &= mvalid[b, None, :c1]
        row_on = np.ones(r1 - r0, dtype=bool) if mvalid is None else mvalid[b, r0:r1]

        def lse_of(s):
            sm = np.where(valid, s, -np.inf)
            mx = sm.max(axis=1)
            mx0 = np.where(np.isfinite(mx), mx, 0.0)
            with np.errstate(divide="ignore"):
                out = mx + np.log(np.exp(sm - mx0[:, None]).sum(axis=1))
            return np.where(row_on, out, 0.0)

        ls, lt = lse_of(ss), lse_of(st)
        lse_s[b, h, r0:r1] = ls
        lse_t[b, h, r0:r1] = lt
        with np.errstate(invalid="ignore", over="ignore"):
            logps = np.where(valid, ss - ls[:, None], 0.0)
            logpt = np.where(valid, st - lt[:, None], 0.0)
            pt = np.where(valid, np.exp(logpt), 0.0)
            term = np.where(valid, pt * (logpt - logps), 0.0)
        kl_rows[b, h, r0:r1] = np.where(row_on, term.sum(axis=1), 0.0)
        if not grad:
            return
        live = row_on & np.isfinite(ls) & np.isfinite(lt)
        v = valid & live[:, None]
        with np.errstate(over="ignore"):
            d = np.where(v, np.exp(np.where(v, logps, 0.0)), 0.0) - np.where(v, pt, 0.0)
        dq[b, h, r0:r1] = sc_s * (d @ k_s)
        part = sc_s * (d.T @ q_s)
        with dk_locks[b][hs]:
            dk[b, hs, :c1] += part

    jobs = [(b, h, r0) for b in range(B) for h in range(Hq) for r0 in range(0, T, block)]
    # longest blocks first (causal blocks grow with r0) so the pool ends evenly
    jobs.sort(key=lambda j: -j[2] if causal else 0)
    n_thr = threads or os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_limits
        limit = threadpool_limits(limits=1)
    except Exception:  # noqa: BLE001 -- threadpoolctl is optional
        limit = None
    try:
        with ThreadPoolExecutor(max_workers=n_thr) as ex:
            for f in [ex.submit(run, *j) for j in jobs]:
                f.result()
    finally:
        if limit is not None:
            limit.restore_original_limits()
    out = {"loss": float(kl_rows.sum()), "lse_s": lse_s, "lse_t": lse_t, "kl_rows": kl_rows}
    if grad:
        out["dq"], out["dk"] = dq, dk
    return out
