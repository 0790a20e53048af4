"""The numpy oracle against fixtures produced by LinearARD's own materialised
oracles (reference_lse / reference_kl / reference_grad and the
integration.py:102-127 autograd formulation).  CPU only."""
import numpy as np
import pytest

import cases as C
from oracle import attn_kl_oracle as O


@pytest.mark.parametrize("case", C.lse_cases(), ids=lambda c: c.name)
def test_oracle_lse_matches_reference(case, golden):
    q, k, mask = C.make_lse_inputs(case)
    assert C.digest(q, k, mask) == str(golden[f"{case.name}/digest"]), "input generator drifted"
    lse = O.oracle_lse(C.to_np(q), C.to_np(k), C.to_np(mask), case.causal, C.sm_scale(case.D))
    np.testing.assert_allclose(lse, golden[f"{case.name}/lse"], rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("case", C.kl_cases(), ids=lambda c: c.name)
def test_oracle_kl_and_grad_match_reference(case, golden):
    qs, ks, qt, kt, mask = C.make_kl_inputs(case)
    assert C.digest(qs, ks, qt, kt, mask) == str(golden[f"{case.name}/digest"])
    a = [C.to_np(x) for x in (qs, ks, qt, kt, mask)]
    sc_s, sc_t = C.sm_scale(case.Ds), C.sm_scale(case.Dt)
    loss, lse_s, lse_t = O.oracle_attn_kl_align(*a[:4], a[4], case.causal, sc_s, sc_t)
    np.testing.assert_allclose(lse_s, golden[f"{case.name}/lse_s"], rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(lse_t, golden[f"{case.name}/lse_t"], rtol=2e-5, atol=2e-5)
    ref_kl = float(golden[f"{case.name}/kl"])
    assert abs(loss - ref_kl) <= 1e-4 * max(1.0, abs(ref_kl)), (loss, ref_kl)
    dq, dk = O.oracle_grad(*a[:2], lse_s, *a[2:4], lse_t, a[4], case.causal, sc_s, sc_t)
    for got, key in ((dq, "dq"), (dk, "dk")):
        ref = golden[f"{case.name}/{key}"]
        scale = max(1e-6, float(np.abs(ref).max()))
        assert np.abs(got - ref).max() <= 1e-4 * scale, key


def test_oracle_cfg1_matches_reference_and_autograd(golden):
    from linearard_b200.synth import CONFIGS, make_relations
    cfg = CONFIGS["cfg1_cpu_check"]
    student, teacher = make_relations(cfg)["q"]
    assert C.digest(student, teacher) == str(golden["cfg1/digest"])
    s, t = C.to_np(student), C.to_np(teacher)
    loss, lse_s, lse_t = O.oracle_attn_kl_align(s, s, t, t)
    assert abs(loss - float(golden["cfg1/kl"])) < 1e-4
    assert abs(loss - float(golden["cfg1/loss_autograd"])) < 1e-4
    # mean over rows, as the CPU-check configuration states it
    assert abs(loss / cfg.seq_len - 0.087692) < 1e-6
    dq, dk = O.oracle_attn_kl_align_backward(s, s, t, t)
    g = dq + dk
    ref = golden["cfg1/grad_autograd"]
    cos = float((g * ref).sum() / np.sqrt((g * g).sum() * (ref * ref).sum()))
    assert cos > 0.99999
    assert np.abs(g - ref).max() <= 1e-4 * np.abs(ref).max()
    np.testing.assert_allclose(g, golden["cfg1/dq_plus_dk"], rtol=1e-3, atol=1e-6)


def test_oracle_empty_rows_and_masked_rows():
    """Rows removed by the padding mask give lse 0, KL 0 and zero gradient."""
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 2, 6, 8)); k = rng.standard_normal((1, 2, 6, 8))
    mask = np.array([[1, 1, 0, 1, 0, 0]])
    lse = O.oracle_lse(q, k, mask, True)
    assert np.all(lse[0, :, [2, 4, 5]] == 0.0)
    rows = O.kl_per_row(q, k, lse, q * 1.1, k, lse, mask, True)
    assert np.all(rows[0, :, [2, 4, 5]] == 0.0)
    dq, dk = O.oracle_grad(q, k, lse, q * 1.1, k, O.oracle_lse(q * 1.1, k, mask, True), mask, True)
    assert np.all(dq[0, :, [2, 4, 5]] == 0.0) and np.all(dk[0, :, [2, 4, 5]] == 0.0)


# ---------------------------------------------------------------- row-blocked oracle
from oracle import attn_kl_blocked as OB  # noqa: E402


def _blocked_vs_dense(qs, ks, qt, kt, mask, causal, block):
    a = (qs, ks, qt, kt)
    loss, lse_s, lse_t = O.oracle_attn_kl_align(*a, mask, causal)
    dq, dk = O.oracle_grad(qs, ks, lse_s, qt, kt, lse_t, mask, causal)
    r = OB.blocked_attn_kl(*a, mask=mask, causal=causal, block=block, threads=3)
    assert abs(r["loss"] - loss) <= 1e-10 * max(1.0, abs(loss))
    np.testing.assert_allclose(r["lse_s"], lse_s, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(r["lse_t"], lse_t, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(r["kl_rows"], O.kl_per_row(qs, ks, lse_s, qt, kt, lse_t, mask,
                                                         causal), rtol=1e-9, atol=1e-12)
    np.testing.assert_allclose(r["dq"], dq, rtol=1e-9, atol=1e-12)
    np.testing.assert_allclose(r["dk"], dk, rtol=1e-9, atol=1e-12)


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("masked", [False, True])
@pytest.mark.parametrize("shape", [(2, 4, 2, 4, 203, 32, 16), (1, 6, 3, 1, 130, 16, 16)])
def test_blocked_oracle_matches_dense(shape, masked, causal):
    """GQA with different student / teacher kv groupings, Ds != Dt, ragged T
    (blocks of 64 rows, last block partial), masks with padded heads/tails."""
    B, Hq, Hkv_s, Hkv_t, T, Ds, Dt = shape
    rng = np.random.default_rng(hash(shape) % 1000)
    qs = rng.standard_normal((B, Hq, T, Ds)); ks = rng.standard_normal((B, Hkv_s, T, Ds))
    qt = rng.standard_normal((B, Hq, T, Dt)); kt = rng.standard_normal((B, Hkv_t, T, Dt))
    mask = None
    if masked:
        mask = (rng.random((B, T)) > 0.3).astype(np.int32)
        mask[:, 0] = 0          # a padded first token: row 0 has no valid column
        mask[:, -5:] = 0        # padded tail
    _blocked_vs_dense(qs, ks, qt, kt, mask, causal, block=64)


def test_blocked_oracle_matches_reference_golden(golden):
    """The reference-generated fixtures, through the blocked evaluation."""
    for case in C.kl_cases()[:6]:
        qs, ks, qt, kt, mask = C.make_kl_inputs(case)
        a = [C.to_np(x) for x in (qs, ks, qt, kt, mask)]
        r = OB.blocked_attn_kl(*a[:4], mask=a[4], causal=case.causal,
                               sm_scale_s=C.sm_scale(case.Ds), sm_scale_t=C.sm_scale(case.Dt),
                               block=48, threads=2)
        ref_kl = float(golden[f"{case.name}/kl"])
        assert abs(r["loss"] - ref_kl) <= 1e-4 * max(1.0, abs(ref_kl)), case.name
        for key in ("dq", "dk"):
            ref = golden[f"{case.name}/{key}"]
            assert np.abs(r[key] - ref).max() <= 1e-4 * max(1e-6, float(np.abs(ref).max()))
    from linearard_b200.synth import CONFIGS, make_relations
    student, teacher = make_relations(CONFIGS["cfg1_cpu_check"])["q"]
    s, t = C.to_np(student), C.to_np(teacher)
    r = OB.blocked_attn_kl(s, s, t, t, block=100, threads=2)
    assert abs(r["loss"] - float(golden["cfg1/kl"])) < 1e-4
    g = r["dq"] + r["dk"]
    ref = golden["cfg1/grad_autograd"]
    assert np.abs(g - ref).max() <= 1e-4 * np.abs(ref).max()
