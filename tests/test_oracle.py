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
