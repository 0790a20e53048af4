"""Shared helpers for the GPU parity tests."""
import numpy as np

from linearard_b200 import _lib

# LinearARD's own tolerances for dq/dk (test_kernel_C.py:348-356)
REF_TOL = {"fp16": (1e-2, 2e-2), "bf16": (2e-2, 3e-2)}


def path_is_tensor_core() -> bool:
    return _lib.lib().lkl_last_path() == 1


class force_generic:
    """Context manager: route lkl_forward / lkl_backward to the CUDA-core kernels."""

    def __init__(self, on=True):
        self.on = on

    def __enter__(self):
        _lib.lib().lkl_set_force_generic(1 if self.on else 0)

    def __exit__(self, *a):
        _lib.lib().lkl_set_force_generic(0)


def grad_metrics(got, ref):
    got = np.asarray(got, dtype=np.float64).ravel()
    ref = np.asarray(ref, dtype=np.float64).ravel()
    denom = np.sqrt((got * got).sum() * (ref * ref).sum())
    cos = float((got * ref).sum() / denom) if denom > 0 else (1.0 if np.abs(got).max() == 0 else 0.0)
    scale = float(np.abs(ref).max())
    rel = float(np.abs(got - ref).max() / scale) if scale > 0 else float(np.abs(got).max())
    return cos, rel


def assert_grad_close(got, ref, name="grad", cos_min=0.999, rel_max=2e-2):
    """Parity bar for gradients: cosine >= 0.999 and max|a-b|/max|b| <= 2e-2."""
    cos, rel = grad_metrics(got, ref)
    assert cos >= cos_min and rel <= rel_max, f"{name}: cosine {cos:.6f}, max rel err {rel:.3e}"


def assert_loss_close(got, ref, rel=1e-3, abs_=1e-3, name="loss"):
    """Parity bar for losses: relative error <= 1e-3 (plus a small absolute floor
    for near-zero sums)."""
    assert abs(got - ref) <= rel * abs(ref) + abs_, f"{name}: {got} vs {ref}"


def check_device_status():
    st = _lib.lib().lkl_device_status()
    assert st == 0, f"device status {_lib.STATUS.get(st)}"


def cuda(t):
    return None if t is None else t.cuda()
