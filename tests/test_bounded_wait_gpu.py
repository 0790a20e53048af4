"""The device-side bounded wait runs out and returns, instead of hanging.

Every mbarrier wait in the tensor-core kernels gives up after a time limit,
sets the device error word and lets the kernel return.  lkl_selftest_bounded_wait
runs that same wait on a barrier that nothing ever completes, with a short
limit; the host then reads LKL_ERR_DEVICE_TIMEOUT from lkl_device_status, and
the context stays usable for the next normal call.  No GPU fault is involved.
"""
import ctypes
import time

import pytest
import torch

from linearard_b200 import _lib

LKL_ERR_DEVICE_TIMEOUT = 9


def test_probe_rejects_bad_limits_before_device_work():
    L = _lib.lib()
    assert L.lkl_selftest_bounded_wait(0, None) == 2
    assert L.lkl_selftest_bounded_wait(2_000_001, None) == 2


@pytest.mark.gpu
def test_bounded_wait_times_out_and_the_context_survives():
    from linearard_b200.attention_KL import attn_kl_forward
    L = _lib.lib()
    torch.cuda.synchronize()
    assert L.lkl_device_status() == 0
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    t0 = time.perf_counter()
    assert L.lkl_selftest_bounded_wait(20_000, stream) == 0     # 20 ms limit
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert waited >= 0.02, waited          # it really waited for the limit
    assert waited < 5.0, waited            # and then gave up
    assert L.lkl_device_status() == LKL_ERR_DEVICE_TIMEOUT
    assert L.lkl_device_status() == 0      # read-and-clear
    # the next normal call runs and reports no device error
    g = torch.Generator(device="cuda").manual_seed(3)
    s = torch.randn(1, 2, 300, 128, device="cuda", generator=g).bfloat16()
    t = (s.float() + 0.1 * torch.randn(s.shape, device="cuda", generator=g)).bfloat16()
    loss, _, _ = attn_kl_forward(s, s, t, t)
    torch.cuda.synchronize()
    assert float(loss) > 0
    assert L.lkl_device_status() == 0
