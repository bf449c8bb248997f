"""The bounded device waits of the tensor-core kernels, made to run out on
purpose without hanging or faulting a GPU.

``bozo_tension_wait_selftest`` launches one CTA that starts a bulk copy and a
tensor-core MMA, then waits on an mbarrier that nothing arrives on with a
limit of about a millisecond.  The test checks that the wait gives up, that
the device error word reports ``BOZO_ERR_DEVICE_TIMEOUT`` (synchronous poll
and the asynchronous per-step check), that the CTA drained its copy and MMA
before releasing TMEM, and that the context still runs a normal tension call
correctly afterwards.  The reference has no device-side waits; its only
timeout is the NCCL one it comments on (train.py:561-564).
"""
import ctypes as C
import math

import pytest
import torch

from oracle import tension_oracle as orc
from tests._tol import assert_close

pytestmark = pytest.mark.gpu
cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs CUDA")

DEVICE_TIMEOUT = 6
BAD_SHAPE = 1


@pytest.fixture(scope="module")
def bz():
    import bozo_b200
    bozo_b200.set_kernel_path("auto")
    return bozo_b200


def _selftest(limit_ns, result):
    from bozo_b200 import _capi
    st = torch.cuda.current_stream().cuda_stream
    return _capi.lib().bozo_tension_wait_selftest(C.c_uint64(limit_ns),
                                                  C.c_void_p(result.data_ptr() if result is not None else 0),
                                                  C.c_void_p(st))


def _poll():
    from bozo_b200 import _capi
    return _capi.lib().bozo_tension_poll_error(C.c_void_p(torch.cuda.current_stream().cuda_stream))


@cuda
def test_wait_runs_out_reports_timeout_and_drains(bz):
    assert _poll() == 0  # start clean
    res = torch.zeros(4, dtype=torch.int32, device="cuda")
    assert _selftest(1_000_000, res) == 0  # 1 ms limit
    assert _poll() == DEVICE_TIMEOUT
    gave_up, copy_ok, mma_ok, waited_us = res.cpu().tolist()
    assert gave_up == 1 and copy_ok == 1 and mma_ok == 1
    assert 1000 <= waited_us < 200_000, waited_us
    assert _poll() == 0  # the read cleared the word


@cuda
def test_context_usable_after_timeout(bz):
    assert _selftest(2_000_000, None) == 0
    torch.manual_seed(12)
    B, T, H, HD, W = 2, 200, 2, 64, 64
    q, k, v, d = [torch.randn(B, T, H, HD, dtype=torch.bfloat16) for _ in range(4)]
    qg, kg, vg = [x.cuda().requires_grad_(True) for x in (q, k, v)]
    out = bz.tension(qg, kg, vg, window=W)
    (out.float() * d.cuda().float()).sum().backward()
    assert bz.last_path() == "tcgen05"
    with pytest.raises(RuntimeError, match="timed out"):
        bz.poll_device_error()  # the self-test's timeout, reported once
    bz.poll_device_error()       # the tension call itself left the word clear

    def fn(a, b, c):
        return orc.fused_reference(a, b, c, window=W, scale=math.sqrt(HD))[0]
    (o,), grads = orc.tension_with_grads(fn, [x.double() for x in (q, k, v)], [d.double()])
    for g, r, what in zip((out, qg.grad, kg.grad, vg.grad), (o, *grads), ("out", "dq", "dk", "dv")):
        assert_close(g, r, torch.bfloat16, f"after timeout/{what}")


@cuda
def test_per_step_check_raises_one_step_late(bz):
    bz.poll_device_error()
    assert _selftest(1_000_000, None) == 0
    bz.check_device_error()          # enqueues the asynchronous read
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="timed out"):
        bz.check_device_error()      # sees the copied word, polls and raises
    bz.check_device_error()
    torch.cuda.synchronize()
    bz.check_device_error()          # clear: no exception


@cuda
def test_selftest_rejects_limits_outside_range(bz):
    assert _selftest(10, None) == BAD_SHAPE
    assert _selftest(5_000_000_000, None) == BAD_SHAPE
