"""Failure detection on the device without a fault: a kernel's bounded wait runs out.

Every mbarrier wait in the pipeline kernels is bounded by the context's timeout (ptx.cuh mbar_wait);
when a partner never arrives the waiting role records a timeout in the device error word and the
kernel returns, and the next synchronisation reports SDVK_E_TIMEOUT (the reference's failures are
exceptions from the engine: VK_CHECK, vk_engine.cpp:33-41; OomError, vk_engine.hpp:30-32).

sdvk_selftest_wait queues one warp waiting on an mbarrier that nothing arrives on, through that same
bounded wait.  The test sets a short timeout, checks that the status arrives within a bounded host
wait, that the error word is cleared by reading it, and that the same context then runs a Q8_0 GEMM
correctly (the context stays usable).  No trap, no bad address, no endless loop.
"""
import time

import pytest
import torch

import sdvk_b200
from sdvk_b200 import torch_ops
from tests._gpu_util import check_gemm, dev, host

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_context_recovers(cuda_ok, orc):
    torch.cuda.set_device(0)
    ctx = sdvk_b200.Context(0)
    try:
        ctx.set_timeout_ms(200)
        t0 = time.monotonic()
        ctx.selftest_wait()
        with pytest.raises(sdvk_b200.SdvkError) as ei:
            ctx.synchronize()
        dt = time.monotonic() - t0
        assert ei.value.status == sdvk_b200.E_TIMEOUT, ei.value
        assert "timed out" in str(ei.value)
        assert 0.15 <= dt < 10.0, dt  # the wait lasted about the timeout, then the kernel returned
        ctx.synchronize()  # reading the status cleared the error word
        ctx.set_timeout_ms(2000)
        # the same context, afterwards: a Q8_0 GEMM against the fp64 truth
        M, N, K = 256, 384, 640
        x = orc.normal_f16(3, 0, (M, K))
        q, _, s = orc.q8_weights(3, 1, N, K)
        X, Q, S = dev(x), dev(q), dev(s)
        C = torch.empty((M, N), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        ctx.gemm_q8_nt(X.data_ptr(), sdvk_b200.F16, Q.data_ptr(), S.data_ptr(), None, C.data_ptr(), sdvk_b200.F32, M,
                       N, K)
        ctx.synchronize()
        ref = orc.gemm_nt_q8_f64(x.astype("float32"), q, s)
        check_gemm(orc, "gemm_after_timeout", host(C), ref, "f16")
    finally:
        ctx.close()


def test_torch_stream_context_reports_timeout(cuda_ok):
    """The same on the context that follows torch's stream (the one the Python ops use)."""
    ctx = torch_ops.context(torch.device("cuda", 0))
    ctx.set_timeout_ms(100)
    try:
        ctx.selftest_wait()
        with pytest.raises(sdvk_b200.SdvkError) as ei:
            ctx.synchronize()
        assert ei.value.status == sdvk_b200.E_TIMEOUT
        ctx.synchronize()
    finally:
        ctx.set_timeout_ms(2000)
