"""Failure detection on the GPU without a fault: every wait of the pipelined
kernels is bounded; when one runs out, the kernel records a code in the device
status word, the other roles of the CTA leave through the abort flag, and the
kernel returns with the context intact.  w4a8_selftest_wait_timeout drives
exactly that path (an mbarrier that is never completed, no TMA or MMA in
flight); the test reads the status word through the C ABI and then runs a
real GEMM on the same context."""
import ctypes
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu

SELFTEST_CODE = 120   # kDevTimeoutSelfTest


def test_expired_wait_sets_status_and_kernel_returns(pkg, cuda):
    L = importlib.import_module("flagos-kernel-gen_b200._lib")
    lib = L.load()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    assert pkg.device_status() == 0
    report = torch.full((3,), -1, dtype=torch.int32, device=cuda)
    rc = lib.w4a8_selftest_wait_timeout(200_000, report.data_ptr(), stream)   # ~0.1 ms at B200 clocks
    assert rc == L.W4A8_OK, lib.w4a8_last_error()
    st = ctypes.c_int32(-1)
    assert lib.w4a8_device_status(ctypes.byref(st), 0, stream) == L.W4A8_OK   # synchronises: the kernel returned
    assert st.value == SELFTEST_CODE
    rep = report.cpu().tolist()
    assert rep[0] == 0 and rep[1] == 0, rep   # both waits failed (neither barrier was ever completed)
    # the second role left through the abort flag long before its own ~2e9-cycle limit
    assert rep[2] < 1_000_000, rep
    assert pkg.device_status(reset=True) == SELFTEST_CODE
    assert pkg.device_status() == 0
    # the context is still usable: a grouped GEMM runs and its status is clean
    W = pkg.workloads
    x_q, xs, w, ws, wz, off = W.make_gemm_inputs(4, 64, 256, 512, 128, seed=1, device=cuda)
    out = torch.zeros((64, 256), dtype=torch.bfloat16, device=cuda)
    pkg.w4a8_group_gemm_moe(x_q, xs, w, ws, wz, off, out, 128)
    torch.cuda.synchronize()
    assert pkg.device_status() == 0
    assert torch.isfinite(out.float()).all()


def test_selftest_rejects_bad_limits(pkg, cuda):
    L = importlib.import_module("flagos-kernel-gen_b200._lib")
    lib = L.load()
    report = torch.zeros((3,), dtype=torch.int32, device=cuda)
    assert lib.w4a8_selftest_wait_timeout(0, report.data_ptr(), None) == L.W4A8_ERR_INVALID
    assert lib.w4a8_selftest_wait_timeout(1 << 40, report.data_ptr(), None) == L.W4A8_ERR_INVALID
