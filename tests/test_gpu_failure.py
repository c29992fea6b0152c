"""Failure detection on the GPU without a fault: a bounded cross-GPU wait runs out.

g4_selftest_peer_timeout runs the all-reduce consumers' poll of tagged exchange words (the
wait every decode step does at world > 1) on a local slot that no producer writes.  The
wait must give up after the control block's timeout, set G4_STATUS_PEER_TIMEOUT and let
the kernel return, leaving the context usable: the call returns in about the timeout, and
the device keeps working (a second self-test and an ordinary library call afterwards).
"""
import ctypes
import time

import pytest
import torch

from gemma4_b200 import _native as N

pytestmark = pytest.mark.gpu


def test_bounded_peer_wait_runs_out_and_reports():
    lib = N.lib()
    torch.cuda.set_device(0)
    st = ctypes.c_int(0)
    t0 = time.perf_counter()
    rc = lib.g4_selftest_peer_timeout(2000, ctypes.byref(st))
    dt = time.perf_counter() - t0
    assert rc == N.G4_OK, lib.g4_last_error()
    assert st.value & N.G4_STATUS_PEER_TIMEOUT
    assert dt < 2.0, dt  # 2 ms of waiting, not the default 2 s
    # the context survived: the same check again, then an ordinary tensor-core call
    st2 = ctypes.c_int(0)
    assert lib.g4_selftest_peer_timeout(1000, ctypes.byref(st2)) == N.G4_OK
    assert st2.value & N.G4_STATUS_PEER_TIMEOUT
    a = torch.randn(128, 256, device="cuda").to(torch.bfloat16)
    b = torch.randn(64, 256, device="cuda").to(torch.bfloat16)
    c = torch.zeros(128, 64, device="cuda")
    stat = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.g4_gemm_bf16(N.ptr(a), 256, N.ptr(b), 256, N.ptr(c), 64, 128, 64, 256, 1, N.ptr(stat),
                          N.stream_handle())
    assert rc == N.G4_OK
    torch.cuda.synchronize()
    assert int(stat.item()) == 0
    torch.testing.assert_close(c, a.float() @ b.float().T, rtol=1e-3, atol=1e-3)


def test_selftest_rejects_bad_arguments():
    lib = N.lib()
    st = ctypes.c_int(0)
    assert lib.g4_selftest_peer_timeout(0, ctypes.byref(st)) == N.G4_ERR_ARG
    assert lib.g4_selftest_peer_timeout(1000, None) == N.G4_ERR_ARG
