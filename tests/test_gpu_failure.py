"""Device-side failure detection without a GPU fault.

Every wait inside the library's kernels is bounded; a wait that runs out
records a code in the device error word and the kernel returns.  These tests
make a wait run out on purpose -- an mbarrier phase that gets one of its two
arrivals, a flag word that nothing sets -- with a 1 ms budget, and check that
the kernel returned, that the word holds the right code, that the Python layer
raises, and that the context still computes correctly afterwards.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("kind,code", [(0, 1), (1, 2)])
def test_timed_out_wait_is_reported_and_raises(cuda, kind, code):
    from mk_iii_technologies_tsrn_b200 import _lib, ops
    lib = _lib.load()
    flag = torch.zeros(4, dtype=torch.int32, device=cuda)    # nothing ever sets it
    prev = ops.set_wait_budget(1e-3)
    try:
        assert prev == pytest.approx(2.0)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        st = lib.tp_selftest_bounded_wait(kind, ctypes.c_void_p(flag.data_ptr()) if kind else None,
                                          _stream())
        assert st == 0, lib.tp_status_string(st)
        torch.cuda.synchronize()                # the kernel returned by itself
        assert time.perf_counter() - t0 < 1.0   # after ~1 ms, far below the 2 s default
        assert lib.tp_device_error(0) == code
        with pytest.raises(ops.DeviceWaitTimeout):
            ops.check_device_error(cuda)
        assert lib.tp_device_error(0) == 0      # check_device_error cleared it
    finally:
        ops.set_wait_budget(prev)
    # the context is still usable: a TMA GEMM with argmax afterwards is exact
    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn(256, 128, device=cuda, generator=g)
    w = torch.randn(2048, 128, device=cuda, generator=g)
    y, am = ops.maxplus(x, w)
    ry, ri = oracle.maxplus_fwd(x.cpu().numpy(), w.cpu().numpy())
    np.testing.assert_array_equal(y.cpu().numpy(), ry)
    np.testing.assert_array_equal(am.cpu().numpy(), ri)


def test_first_code_is_kept(cuda):
    """Two timed-out waits in a row: the word keeps the first code."""
    from mk_iii_technologies_tsrn_b200 import _lib, ops
    lib = _lib.load()
    flag = torch.zeros(1, dtype=torch.int32, device=cuda)
    prev = ops.set_wait_budget(1e-3)
    try:
        assert lib.tp_selftest_bounded_wait(1, ctypes.c_void_p(flag.data_ptr()), _stream()) == 0
        assert lib.tp_selftest_bounded_wait(0, None, _stream()) == 0
        torch.cuda.synchronize()
        assert lib.tp_device_error(1) == 2
        assert lib.tp_device_error(0) == 0
    finally:
        ops.set_wait_budget(prev)


def test_wait_budget_bounds(cuda):
    from mk_iii_technologies_tsrn_b200 import _lib, ops
    lib = _lib.load()
    prev = ctypes.c_int64(0)
    assert lib.tp_set_wait_budget_ns(999, ctypes.byref(prev)) == -1
    assert lib.tp_set_wait_budget_ns(60_000_000_001, ctypes.byref(prev)) == -1
    with pytest.raises(RuntimeError):
        ops.set_wait_budget(0.0)
    assert ops.set_wait_budget(2.0) == pytest.approx(2.0)
