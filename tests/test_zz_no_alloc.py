"""The allocation-free scan backward (tp_scan_bwd_noalloc) against the regular
entry point (tp_scan_bwd with a caller-provided workspace).

tp_scan_bwd_noalloc exists for callers that cannot allocate device memory
themselves -- a thin FFI layer that only forwards pointers of buffers another
runtime owns, or a process whose device memory belongs to another framework's
pool.  It keeps its partial sums in a fixed array inside the library instead.
This file is collected last so that a run stopping at the first failure has
already run every other test; it also passes when run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_LANES = 262144  # B*C limit documented in include/tropical_b200.h


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _inputs(B, T, C, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    a = -torch.rand(C, device=dev, generator=g)
    b = 0.1 * torch.randn(B, T, C, device=dev, generator=g)
    x = torch.randn(B, T, C, device=dev, generator=g)
    gh = torch.randn(B, T, C, device=dev, generator=g)
    h0 = torch.randn(B, C, device=dev, generator=g)
    return a, b, x, gh, h0


def _backward(lib, noalloc, B, T, C, gh, b, x, a, h0, h, mask, stream):
    gu = torch.full_like(gh, float("nan"))
    ga = torch.full((C,), float("nan"), device=gh.device)
    gh0 = torch.full((B, C), float("nan"), device=gh.device)
    if noalloc:
        st = lib.tp_scan_bwd_noalloc(B, T, C, _p(gh), _p(b), _p(x), _p(a), 0.0, _p(h0), _p(h),
                                     _p(mask), _p(gu), _p(ga), _p(gh0), stream)
    else:
        ws = torch.empty(B, C, device=gh.device)
        st = lib.tp_scan_bwd(B, T, C, _p(gh), _p(b), _p(x), _p(a), 0.0, _p(h0), _p(h),
                             _p(mask), _p(gu), _p(ga), _p(gh0), _p(ws), stream)
    assert st == 0, lib.tp_status_string(st).decode()
    return gu, ga, gh0


@pytest.mark.parametrize("use_mask", [False, True])
def test_noalloc_matches_workspace_entry_point_twice(cuda, use_mask):
    from mk_iii_technologies_tsrn_b200 import _lib, ops
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    # calls in a row with different shapes: each must not see the previous
    # call's leftovers in the shared array.  C % 4 == 0 runs the TMA backward
    # kernel, C = 33 the plain-load kernel; both write the array.
    for seed, (B, T, C) in enumerate([(6, 300, 96), (3, 129, 40), (5, 77, 33)]):
        a, b, x, gh, h0 = _inputs(B, T, C, seed, cuda)
        h, mask = ops.scan_forward(b, x, a, 0.0, h0, need_mask=True)
        kw = (None, None, None, mask) if use_mask else (b, x, h, None)
        ref = _backward(lib, False, B, T, C, gh, kw[0], kw[1], a, h0, kw[2], kw[3], stream)
        got = _backward(lib, True, B, T, C, gh, kw[0], kw[1], a, h0, kw[2], kw[3], stream)
        torch.cuda.synchronize()
        for r, o in zip(ref, got):
            np.testing.assert_array_equal(o.cpu().numpy(), r.cpu().numpy())
    assert lib.tp_device_error(0) == 0


def test_noalloc_rejects_oversize(cuda):
    from mk_iii_technologies_tsrn_b200 import _lib
    lib = _lib.load()
    B, T, C = 2, 4, MAX_LANES // 2 + 32      # B*C over the limit
    gh = torch.zeros(1, device=cuda)
    ga = torch.zeros(1, device=cuda)
    st = lib.tp_scan_bwd_noalloc(B, T, C, _p(gh), _p(gh), None, _p(gh), 0.0, None, _p(gh),
                                 None, _p(gh), _p(ga), None, None)
    assert st == -5  # TP_ERR_TOO_LARGE, nothing launched
    assert "limit" in lib.tp_status_string(st).decode()
