"""The C-ABI library loads on a CPU-only host and exports every declared symbol;
host-side validation rejects bad arguments before touching a GPU."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "tropical_b200.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"TP_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared()
    for n in ("tp_maxplus_fwd", "tp_maxplus_fwd_strided", "tp_maxplus_lse_fwd_strided",
              "tp_maxplus_bwd_argmax_strided", "tp_maxplus_bwd_smooth", "tp_scan_fwd",
              "tp_scan_bwd", "maxplus_forward_cuda", "maxplus_backward_cuda",
              "maxplus_matmul_cuda"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from mk_iii_technologies_tsrn_b200 import _lib
    lib = _lib.load()
    for n in _declared():
        assert hasattr(lib, n), f"missing export {n}"
        assert n in _lib.SIGNATURES, f"no ctypes signature for {n}"


def test_no_undeclared_exports_in_signature_table():
    from mk_iii_technologies_tsrn_b200 import _lib
    assert set(_lib.SIGNATURES) == set(_declared())


def test_status_strings():
    from mk_iii_technologies_tsrn_b200 import _lib
    assert _lib.status_text(0) == "ok"
    assert "NULL" in _lib.status_text(-2)
    assert "workspace" in _lib.status_text(-7)
    assert _lib.load().tp_abi_version() == 1


def test_validation_rejects_before_launch():
    from mk_iii_technologies_tsrn_b200 import _lib
    lib = _lib.load()
    # negative sizes / bad leading dims are rejected on the host
    assert lib.tp_maxplus_fwd(0, -1, 4, 4, None, 4, None, 4, None, None, 4, None, 0, None) == -1
    assert lib.tp_maxplus_fwd(0, 4, 4, 8, None, 4, None, 8, None, None, 4, None, 0, None) == -1
    assert lib.tp_maxplus_fwd(7, 4, 4, 4, None, 4, None, 4, None, None, 4, None, 0, None) == -4
    assert lib.tp_maxplus_bwd_smooth(9, 1.0, 0, 1, 4, 4, 4, None, None, None, None, None, None,
                                     None, 0, None) == -1
    assert lib.tp_maxplus_bwd_smooth(1, 0.0, 0, 1, 4, 4, 4, None, None, None, None, None, None,
                                     None, 0, None) == -1
    assert lib.tp_scan_fwd(-1, 4, 4, None, None, None, 0.0, None, None, None, None) == -1
    # empty problems are a no-op success
    assert lib.tp_maxplus_fwd(0, 0, 4, 4, None, 4, None, 4, None, None, 4, None, 0, None) == 0
    assert lib.tp_scan_fwd(0, 4, 4, None, None, None, 0.0, None, None, None, None) == 0
    assert lib.tp_probe_addmax(10, 1, 256, 1, None, None) == -1


def test_null_pointer_rejected_without_pointer_checks():
    from mk_iii_technologies_tsrn_b200 import _lib
    lib = _lib.load()
    old = lib.tp_set_pointer_checks(0)
    try:
        st = lib.tp_maxplus_fwd(0, 4, 4, 4, None, 4, None, 4, None, None, 4, None, 0, None)
        assert st == -2
        # (B, T, C, gh, bb, xx, a, h_init, h0, h, win_mask, gu, ga, gh0, workspace, stream)
        st = lib.tp_scan_bwd(2, 4, 4, None, None, None, None, 0.0, None, None, None, None,
                             ctypes.c_void_p(16), None, None, None)
        assert st == -7   # ga requested without a workspace
    finally:
        lib.tp_set_pointer_checks(old)


def test_workspace_size():
    from mk_iii_technologies_tsrn_b200 import _lib
    lib = _lib.load()
    # six [M][N] stat planes per batch (three, and the same three transposed)
    assert lib.tp_maxplus_bwd_smooth_workspace_bytes(2, 3, 5, 7) == 2 * 6 * 3 * 5 * 4
    assert lib.tp_maxplus_bwd_smooth_workspace_bytes(-1, 3, 5, 7) == 0
    # a projection-shaped problem (M=8192 rows, N=K=256): both gradients in one
    # pass, the weight gradient's partials per 64-row tile [128][256][256]
    # (larger than the two-pass split's [32][256][256])
    stats = 6 * 8192 * 256
    assert lib.tp_maxplus_bwd_smooth_workspace_bytes(1, 8192, 256, 256) == \
        (stats + 128 * 256 * 256) * 4
    # the input gradient's 2 tiles cut into 16 slices of n: two passes, partials
    # [16][64][128]
    assert lib.tp_maxplus_bwd_smooth_workspace_bytes(1, 64, 4096, 128) == \
        (6 * 64 * 4096 + 16 * 64 * 128) * 4


def test_failure_entry_points_validate_on_the_host():
    from mk_iii_technologies_tsrn_b200 import _lib
    lib = _lib.load()
    prev = ctypes.c_int64(0)
    # out-of-range budgets and self-test kinds are rejected before any CUDA call
    assert lib.tp_set_wait_budget_ns(0, ctypes.byref(prev)) == -1
    assert lib.tp_set_wait_budget_ns(-5, None) == -1
    assert lib.tp_set_wait_budget_ns(10 ** 11, None) == -1
    assert lib.tp_selftest_bounded_wait(2, None, None) == -1
    assert lib.tp_selftest_bounded_wait(1, None, None) == -2   # kind 1 needs its flag word


def test_noalloc_checks_arguments_before_its_limit():
    from mk_iii_technologies_tsrn_b200 import _lib
    lib = _lib.load()
    big_c = 262144 // 2 + 32          # B*C over the array's limit at B = 2
    # NULL required pointers (here `a`) are reported as tp_scan_bwd reports
    # them, although ga is requested and B*C is over the limit; the checks stop
    # at the NULL before touching the (fake, never dereferenced) ga address
    fake_ga = ctypes.c_void_p(4096)
    assert lib.tp_scan_bwd_noalloc(2, 4, big_c, None, None, None, None, 0.0, None, None, None,
                                   None, fake_ga, None, None) == -2
    # negative sizes
    assert lib.tp_scan_bwd_noalloc(2, -1, 4, None, None, None, None, 0.0, None, None, None,
                                   None, None, None, None) == -1


def test_chunked_scan_validates_on_the_host():
    from mk_iii_technologies_tsrn_b200 import _lib
    lib = _lib.load()
    assert lib.tp_scan_chunked_workspace_bytes(2, 256, 64, 33) == -1
    assert lib.tp_scan_chunked_workspace_bytes(2, 256, 64, 64) > 0
    assert lib.tp_scan_chunked_workspace_bytes(0, 256, 64, 0) == 0
    # chunk lengths must be multiples of 32; negative sizes; NULL inputs
    assert lib.tp_scan_fwd_chunked(2, 64, 8, None, None, None, 0.0, None, None, None, 48,
                                   None, 0, None) == -1
    assert lib.tp_scan_fwd_chunked(-1, 64, 8, None, None, None, 0.0, None, None, None, 32,
                                   None, 0, None) == -1
    assert lib.tp_scan_fwd_chunked(2, 64, 8, None, None, None, 0.0, None, None, None, 32,
                                   None, 0, None) == -2
    assert lib.tp_scan_bwd_chunked(2, 64, 8, None, None, None, None, 0.0, None, None, None,
                                   None, None, None, 32, None, 0, None) == -2


def test_attention_path_selector_and_workspace():
    from mk_iii_technologies_tsrn_b200 import _lib
    lib = _lib.load()
    prev = ctypes.c_int(-1)
    assert lib.tp_tsrn_attention_set_path(3, None) == -1
    assert lib.tp_tsrn_attention_set_path(-1, None) == -1
    assert lib.tp_tsrn_attention_set_path(_lib.TP_ATT_PATH_CUDA_CORES, ctypes.byref(prev)) == 0
    assert prev.value == _lib.TP_ATT_PATH_AUTO
    assert lib.tp_tsrn_attention_set_path(_lib.TP_ATT_PATH_AUTO, ctypes.byref(prev)) == 0
    assert prev.value == _lib.TP_ATT_PATH_CUDA_CORES
    # the workspace covers the tensor-core kernel's padded hi/lo feature planes
    # (128-row query tiles, 64-key tiles, 96 channels) as well as the CUDA-core
    # kernel's transposed features
    B, H, T, Tkv, dh = 2, 3, 200, 260, 80
    tp, kp = 256, 320
    tc_floats = 2 * B * H * tp * 96 + 2 * B * H * kp * 96 + B * H * T + B * H * kp
    assert lib.tp_tsrn_attention_workspace_bytes(B, H, T, Tkv, dh) >= 4 * tc_floats
    cc_floats = B * H * (T + Tkv) * (dh + 1)
    assert lib.tp_tsrn_attention_workspace_bytes(1, 1, 8, 8, 128) >= 4 * 16 * 129
    assert lib.tp_tsrn_attention_workspace_bytes(B, H, T, Tkv, dh) >= 4 * cc_floats
