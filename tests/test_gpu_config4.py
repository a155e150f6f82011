"""Oracle parity of the large max-plus GEMM at the sweep sizes M = N = K in
{2048, 4096, 8192} (and a sampled 16384): x, W ~ N(0,1), 5% of W = -inf
(Bernoulli, seed 2) -- the inputs the benchmark times.

64 sampled rows x ALL columns are compared bit for bit with the oracle
(oracle.maxplus_fwd: the reference expression tropformer.py:131,141) for fp32
operands under every schedule of the TMA kernel (auto, whole tiles, even
stream-K split, k-aligned pieces), with and without argmax; for bf16 storage
(widened exactly, fp32 arithmetic) against the oracle on the upcast inputs;
and for bf16 arithmetic against the reference expression evaluated by torch
on bf16 tensors (oracle.torch_ref.maxplus_fwd_torch).
"""
import os

import numpy as np
import pytest
import torch

import oracle
from oracle.torch_ref import maxplus_fwd_torch

pytestmark = pytest.mark.gpu

_CACHE = {}


@pytest.fixture(scope="module", autouse=True)
def _free_inputs():
    yield
    _CACHE.clear()


def _inputs(S):
    if S not in _CACHE:
        _CACHE.clear()
        dev = torch.device("cuda:0")
        x = torch.randn(S, S, device=dev, generator=torch.Generator(device=dev).manual_seed(0))
        W = torch.randn(S, S, device=dev, generator=torch.Generator(device=dev).manual_seed(1))
        mask = torch.rand(S, S, device=dev,
                          generator=torch.Generator(device=dev).manual_seed(2)) < 0.05
        W[mask] = float("-inf")
        _CACHE[S] = (x, W)
    return _CACHE[S]


def _rows(S, n=64):
    rng = np.random.default_rng(S)
    edge = [0, 1, 127, 128, S // 2 - 1, S // 2, S - 129, S - 128, S - 1]
    rest = rng.choice(np.setdiff1d(np.arange(S), edge), n - len(edge), replace=False)
    return np.sort(np.concatenate([edge, rest]))


def _sample(t, rows):
    return t[torch.as_tensor(rows, device=t.device)].cpu().numpy()


@pytest.mark.parametrize("S", [2048, 4096, 8192])
def test_fp32_every_schedule(cuda, S):
    from mk_iii_technologies_tsrn_b200 import _lib, ops
    lib = _lib.load()
    x, W = _inputs(S)
    rows = _rows(S)
    ry, ri = oracle.maxplus_fwd(_sample(x, rows), W.cpu().numpy())
    old = lib.tp_set_stream_k(1)
    try:
        for mode in (1, 0, 2, 3):      # auto, whole tiles, even split, k-aligned pieces
            lib.tp_set_stream_k(mode)
            y, am = ops.maxplus(x, W)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(_sample(y, rows), ry, err_msg=f"values, mode {mode}")
            np.testing.assert_array_equal(_sample(am, rows), ri, err_msg=f"argmax, mode {mode}")
            del y, am
        for mode in (1, 2):            # value-only kernel
            lib.tp_set_stream_k(mode)
            y, _ = ops.maxplus(x, W, argmax=False)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(_sample(y, rows), ry, err_msg=f"value-only, mode {mode}")
            del y
    finally:
        lib.tp_set_stream_k(old)


@pytest.mark.parametrize("S", [2048, 4096, 8192])
def test_bf16_storage(cuda, S):
    from mk_iii_technologies_tsrn_b200 import _lib, ops
    lib = _lib.load()
    x, W = _inputs(S)
    xb, Wb = x.bfloat16(), W.bfloat16()
    rows = _rows(S)
    ry, ri = oracle.maxplus_fwd(_sample(xb.float(), rows), Wb.float().cpu().numpy())
    old = lib.tp_set_stream_k(1)
    try:
        for mode in (1, 2):
            lib.tp_set_stream_k(mode)
            y, am = ops.maxplus(xb, Wb)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(_sample(y, rows), ry, err_msg=f"values, mode {mode}")
            np.testing.assert_array_equal(_sample(am, rows), ri, err_msg=f"argmax, mode {mode}")
            del y, am
    finally:
        lib.tp_set_stream_k(old)


@pytest.mark.parametrize("S", [2048, 4096, 8192])
def test_bf16_arithmetic(cuda, S):
    from mk_iii_technologies_tsrn_b200 import ops
    x, W = _inputs(S)
    xb, Wb = x.bfloat16(), W.bfloat16()
    rows = _rows(S)
    torch.set_num_threads(os.cpu_count() or 1)
    rv, ridx = maxplus_fwd_torch(xb[torch.as_tensor(rows, device=xb.device)].cpu(), Wb.cpu())
    y, am = ops.maxplus(xb, Wb, arith="bf16")
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_sample(y, rows), rv.float().numpy())
    np.testing.assert_array_equal(_sample(am, rows), ridx.numpy())
    y2, _ = ops.maxplus(xb, Wb, argmax=False, arith="bf16")
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_sample(y2, rows), rv.float().numpy())


def test_fp32_16384_sampled(cuda):
    from mk_iii_technologies_tsrn_b200 import ops
    free, _ = torch.cuda.mem_get_info()
    if free < 8 << 30:
        pytest.skip("needs ~5 GiB of free device memory")
    S = 16384
    x, W = _inputs(S)
    rows = _rows(S, n=16)
    ry, ri = oracle.maxplus_fwd(_sample(x, rows), W.cpu().numpy())
    y, am = ops.maxplus(x, W)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_sample(y, rows), ry)
    np.testing.assert_array_equal(_sample(am, rows), ri)
