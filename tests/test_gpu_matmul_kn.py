"""A (x) B with B stored [K, N] -- the layout of the reference's
``maxplus_matmul_kernel`` (cuda/maxplus_gemm.cu:269-290) and of
``_tropical_matmul`` (benchmarks/synthetic_scheduling.py:35-38) -- at real
sizes, with -inf entries, bit-exact against the oracle; the repeated products
of ``_tropical_eigenvalue`` (:41-55) and repeated squaring, chained on the GPU.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _ab(M, K, N, seed, neg_inf=0.05):
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    B[rng.random((K, N)) < neg_inf] = -np.inf
    A[rng.random((M, K)) < neg_inf / 5] = -np.inf
    return A, B


@pytest.mark.parametrize("M,K,N", [(512, 512, 512), (1024, 2048, 768), (333, 1000, 517),
                                   (4096, 4096, 4096)])
def test_matmul_kn_layout(cuda, M, K, N):
    from mk_iii_technologies_tsrn_b200 import ops
    A, B = _ab(M, K, N, M + K + N)
    y, am = ops.maxplus_matmul(torch.tensor(A, device=cuda), torch.tensor(B, device=cuda),
                               argmax=True)
    torch.cuda.synchronize()
    rows = np.arange(M) if M <= 1024 else np.concatenate(
        [[0, M - 1], np.random.default_rng(1).choice(M, 62, replace=False)])
    ry, ri = oracle.maxplus_matmul(A[rows], B)
    np.testing.assert_array_equal(y.cpu().numpy()[rows], ry)
    np.testing.assert_array_equal(am.cpu().numpy()[rows], ri)


def test_matmul_kn_strided_and_copied_paths_agree(cuda):
    # the in-place strided read of B and the transposed-copy TMA path
    from mk_iii_technologies_tsrn_b200 import ops
    A, B = _ab(1536, 640, 1280, 9)
    At, Bt = torch.tensor(A, device=cuda), torch.tensor(B, device=cuda)
    y1 = ops.maxplus_matmul(At, Bt)
    y2, _ = ops.maxplus_strided(At, Bt.t(), argmax=False)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)


def test_legacy_matmul_symbol_at_size(cuda):
    # maxplus_matmul_cuda(A, B, C, M, K, N), B row-major [K, N]
    from mk_iii_technologies_tsrn_b200 import _lib
    M, K, N = 512, 384, 640
    A, B = _ab(M, K, N, 3)
    At, Bt = torch.tensor(A, device=cuda), torch.tensor(B, device=cuda)
    C = torch.empty(M, N, device=cuda)
    lib = _lib.load()
    lib.maxplus_matmul_cuda(ctypes.c_void_p(At.data_ptr()), ctypes.c_void_p(Bt.data_ptr()),
                            ctypes.c_void_p(C.data_ptr()), M, K, N)
    assert lib.tp_last_error() == 0
    torch.cuda.synchronize()
    ry, _ = oracle.maxplus_matmul(A, B)
    np.testing.assert_array_equal(C.cpu().numpy(), ry)


@pytest.mark.parametrize("n,steps", [(96, 50), (300, 12)])
def test_eigenvalue_power_chain(cuda, n, steps):
    # _tropical_eigenvalue: Ak = Ak (x) A repeated, then max diag / k.  Every
    # product is exact in max and one rounded add per term, so the chained GPU
    # products equal the chained oracle bit for bit.
    from mk_iii_technologies_tsrn_b200 import ops
    rng = np.random.default_rng(n)
    A = (rng.standard_normal((n, n)) * 0.5).astype(np.float32)
    A[rng.random((n, n)) < 0.3] = -np.inf           # sparse precedence graph
    Ad = torch.tensor(A, device=cuda)
    Ak = Ad.clone()
    for _ in range(steps):
        Ak = ops.maxplus_matmul(Ak, Ad)
    ref, lam = oracle.tropical_power_chain(A, steps)
    np.testing.assert_array_equal(Ak.cpu().numpy(), ref)
    diag_max = np.float32(torch.diagonal(Ak).max().item())
    assert diag_max == np.diag(ref).max()
    assert float(diag_max / np.float32(steps + 1)) == pytest.approx(lam, rel=1e-7)


def test_repeated_squaring(cuda):
    # A^(2^j) by squaring, j = 1..6, at n = 512 (the TMA path at the top sizes)
    from mk_iii_technologies_tsrn_b200 import ops
    rng = np.random.default_rng(5)
    n = 512
    A = (rng.standard_normal((n, n)) - 2.0).astype(np.float32)
    A[rng.random((n, n)) < 0.2] = -np.inf
    Ad = torch.tensor(A, device=cuda)
    ref = A
    for _ in range(6):
        Ad = ops.maxplus_matmul(Ad, Ad)
        ref, _ = oracle.maxplus_matmul(ref, ref)
    np.testing.assert_array_equal(Ad.cpu().numpy(), ref)
