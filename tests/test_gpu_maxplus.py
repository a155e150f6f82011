"""Max-plus GEMM forward on the GPU vs the oracle: values and int32 argmax bit-exact."""
import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden

pytestmark = pytest.mark.gpu


def _ops():
    from mk_iii_technologies_tsrn_b200 import ops
    return ops


@pytest.fixture(autouse=True, params=["auto", "tma"])
def argmax_path(request):
    """Every test runs with the library's default kernel choice and again with the
    TMA kernel forced for every eligible forward with argmax (its deferred
    argmax search is otherwise used only above 2^30 terms)."""
    from mk_iii_technologies_tsrn_b200 import _lib
    lib = _lib.load()
    if request.param == "auto":
        yield request.param
        return
    old = lib.tp_set_argmax_tma_min_terms(0)
    try:
        yield request.param
    finally:
        lib.tp_set_argmax_tma_min_terms(old)


def _run(x, w, bias=None, argmax=True, dev="cuda:0", dtype=torch.float32):
    ops = _ops()
    xt = torch.tensor(x, device=dev).to(dtype)
    wt = torch.tensor(w, device=dev).to(dtype)
    bt = torch.tensor(bias, device=dev) if bias is not None else None
    y, am = ops.maxplus(xt, wt, bt, argmax=argmax)
    torch.cuda.synchronize()
    return y.cpu().numpy(), (am.cpu().numpy() if am is not None else None)


def _check(x, w, bias=None, argmax=True, dtype=torch.float32):
    y, am = _run(x, w, bias, argmax, dtype=dtype)
    if dtype == torch.bfloat16:
        x = torch.tensor(x).bfloat16().float().numpy()
        w = torch.tensor(w).bfloat16().float().numpy()
    ry, ri = oracle.maxplus_fwd(x, w, bias)
    np.testing.assert_array_equal(y, ry)
    if argmax:
        np.testing.assert_array_equal(am, ri)


def test_kat_2x2_matmul_layout(cuda):
    # cuda/test_kernel.py:117-136 through the A (x) B layout (B stored [K, N])
    from mk_iii_technologies_tsrn_b200 import ops
    g = load_golden("kat_2x2")
    A = torch.tensor(g["A"], device=cuda)
    B = torch.tensor(g["B"], device=cuda)
    # w[n, k] = B[k, n]: a transposed view, strides (1, N)
    y, am = ops.maxplus_strided(A, B.t())
    np.testing.assert_array_equal(y.cpu().numpy(), g["expected"])
    np.testing.assert_array_equal(am.cpu().numpy(), g["idx"])


def test_kat_legacy_symbol(cuda):
    # the reference C symbol maxplus_matmul_cuda(A, B, C, M, K, N), B row-major [K, N]
    import ctypes
    from mk_iii_technologies_tsrn_b200 import _lib
    g = load_golden("kat_2x2")
    A = torch.tensor(g["A"], device=cuda)
    B = torch.tensor(g["B"], device=cuda)
    C = torch.empty(2, 2, device=cuda)
    lib = _lib.load()
    lib.maxplus_matmul_cuda(ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(B.data_ptr()),
                            ctypes.c_void_p(C.data_ptr()), 2, 2, 2)
    assert lib.tp_last_error() == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(C.cpu().numpy(), g["expected"])


@pytest.mark.parametrize("name", ["linear_seed42", "linear_gauss", "linear_ties",
                                  "linear_neginf", "linear_nan"])
def test_golden_forward(cuda, name):
    g = load_golden(name)
    y, am = _run(g["x"], g["W"])
    np.testing.assert_array_equal(y, g["max"])
    np.testing.assert_array_equal(am, g["idx"])


def _gauss(M, N, K, seed, neg_frac=0.05):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = rng.standard_normal((N, K)).astype(np.float32)
    if neg_frac:
        w[rng.random((N, K)) < neg_frac] = -np.inf
    return x, w


# shapes chosen to exercise the TMA kernel's M/N/K tails and the generic kernel
SHAPES = [
    (1024, 256, 256),    # config 1 (tropical linear)
    (256, 256, 64),
    (300, 200, 100),     # M, N, K tails; K % 32 != 0
    (129, 257, 96),
    (512, 384, 1000),
    (640, 512, 2048),
    (17, 3, 45),         # generic path
    (1, 1, 1),
    (33, 65, 7),
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_forward_shapes(cuda, M, N, K):
    x, w = _gauss(M, N, K, seed=M * 7 + N * 3 + K)
    _check(x, w)


@pytest.mark.parametrize("M,N,K", [(512, 384, 1000), (300, 200, 100)])
def test_forward_value_only(cuda, M, N, K):
    x, w = _gauss(M, N, K, seed=11)
    y, _ = _run(x, w, argmax=False)
    np.testing.assert_array_equal(y, oracle.maxplus_fwd(x, w)[0])


@pytest.mark.parametrize("M,N,K", [(384, 256, 192), (50, 40, 30)])
def test_forward_bias(cuda, M, N, K):
    x, w = _gauss(M, N, K, seed=5)
    bias = np.random.default_rng(6).standard_normal(N).astype(np.float32)
    _check(x, w, bias)
    y, _ = _run(x, w, bias, argmax=False)
    np.testing.assert_array_equal(y, oracle.maxplus_fwd(x, w, bias)[0])


@pytest.mark.parametrize("M,N,K", [(512, 256, 320), (40, 30, 20)])
def test_forward_ties(cuda, M, N, K):
    rng = np.random.default_rng(9)
    x = rng.integers(-2, 3, (M, K)).astype(np.float32)
    w = rng.integers(-2, 3, (N, K)).astype(np.float32)
    _check(x, w)


@pytest.mark.parametrize("M,N,K", [(512, 256, 320), (40, 30, 70)])
def test_forward_nan_inf(cuda, M, N, K):
    x, w = _gauss(M, N, K, seed=3)
    rng = np.random.default_rng(4)
    x[rng.random((M, K)) < 0.0005] = np.nan
    x[rng.random((M, K)) < 0.001] = np.inf
    x[7, :] = -np.inf          # an all -inf row
    _check(x, w)


@pytest.mark.parametrize("M,N,K", [(512, 256, 320), (33, 20, 50), (1024, 640, 200)])
def test_forward_bf16_inputs(cuda, M, N, K):
    x, w = _gauss(M, N, K, seed=21)
    _check(x, w, dtype=torch.bfloat16)


def test_forward_planted_long_k(cuda):
    # K = 20000 spans 313 argmax chunks.  Every row gets a unique planted max at a
    # random k; rows m % 3 == 0 also get an exact tie between k1 < k2 in late
    # chunks, which must resolve to k1 (size-independent check of the chunked
    # argmax recovery).
    ops = _ops()
    M, N, K = 512, 512, 20000
    k1, k2 = 19200, 19999
    gen = torch.Generator(device=cuda).manual_seed(0)
    x = torch.rand(M, K, device=cuda, generator=gen) - 1.0          # in [-1, 0)
    w = torch.rand(N, K, device=cuda, generator=gen) - 1.0
    w[:, k1] = 0.5
    w[:, k2] = 0.5
    rows = torch.arange(M, device=cuda)
    kstar = torch.randint(0, K, (M,), device=cuda, generator=gen)
    x[rows, kstar] = 5.0
    tie = rows % 3 == 0
    x[tie, k1] = 5.0
    x[tie, k2] = 5.0
    y, am = ops.maxplus(x, w)
    exp_y = 5.0 + w[torch.arange(N, device=cuda)[None, :], kstar[:, None]]
    exp_i = kstar[:, None].expand(M, N).to(torch.int32)
    exp_y = torch.where(tie[:, None], torch.full_like(exp_y, 5.5), exp_y)
    exp_i = torch.where(tie[:, None], torch.full_like(exp_i, k1), exp_i)
    assert torch.equal(y, exp_y)
    assert torch.equal(am, exp_i)


def test_empty_and_k0(cuda):
    ops = _ops()
    x = torch.empty(5, 0, device=cuda)
    w = torch.empty(4, 0, device=cuda)
    y, am = ops.maxplus(x, w)
    assert torch.all(torch.isneginf(y)) and torch.all(am == 0)
    y, am = ops.maxplus(torch.empty(0, 8, device=cuda), torch.randn(3, 8, device=cuda))
    assert y.shape == (0, 3)


def test_rejects_cpu_tensors():
    from mk_iii_technologies_tsrn_b200 import ops
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ops.maxplus(torch.randn(4, 4), torch.randn(4, 4))


def test_bad_pointer_is_reported(cuda):
    import ctypes
    from mk_iii_technologies_tsrn_b200 import _lib
    lib = _lib.load()
    host = torch.randn(4, 4)
    dev = torch.randn(4, 4, device=cuda)
    y = torch.empty(4, 4, device=cuda)
    st = lib.tp_maxplus_fwd(0, 4, 4, 4, ctypes.c_void_p(host.data_ptr()), 4,
                            ctypes.c_void_p(dev.data_ptr()), 4, None,
                            ctypes.c_void_p(y.data_ptr()), 4, None, 0, None)
    assert st == -6  # TP_ERR_BAD_POINTER
    assert lib.tp_device_error(0) == 0


def test_bf16_widening_exact(cuda):
    from mk_iii_technologies_tsrn_b200 import ops
    bits = torch.randint(0, 1 << 16, (100003,), dtype=torch.int32).to(torch.int16)
    src = bits.view(torch.bfloat16).to(cuda)
    out = ops.widen_bf16(src)
    assert torch.equal(out.view(torch.int32), src.float().view(torch.int32))
    odd = src[1:]                      # unaligned start: scalar path
    assert torch.equal(ops.widen_bf16(odd).view(torch.int32), odd.float().view(torch.int32))


def test_forward_large_sampled(cuda):
    # above the default TMA threshold (1100*1030*1000 > 2^30 terms), with M, N, K
    # tails, integer ties, NaN, +inf, an all -inf row and a bias; rows sampled
    # for the oracle
    rng = np.random.default_rng(31)
    M, N, K = 1100, 1030, 1000
    x = rng.integers(-3, 4, (M, K)).astype(np.float32)
    w = rng.standard_normal((N, K)).astype(np.float32)
    w[:, ::7] = np.round(w[:, ::7])
    x[rng.random((M, K)) < 0.0003] = np.nan
    x[rng.random((M, K)) < 0.0005] = np.inf
    x[5, :] = -np.inf
    bias = rng.standard_normal(N).astype(np.float32)
    y, am = _run(x, w, bias)
    rows = np.concatenate([[0, 5, M - 1], rng.choice(M, 61, replace=False)])
    ry, ri = oracle.maxplus_fwd(x[rows], w, bias)
    np.testing.assert_array_equal(y[rows], ry)
    np.testing.assert_array_equal(am[rows], ri)


# ----------------------------------------------------------------- bf16 arithmetic
def _run_bf16_arith(x, w, bias=None, argmax=True):
    ops = _ops()
    xt = torch.tensor(x, device="cuda").bfloat16()
    wt = torch.tensor(w, device="cuda").bfloat16()
    bt = torch.tensor(bias, device="cuda") if bias is not None else None
    y, am = ops.maxplus(xt, wt, bt, argmax=argmax, arith="bf16")
    torch.cuda.synchronize()
    return y.cpu().numpy(), (am.cpu().numpy() if am is not None else None)


@pytest.mark.parametrize("name", ["linear_bf16_gauss", "linear_bf16_ties"])
def test_bf16_arith_golden(cuda, name):
    # the reference TropicalLinear on bf16 tensors: bit-exact max and index
    g = load_golden(name)
    y, am = _run_bf16_arith(g["x"], g["W"])
    np.testing.assert_array_equal(y, g["max"])
    np.testing.assert_array_equal(am, g["idx"])


@pytest.mark.parametrize("M,N,K", [(1024, 256, 256), (300, 200, 136), (512, 384, 1000),
                                   (256, 130, 4100), (33, 20, 50)])
def test_bf16_arith_shapes(cuda, M, N, K):
    rng = np.random.default_rng(M + N + K)
    x = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 3).astype(np.float32)
    x[rng.random((M, K)) < 0.0005] = np.nan
    w[rng.random((N, K)) < 0.05] = -np.inf
    x[min(3, M - 1), :] = -np.inf
    y, am = _run_bf16_arith(x, w)
    ry, ri = oracle.maxplus_fwd_bf16(x, w)
    np.testing.assert_array_equal(y, ry)
    np.testing.assert_array_equal(am, ri)


@pytest.mark.parametrize("M,N,K", [(512, 256, 320), (40, 30, 70)])
def test_bf16_arith_ties_bias_value_only(cuda, M, N, K):
    rng = np.random.default_rng(7)
    x = (rng.integers(-4, 5, (M, K)) * 0.25).astype(np.float32)
    w = (rng.integers(-4, 5, (N, K)) * 0.25).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    y, am = _run_bf16_arith(x, w, bias)
    ry, ri = oracle.maxplus_fwd_bf16(x, w, bias)
    np.testing.assert_array_equal(y, ry)
    np.testing.assert_array_equal(am, ri)
    y2, _ = _run_bf16_arith(x, w, bias, argmax=False)
    np.testing.assert_array_equal(y2, ry)


def test_bf16_arith_large_sampled(cuda):
    # above the default TMA threshold: the packed bf16x2 kernel with its argmax search
    rng = np.random.default_rng(41)
    M, N, K = 1100, 1030, 1000
    x = (rng.standard_normal((M, K)) * 2).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 2).astype(np.float32)
    x[rng.random((M, K)) < 0.0003] = np.nan
    bias = rng.standard_normal(N).astype(np.float32)
    y, am = _run_bf16_arith(x, w, bias)
    rows = np.concatenate([[0, M - 1], rng.choice(M, 62, replace=False)])
    ry, ri = oracle.maxplus_fwd_bf16(x[rows], w, bias)
    np.testing.assert_array_equal(y[rows], ry)
    np.testing.assert_array_equal(am[rows], ri)
