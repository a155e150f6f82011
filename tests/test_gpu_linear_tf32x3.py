"""fp32-accurate projections on the TF32 tensor cores (``ops.split_tf32``,
``ops.linear_tf32x3``, ``ops.linear``) -- the nn.Linear layers around the
tropical branches (research/tsrn_dml.py:462-548, 808-843, 917-980) in
inference.

The split is exact (hi + lo == x bit for bit, hi has no bits below TF32's);
the three-product GEMM agrees with float64 within 1e-5 of the output's scale
(fp32 SGEMM itself is ~1.5e-6 at K = 640)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ops():
    from mk_iii_technologies_tsrn_b200 import ops
    return ops


@pytest.mark.parametrize("n", [0, 1, 3, 4, 1027, 1 << 20])
def test_split_is_exact(cuda, n):
    g = torch.Generator(device=cuda).manual_seed(n)
    x = torch.randn(n, device=cuda, generator=g) * 1e3
    hi, lo = _ops().split_tf32(x)
    assert torch.equal(hi + lo, x)
    assert torch.equal(hi.view(torch.int32) & 0x1FFF, torch.zeros_like(hi, dtype=torch.int32))
    assert (lo.abs() <= hi.abs() * 2.0 ** -10).all()


def test_split_special_values(cuda):
    x = torch.tensor([float("inf"), float("-inf"), float("nan"), 0.0, -0.0, 1e-40, 3.0],
                     device=cuda)
    hi, lo = _ops().split_tf32(x)
    assert torch.isinf(hi[:2]).all() and (lo[:2] == 0).all()
    assert torch.isnan(hi[2]) and lo[2] == 0
    assert torch.equal(hi[3:] + lo[3:], x[3:])


@pytest.mark.parametrize("M,K,N,bias", [(8192, 640, 1920, False), (4099, 320, 640, True),
                                        (5000, 77, 130, True)])
def test_linear_tf32x3_vs_float64(cuda, M, K, N, bias):
    g = torch.Generator(device=cuda).manual_seed(M + K + N)
    x = torch.randn(M, K, device=cuda, generator=g)
    w = torch.randn(N, K, device=cuda, generator=g) / K ** 0.5
    b = torch.randn(N, device=cuda, generator=g) if bias else None
    y = _ops().linear_tf32x3(x, w, b)
    ref = x.double() @ w.double().T + (b.double() if bias else 0.0)
    err = ((y.double() - ref).abs().max() / ref.abs().max()).item()
    assert err < 1e-5, err
    f32 = torch.nn.functional.linear(x, w, b)
    assert ((y - f32).abs().max() / f32.abs().max()).item() < 1e-5


def test_linear_dispatch_and_tf32_setting(cuda):
    ops = _ops()
    m = torch.backends.cuda.matmul
    prev = m.allow_tf32
    g = torch.Generator(device=cuda).manual_seed(3)
    w = torch.randn(64, 48, device=cuda, generator=g)
    small = torch.randn(10, 48, device=cuda, generator=g)
    # few rows: the plain fp32 GEMM, bit for bit
    assert torch.equal(ops.linear(small, w), torch.nn.functional.linear(small, w))
    big = torch.randn(ops.LINEAR_TF32X3_MIN_ROWS, 48, device=cuda, generator=g)
    with torch.no_grad():
        y = ops.linear(big, w)
    assert torch.equal(y, ops.linear_tf32x3(big, w))
    # autograd: the same products, with a 3xTF32 backward
    wg = w.clone().requires_grad_(True)
    yg = ops.linear(big, wg)
    assert yg.requires_grad
    assert torch.equal(yg.detach(), ops.linear_tf32x3(big, w))
    # few rows under autograd: the plain fp32 GEMM
    ys = ops.linear(small, wg)
    assert torch.equal(ys.detach(), torch.nn.functional.linear(small, w))
    # the caller's TF32 setting is left as it was
    assert m.allow_tf32 == prev


def test_linear_autograd_vs_float64(cuda):
    ops = _ops()
    g = torch.Generator(device=cuda).manual_seed(11)
    M, K, N = 6000, 320, 192
    x = torch.randn(M, K, device=cuda, generator=g)
    w = torch.randn(N, K, device=cuda, generator=g) / K ** 0.5
    b = torch.randn(N, device=cuda, generator=g)
    dy = torch.randn(M, N, device=cuda, generator=g)
    xr, wr, br = (t.clone().requires_grad_(True) for t in (x, w, b))
    y = ops.linear(xr, wr, br)
    assert y.grad_fn is not None and "LinearTF32x3" in type(y.grad_fn).__name__
    y.backward(dy)
    xd, wd, bd = (t.double().requires_grad_(True) for t in (x, w, b))
    (torch.nn.functional.linear(xd, wd, bd) * dy.double()).sum().backward()
    # the output and dx reduce over K = 320, dW and db over M = 6000 rows (fp32
    # accumulation over that many rows: a few 1e-5 of the scale, as for SGEMM)
    for got, ref, tol in ((y, xd.double() @ wd.double().T + bd, 1e-5), (xr.grad, xd.grad, 1e-5),
                          (wr.grad, wd.grad, 5e-5), (br.grad, bd.grad, 5e-5)):
        err = ((got.double() - ref).abs().max() / ref.abs().max()).item()
        assert err < tol, err


def test_matmul_helpers(cuda):
    ops = _ops()
    g = torch.Generator(device=cuda).manual_seed(12)
    a = torch.randn(700, 96, device=cuda, generator=g)
    b = torch.randn(96, 50, device=cuda, generator=g)
    c = torch.randn(700, 50, device=cuda, generator=g)
    for got, ref in ((ops.matmul_tf32x3(a, b), a.double() @ b.double()),
                     (ops.matmul_tn_tf32x3(a, c), a.double().T @ c.double())):
        err = ((got.double() - ref).abs().max() / ref.abs().max()).item()
        assert err < 1e-5, err


@pytest.mark.parametrize("R,C", [(1, 4), (37, 640), (4099, 1920)])
def test_split_cat_parts(cuda, R, C):
    ops = _ops()
    g = torch.Generator(device=cuda).manual_seed(R + C)
    x = torch.randn(R, C, device=cuda, generator=g) * 100.0
    x[0, 0] = float("inf")
    hi, lo = ops.split_tf32(x)
    for nparts in (1, 2, 3):
        for mask in range(1 << nparts):
            out = ops.split_tf32_cat(x, nparts, mask)
            assert out.shape == (R, nparts * C)
            for part in range(nparts):
                want = lo if (mask >> part) & 1 else hi
                assert torch.equal(out[:, part * C:(part + 1) * C], want)


@pytest.mark.parametrize("M,K,N", [(5000, 640, 324), (5000, 640, 320), (4099, 320, 640)])
def test_linear_forms_agree(cuda, M, K, N):
    # K a multiple of 4: hi.hi and the two corrections as one GEMM of depth 2K;
    # three GEMMs otherwise -- both within 1e-5 of float64 (fp32 SGEMM: ~1e-6)
    ops = _ops()
    g = torch.Generator(device=cuda).manual_seed(M + K + N)
    x = torch.randn(M, K, device=cuda, generator=g)
    w = torch.randn(N, K, device=cuda, generator=g) / K ** 0.5
    ref = x.double() @ w.double().T
    xh, xl = ops.split_tf32(x)
    wh, wl = ops.split_tf32(w)
    for y in (ops.linear_tf32x3(x, w), ops._linear3(xh, xl, wh, wl, None)):
        assert ((y.double() - ref).abs().max() / ref.abs().max()).item() < 5e-6
