"""Max-plus backward on the GPU: argmax scatter, STE and LSE vs the oracle and the
reference's own autograd (golden vectors)."""
import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden

pytestmark = pytest.mark.gpu


def _fn():
    from mk_iii_technologies_tsrn_b200 import ops
    return ops


def _grads(x, w, b, g, mode, tau, dev):
    ops = _fn()
    xt = torch.tensor(x, device=dev, requires_grad=True)
    wt = torch.tensor(w, device=dev, requires_grad=True)
    bt = torch.tensor(b, device=dev, requires_grad=True) if b is not None else None
    y = ops.MaxPlusLinearFunction.apply(xt, wt, bt, mode, tau)
    (y * torch.tensor(g, device=dev)).sum().backward()
    out = [y.detach().cpu().numpy(), xt.grad.cpu().numpy(), wt.grad.cpu().numpy()]
    out.append(bt.grad.cpu().numpy() if bt is not None else None)
    return out


@pytest.mark.parametrize("name", ["linear_seed42", "linear_gauss", "linear_ties"])
def test_golden_eval_grads(cuda, name):
    g = load_golden(name)
    y, gx, gw, gb = _grads(g["x"], g["W"], g.get("bias"), g["g"], "argmax", 1.0, cuda)
    np.testing.assert_array_equal(y, g["y_eval"])
    np.testing.assert_allclose(gx, g["gx_eval"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(gw, g["gw_eval"], rtol=1e-6, atol=1e-5)
    if gb is not None:
        np.testing.assert_allclose(gb, g["gb_eval"], rtol=1e-6, atol=1e-5)


@pytest.mark.parametrize("name", ["linear_seed42", "linear_gauss", "linear_gauss_tau05",
                                  "linear_ties"])
def test_golden_train_grads(cuda, name):
    g = load_golden(name)
    tau = float(g["ste_temp"])
    y, gx, gw, gb = _grads(g["x"], g["W"], g.get("bias"), g["g"], "ste", tau, cuda)
    np.testing.assert_array_equal(y, g["y_train"])
    np.testing.assert_allclose(gx, g["gx_train"], rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(gw, g["gw_train"], rtol=1e-4, atol=2e-5)
    if gb is not None:
        np.testing.assert_allclose(gb, g["gb_train"], rtol=1e-5, atol=1e-5)


def _rel_err(a, b):
    scale = max(1.0, float(np.abs(b).max()))
    return float(np.abs(a - b).max()) / scale


@pytest.mark.parametrize("mode,tau", [("ste", 1.0), ("lse", 1.0), ("lse", 50.0), ("ste", 0.25)])
def test_config1_smooth_vs_oracle(cuda, mode, tau):
    # config 1: x [1024,256], W [256,256] ~ N(0,1), upstream g ~ N(0,1)
    rng = np.random.default_rng(0)
    x = rng.standard_normal((1024, 256)).astype(np.float32)
    w = rng.standard_normal((256, 256)).astype(np.float32)
    g = rng.standard_normal((1024, 256)).astype(np.float32)
    _, gx, gw, _ = _grads(x, w, None, g, mode, tau, cuda)
    rgx, rgw, _ = oracle.maxplus_bwd_smooth(mode, tau, x, w, g)
    # tolerance: 1e-5 relative to the gradient scale (fp32 exp and sums vs fp64)
    assert _rel_err(gx, rgx) < 1e-5
    assert _rel_err(gw, rgw) < 1e-5


def test_config1_argmax_vs_oracle(cuda):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((1024, 256)).astype(np.float32)
    w = rng.standard_normal((256, 256)).astype(np.float32)
    b = rng.standard_normal(256).astype(np.float32)
    g = rng.standard_normal((1024, 256)).astype(np.float32)
    y, gx, gw, gb = _grads(x, w, b, g, "argmax", 1.0, cuda)
    ry, ri = oracle.maxplus_fwd(x, w, b)
    np.testing.assert_array_equal(y, ry)
    rgx, rgw, rgb = oracle.maxplus_bwd_argmax(ri, g, 256)
    np.testing.assert_allclose(gx, rgx, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(gw, rgw, rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(gb, rgb, rtol=1e-5, atol=1e-4)


def test_bf16_smooth_backward(cuda):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((96, 80)).astype(np.float32)
    w = rng.standard_normal((64, 80)).astype(np.float32)
    g = rng.standard_normal((96, 64)).astype(np.float32)
    ops = _fn()
    xb = torch.tensor(x, device=cuda).bfloat16()
    wb = torch.tensor(w, device=cuda).bfloat16()
    gx, gw, _ = ops.maxplus_backward_smooth("ste", 1.0, xb, wb, torch.tensor(g, device=cuda))
    rgx, rgw, _ = oracle.maxplus_bwd_smooth("ste", 1.0, xb.float().cpu().numpy(),
                                            wb.float().cpu().numpy(), g)
    assert _rel_err(gx.cpu().numpy(), rgx) < 1e-5
    assert _rel_err(gw.cpu().numpy(), rgw) < 1e-5


def test_empty_rows(cuda):
    ops = _fn()
    x = torch.randn(0, 16, device=cuda, requires_grad=True)
    w = torch.randn(8, 16, device=cuda, requires_grad=True)
    y = ops.MaxPlusLinearFunction.apply(x, w, None, "ste", 1.0)
    y.sum().backward()
    assert torch.all(w.grad == 0)


@pytest.mark.parametrize("batch,M,N,K", [(1, 64, 4096, 128), (3, 2048, 64, 64), (1, 8, 1500, 40)])
def test_smooth_split_reduction(cuda, batch, M, N, K):
    # shapes whose gradient outputs are too small to fill the GPU: the reduced
    # index (n for gx, m for gw) is cut into slices whose partials are added in
    # slice order -- same tolerance as the unsplit path, and bitwise repeatable
    ops = _fn()
    rng = np.random.default_rng(3)
    x = rng.standard_normal((batch, M, K)).astype(np.float32)
    w = rng.standard_normal((batch, N, K)).astype(np.float32)
    g = rng.standard_normal((batch, M, N)).astype(np.float32)
    xt, wt, gt = (torch.tensor(a, device=cuda) for a in (x, w, g))
    gx, gw, gb = ops.maxplus_backward_smooth("ste", 0.5, xt, wt, gt, need_gbias=True)
    gx2, gw2, gb2 = ops.maxplus_backward_smooth("ste", 0.5, xt, wt, gt, need_gbias=True)
    assert torch.equal(gx, gx2) and torch.equal(gw, gw2) and torch.equal(gb, gb2)
    for b in range(batch):
        rgx, rgw, rgb = oracle.maxplus_bwd_smooth("ste", 0.5, x[b], w[b], g[b])
        assert _rel_err(gx[b].cpu().numpy(), rgx) < 1e-5
        assert _rel_err(gw[b].cpu().numpy(), rgw) < 1e-5
    np.testing.assert_allclose(gb.cpu().numpy(), g.sum(axis=(0, 1)), rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(512, 256, 256), (96, 72, 40)])
def test_smooth_backward_with_forward_max(cuda, dtype, M, N, K):
    # the stats pass seeded with the forward's maxima gives the same gradients
    ops = _fn()
    rng = np.random.default_rng(8)
    x = torch.tensor(rng.standard_normal((M, K)).astype(np.float32), device=cuda).to(dtype)
    w = torch.tensor(rng.standard_normal((N, K)).astype(np.float32), device=cuda).to(dtype)
    g = torch.tensor(rng.standard_normal((M, N)).astype(np.float32), device=cuda)
    y0, _ = ops.maxplus(x.float(), w.float(), argmax=False)
    a = ops.maxplus_backward_smooth("ste", 0.7, x, w, g)
    b = ops.maxplus_backward_smooth("ste", 0.7, x, w, g, ref_max=y0)
    for u, v in zip(a[:2], b[:2]):
        assert _rel_err(v.cpu().numpy(), u.cpu().numpy()) < 1e-5


def _smooth_both_paths(ops, lib, *args, **kw):
    old = lib.tp_set_smooth_fused(1)
    try:
        fused = ops.maxplus_backward_smooth(*args, **kw)
        lib.tp_set_smooth_fused(0)
        split = ops.maxplus_backward_smooth(*args, **kw)
    finally:
        lib.tp_set_smooth_fused(old)
    return fused, split


@pytest.mark.parametrize("mode,tau", [("ste", 0.5), ("lse", 1.0)])
@pytest.mark.parametrize("batch,M,N,K", [(1, 4096, 36, 320), (2, 4100, 20, 324)])
def test_smooth_fused_gradients_vs_oracle(cuda, mode, tau, batch, M, N, K):
    # shapes whose gx tiles fill the GPU: gx and gW come from one pass (row-tile
    # gW partials added in tile order); tails in every dimension in the second
    from mk_iii_technologies_tsrn_b200 import _lib
    ops, lib = _fn(), _lib.load()
    rng = np.random.default_rng(11)
    x = rng.standard_normal((batch, M, K)).astype(np.float32)
    w = rng.standard_normal((batch, N, K)).astype(np.float32)
    g = rng.standard_normal((batch, M, N)).astype(np.float32)
    xt, wt, gt = (torch.tensor(a, device=cuda) for a in (x, w, g))
    (gx, gw, _), (sx, sw, _) = _smooth_both_paths(ops, lib, mode, tau, xt, wt, gt)
    again = ops.maxplus_backward_smooth(mode, tau, xt, wt, gt)
    assert torch.equal(gx, again[0]) and torch.equal(gw, again[1])     # deterministic
    for b in range(batch):
        rgx, rgw, _ = oracle.maxplus_bwd_smooth(mode, tau, x[b], w[b], g[b])
        assert _rel_err(gx[b].cpu().numpy(), rgx) < 1e-5
        assert _rel_err(gw[b].cpu().numpy(), rgw) < 1e-5
    assert _rel_err(gx.cpu().numpy(), sx.cpu().numpy()) < 1e-5
    assert _rel_err(gw.cpu().numpy(), sw.cpu().numpy()) < 1e-5


def test_smooth_fused_projection_shape(cuda):
    # the DTN projection (M=8192, N=K=256, forward maxima given): the one-pass
    # kernel runs, agrees with the two-pass one, and its gx rows with the oracle
    from torch.profiler import ProfilerActivity, profile
    from mk_iii_technologies_tsrn_b200 import _lib
    ops, lib = _fn(), _lib.load()
    gen = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn(8192, 256, device=cuda, generator=gen)
    w = torch.randn(256, 256, device=cuda, generator=gen) * 0.02
    g = torch.randn(8192, 256, device=cuda, generator=gen)
    y0, _ = ops.maxplus(x, w, argmax=False)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        ops.maxplus_backward_smooth("ste", 1.0, x, w, g, ref_max=y0)
        torch.cuda.synchronize()
    assert any("smooth_grad_fused_kernel" in e.name for e in prof.events())
    (gx, gw, _), (sx, sw, _) = _smooth_both_paths(ops, lib, "ste", 1.0, x, w, g, ref_max=y0)
    assert _rel_err(gx.cpu().numpy(), sx.cpu().numpy()) < 1e-5
    assert _rel_err(gw.cpu().numpy(), sw.cpu().numpy()) < 1e-5
    rgx, _, _ = oracle.maxplus_bwd_smooth("ste", 1.0, x[:64].cpu().numpy(), w.cpu().numpy(),
                                          g[:64].cpu().numpy())
    assert _rel_err(gx[:64].cpu().numpy(), rgx) < 1e-5
