"""Tropical SSM scan on the GPU vs the sequential recurrence: bit-exact."""
import numpy as np
import pytest
import torch

from oracle import scan as oscan
from conftest import load_golden

pytestmark = pytest.mark.gpu


def _ops():
    from mk_iii_technologies_tsrn_b200 import ops
    return ops


def _inputs(B, T, C, seed):
    rng = np.random.default_rng(seed)
    a = -rng.random(C).astype(np.float32)                        # a = -U(0,1)
    b = (0.1 * rng.standard_normal((B, T, C))).astype(np.float32)  # b ~ N(0, 0.1)
    x = rng.standard_normal((B, T, C)).astype(np.float32)         # x ~ N(0, 1)
    return a, b, x


SHAPES = [(2, 100, 64), (3, 64, 40), (1, 33, 5), (2, 1, 32), (4, 257, 96), (1, 31, 128)]


@pytest.mark.parametrize("B,T,C", SHAPES)
@pytest.mark.parametrize("h_init", [float("-inf"), 0.0])
def test_forward_exact(cuda, B, T, C, h_init):
    a, b, x = _inputs(B, T, C, seed=B * 100 + T + C)
    ops = _ops()
    h, mask = ops.scan_forward(torch.tensor(b, device=cuda), torch.tensor(x, device=cuda),
                               torch.tensor(a, device=cuda), h_init, need_mask=True)
    u = (b + x).astype(np.float32)
    rh, win = oscan.scan_fwd(u, a, h_init)
    np.testing.assert_array_equal(h.cpu().numpy(), rh)
    np.testing.assert_array_equal(mask.cpu().numpy().view(np.uint32),
                                  oscan.win_mask_words(win))


@pytest.mark.parametrize("B,T,C", [(2, 100, 64), (1, 33, 5)])
def test_forward_h0_and_no_x(cuda, B, T, C):
    a, b, _ = _inputs(B, T, C, seed=7)
    h0 = np.random.default_rng(8).standard_normal((B, C)).astype(np.float32)
    ops = _ops()
    h, _ = ops.scan_forward(torch.tensor(b, device=cuda), None, torch.tensor(a, device=cuda),
                            0.0, torch.tensor(h0, device=cuda))
    rh, _ = oscan.scan_fwd(b, a, 0.0, h0)
    np.testing.assert_array_equal(h.cpu().numpy(), rh)


@pytest.mark.parametrize("B,T,C", [(2, 100, 64), (3, 64, 40), (1, 33, 5), (4, 257, 96)])
@pytest.mark.parametrize("use_mask", [True, False])
def test_backward_exact(cuda, B, T, C, use_mask):
    a, b, x = _inputs(B, T, C, seed=B + T + C)
    h0 = np.random.default_rng(3).standard_normal((B, C)).astype(np.float32)
    gh = np.random.default_rng(4).standard_normal((B, T, C)).astype(np.float32)
    ops = _ops()
    bt, xt, at = (torch.tensor(v, device=cuda) for v in (b, x, a))
    h0t = torch.tensor(h0, device=cuda)
    h, mask = ops.scan_forward(bt, xt, at, 0.0, h0t, need_mask=True)
    kw = dict(mask=mask) if use_mask else dict(b=bt, x=xt, h=h)
    gu, ga, gh0 = ops.scan_backward(torch.tensor(gh, device=cuda), at, 0.0, h0t,
                                    need_ga=True, need_gh0=True, **kw)
    _, win = oscan.scan_fwd((b + x).astype(np.float32), a, 0.0, h0)
    rgu, rga, rgh0 = oscan.scan_bwd(gh, win, dtype=np.float32)
    np.testing.assert_array_equal(gu.cpu().numpy(), rgu)
    np.testing.assert_array_equal(ga.cpu().numpy(), rga)
    np.testing.assert_array_equal(gh0.cpu().numpy(), rgh0)


def test_config3_full_size(cuda):
    # config 3: B=16, T=4096, C=1024, a=-U(0,1), b~N(0,0.1), x~N(0,1), h0=-inf
    B, T, C = 16, 4096, 1024
    gen = torch.Generator(device=cuda).manual_seed(0)
    a = -torch.rand(C, device=cuda, generator=gen)
    b = 0.1 * torch.randn(B, T, C, device=cuda, generator=gen)
    x = torch.randn(B, T, C, device=cuda, generator=gen)
    ops = _ops()
    h, mask = ops.scan_forward(b, x, a, float("-inf"), need_mask=True)
    rh, win = oscan.scan_fwd((b + x).cpu().numpy(), a.cpu().numpy(), -np.inf)
    np.testing.assert_array_equal(h.cpu().numpy(), rh)
    gh = torch.randn(B, T, C, device=cuda, generator=gen)
    gu, ga, _ = ops.scan_backward(gh, a, float("-inf"), mask=mask)
    gu2, ga2, _ = ops.scan_backward(gh, a, float("-inf"), b=b, x=x, h=h)
    assert torch.equal(gu, gu2) and torch.equal(ga, ga2)
    rgu, rga, _ = oscan.scan_bwd(gh.cpu().numpy(), win, dtype=np.float32)
    np.testing.assert_array_equal(gu.cpu().numpy(), rgu)
    np.testing.assert_array_equal(ga.cpu().numpy(), rga)


def test_reference_closed_form_tolerance(cuda):
    # the reference module's closed form (research/tsrn_dml.py:961-972) vs our exact
    # recurrence: equal up to O(T ulp)
    g = load_golden("tsrn_ssm")
    ops = _ops()
    u = torch.tensor(g["u"], device=cuda)
    h, _ = ops.scan_forward(u, None, torch.tensor(g["A_c"], device=cuda), 0.0)
    T = u.shape[1]
    tol = 4 * T * np.finfo(np.float32).eps * max(1.0, float(np.abs(g["H"]).max()))
    np.testing.assert_allclose(h.cpu().numpy(), g["H"], rtol=0, atol=tol)
