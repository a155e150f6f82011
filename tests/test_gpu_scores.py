"""Batched tropical attention scores on the GPU (hard max and log-sum-exp)."""
import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden

pytestmark = pytest.mark.gpu


def _ops():
    from mk_iii_technologies_tsrn_b200 import ops
    return ops


@pytest.mark.parametrize("smooth", [False, True])
def test_dtn_scores_golden(cuda, smooth):
    g = load_golden("dtn_scores")
    ops = _ops()
    Q = torch.tensor(g["Q"], device=cuda, requires_grad=True)
    K = torch.tensor(g["K"], device=cuda, requires_grad=True)
    tau = float(g["smooth_temp"]) if smooth else None
    S = ops.TropicalScoreFunction.apply(Q, K, float(g["scale"]), tau)
    (S * torch.tensor(g["gS"], device=cuda)).sum().backward()
    tag = "smooth" if smooth else "hard"
    np.testing.assert_array_equal(S.detach().cpu().numpy(), g[f"S_{tag}"])
    np.testing.assert_allclose(Q.grad.cpu().numpy(), g[f"gQ_{tag}"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(K.grad.cpu().numpy(), g[f"gK_{tag}"], rtol=1e-5, atol=1e-6)


def test_config2_scores_head_views(cuda):
    # config 2 score shapes: B=128, L=64, d_model=256, H=8 -> Q/K [B,H,L,32] as views
    # of [B, L, 256] (deep_tropical_net.py:140-150)
    B, L, D, H = 128, 64, 256, 8
    dk = D // H
    gen = torch.Generator(device=cuda).manual_seed(0)
    q = torch.randn(B, L, D, device=cuda, generator=gen)
    k = torch.randn(B, L, D, device=cuda, generator=gen)
    Q = q.view(B, L, H, dk).transpose(1, 2)
    K = k.view(B, L, H, dk).transpose(1, 2)
    ops = _ops()
    S, am = ops.tropical_scores(Q, K, dk ** -0.5)
    ref = (Q.unsqueeze(3) + K.unsqueeze(2)).max(dim=-1)    # same expression on GPU
    Qn, Kn = Q.cpu().numpy(), K.cpu().numpy()
    Sn, An = S.cpu().numpy(), am.cpu().numpy()
    for b in (0, 77, 127):
        for h in (0, 5):
            y, i = oracle.maxplus_fwd(Qn[b, h], Kn[b, h], scale=dk ** -0.5)
            np.testing.assert_array_equal(Sn[b, h], y)
            np.testing.assert_array_equal(An[b, h], i)
    assert torch.equal(S, ref.values * dk ** -0.5)
    assert torch.equal(am.long(), ref.indices)


def test_tsrn_lse_scores_golden(cuda):
    g = load_golden("tsrn_scores")
    ops = _ops()
    S = ops.lse_scores(torch.tensor(g["Q"], device=cuda), torch.tensor(g["K"], device=cuda))
    np.testing.assert_allclose(S.cpu().numpy(), g["S64"], rtol=1e-5, atol=1e-5)


def test_tsrn_lse_scores_config5_slice(cuda):
    # config 5 head size d_h = 80, T = 1024, strided head views of [B, T, 640]
    B, T, H, dh = 2, 1024, 8, 80
    gen = torch.Generator(device=cuda).manual_seed(1)
    q = torch.randn(B, T, H * dh, device=cuda, generator=gen)
    k = torch.randn(B, T, H * dh, device=cuda, generator=gen)
    Q = q.view(B, T, H, dh).permute(0, 2, 1, 3)
    K = k.view(B, T, H, dh).permute(0, 2, 1, 3)
    ops = _ops()
    S = ops.lse_scores(Q, K).cpu().numpy()
    Qn, Kn = Q.cpu().numpy(), K.cpu().numpy()
    for b, h in ((0, 0), (1, 7)):
        ref = oracle.maxplus_lse_fwd(Qn[b, h, :128], Kn[b, h], 1.0)
        np.testing.assert_allclose(S[b, h, :128], ref, rtol=1e-5, atol=1e-5)


def test_lse_scores_gradient(cuda):
    g = load_golden("tsrn_scores")
    ops = _ops()
    Q = torch.tensor(g["Q"], device=cuda, requires_grad=True)
    K = torch.tensor(g["K"], device=cuda, requires_grad=True)
    S = ops.LSEScoreFunction.apply(Q, K, 1.0)
    gS = torch.randn_like(S)
    (S * gS).sum().backward()
    Q64 = torch.tensor(g["Q"], dtype=torch.float64, requires_grad=True)
    K64 = torch.tensor(g["K"], dtype=torch.float64, requires_grad=True)
    S64 = torch.logsumexp(Q64.unsqueeze(3) + K64.unsqueeze(2), dim=-1)
    (S64 * gS.double().cpu()).sum().backward()
    np.testing.assert_allclose(Q.grad.cpu().numpy(), Q64.grad.numpy(), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(K.grad.cpu().numpy(), K64.grad.numpy(), rtol=1e-5, atol=1e-5)
