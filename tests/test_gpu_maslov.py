"""Gated Maslov softmax kernel vs the PyTorch fp32 expression of the reference
modules (deep_tropical_net.py:152-160, tropformer.py:206-212), forward and
autograd backward, with and without the gate, with broadcast masks."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _tau(log_temps):
    return log_temps.exp().clamp(min=0.02, max=10.0)


def _ref(T, C, g, log_temps, mask):
    if C is not None:
        gg = g.permute(0, 2, 1).unsqueeze(-1)
        s = gg * T + (1.0 - gg) * C
    else:
        s = T
    if mask is not None:
        s = s.masked_fill(mask == 0, -1e9)
    return torch.softmax(s / _tau(log_temps).view(1, -1, 1, 1), dim=-1)


def _ours(T, C, g, log_temps, mask):
    from mk_iii_technologies_tsrn_b200 import ops
    return ops.maslov_softmax(T, _tau(log_temps), classical=C, gate=g, mask=mask)


def _mask(kind, B, H, Lq, Lk, dev, gen):
    if kind is None:
        return None
    if kind == "causal":       # [Lq, Lk], broadcast over B and H
        return torch.ones(Lq, Lk, device=dev).tril()
    if kind == "pad":          # [B, 1, 1, Lk] padding (bool)
        keep = torch.rand(B, 1, 1, Lk, device=dev, generator=gen) > 0.3
        keep[..., 0] = True
        return keep
    if kind == "rows":         # full [B, H, Lq, Lk] with some rows entirely masked
        m = (torch.rand(B, H, Lq, Lk, device=dev, generator=gen) > 0.2).float()
        m[0, 0, : max(1, Lq // 3)] = 0.0
        return m
    raise ValueError(kind)


@pytest.mark.parametrize("B,H,Lq,Lk", [(4, 8, 64, 64), (2, 3, 17, 1), (2, 3, 5, 33),
                                       (3, 2, 40, 100), (2, 2, 9, 256), (2, 2, 7, 300)])
@pytest.mark.parametrize("gated", [True, False])
@pytest.mark.parametrize("mask_kind", [None, "causal", "pad", "rows"])
def test_maslov_softmax_matches_torch(cuda, B, H, Lq, Lk, gated, mask_kind):
    if mask_kind == "causal" and Lq > Lk:
        pytest.skip("causal mask needs Lq <= Lk here")
    gen = torch.Generator(device=cuda).manual_seed(B * 1000 + Lk)
    T = (torch.randn(B, H, Lq, Lk, device=cuda, generator=gen) * 2).requires_grad_(True)
    C = (torch.randn(B, H, Lq, Lk, device=cuda, generator=gen) * 2).requires_grad_(gated)
    g = torch.rand(B, Lq, H, device=cuda, generator=gen).requires_grad_(gated)
    log_temps = torch.log(torch.rand(H, device=cuda, generator=gen) * 0.9 + 0.1)
    log_temps.requires_grad_(True)
    mask = _mask(mask_kind, B, H, Lq, Lk, cuda, gen)
    if not gated:
        C = g = None
    up = torch.randn(B, H, Lq, Lk, device=cuda, generator=gen)

    leaves = [t for t in (T, C, g, log_temps) if t is not None]
    names = ("T", "C", "g", "log_temps") if gated else ("T", "log_temps")
    # reference: the module expression in fp64 (fp32 PyTorch rounds the
    # temperature gradient of a fully masked row to noise: -1e9 * sum(dz))
    leaves64 = [t.detach().double().requires_grad_(True) for t in leaves]
    l64 = dict(zip(names, leaves64))
    P_ref = _ref(l64["T"], l64.get("C"), l64.get("g"), l64["log_temps"], mask)
    grads_ref = torch.autograd.grad((P_ref * up.double()).sum(), leaves64)
    P = _ours(T, C, g, log_temps, mask)
    grads = torch.autograd.grad((P * up).sum(), leaves)

    torch.testing.assert_close(P, P_ref.float(), rtol=1e-5, atol=1e-6)
    for name, a, b in zip(names, grads, grads_ref):
        scale = max(1.0, b.abs().max().item())
        torch.testing.assert_close(a, b.float(), rtol=1e-4, atol=2e-5 * scale, msg=name)


def test_maslov_softmax_empty(cuda):
    from mk_iii_technologies_tsrn_b200 import ops
    log_temps = torch.zeros(3, device=cuda, requires_grad=True)
    for shape in ((0, 3, 4, 5), (2, 3, 0, 5)):
        T = torch.randn(*shape, device=cuda, requires_grad=True)
        P = ops.maslov_softmax(T, _tau(log_temps))
        assert P.shape == T.shape
        P.sum().backward()
    # no keys: empty rows, zero gate and temperature gradients
    T = torch.randn(2, 3, 4, 0, device=cuda, requires_grad=True)
    C = torch.randn(2, 3, 4, 0, device=cuda)
    g = torch.rand(2, 4, 3, device=cuda, requires_grad=True)
    P = ops.maslov_softmax(T, _tau(log_temps), classical=C, gate=g)
    assert P.shape == T.shape
    P.sum().backward()
    assert torch.all(g.grad == 0)


def test_maslov_softmax_rejects_bad_arguments(cuda):
    from mk_iii_technologies_tsrn_b200 import ops
    T = torch.randn(2, 3, 4, 5, device=cuda)
    tau = torch.ones(3, device=cuda)
    with pytest.raises(ValueError):
        ops.maslov_softmax(T, torch.ones(2, device=cuda))
    with pytest.raises(ValueError):
        ops.maslov_softmax(T, tau, classical=T)                 # classical without gate
    with pytest.raises(ValueError):
        ops.maslov_softmax(T, tau, classical=T, gate=torch.rand(2, 3, 4, device=cuda))
    with pytest.raises(RuntimeError):
        ops.maslov_softmax(T.cpu(), tau.cpu())                  # no CPU path


def test_maslov_module_and_dtn_use_kernel(cuda):
    """MaslovTemperature and DTNAttention run the fused kernel (its autograd node)."""
    from mk_iii_technologies_tsrn_b200.dtn import DTNAttention
    from mk_iii_technologies_tsrn_b200.tropical import MaslovTemperature
    m = MaslovTemperature(4).to(cuda)
    s = torch.randn(2, 4, 8, 8, device=cuda, requires_grad=True)
    out = m(s)
    assert type(out.grad_fn).__name__.startswith("MaslovSoftmaxFunction")
    attn = DTNAttention(32, 4, dropout=0.0).to(cuda)
    _, w = attn(torch.randn(2, 8, 32, device=cuda))
    assert type(w.grad_fn).__name__.startswith("MaslovSoftmaxFunction")
