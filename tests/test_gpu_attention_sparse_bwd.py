"""Sparse backward of the fused TSRN attention (``ops.tsrn_attention_train_fwd`` +
``ops.tsrn_attention_sparse_bwd``, used by ``TopKAttentionFunction``) against
float64 autograd of the reference expression (research/tsrn_dml.py:438-460,
:509-524; oracle/torch_ref.py) on inputs without near-ties at the top-k cut,
against the dense backward on the same inputs, and for repeatability.

Tolerance: 2e-4 of each gradient's scale (the kernels' exp / log and sums are
fp32; the reference is float64)."""
import pytest
import torch

from oracle.torch_ref import tsrn_attention_torch

pytestmark = pytest.mark.gpu


def _ops():
    from mk_iii_technologies_tsrn_b200 import ops
    return ops


def _close(got, ref, rtol=2e-4, atol=2e-5):
    got = got.detach().double().cpu()
    ref = ref.detach().double().cpu()
    scale = ref.abs().max().item() + 1e-30
    err = (got - ref).abs().max().item()
    assert err <= atol * max(1.0, scale) + rtol * scale, err / scale


def _unambiguous(B, H, T, dh, top_k, causal=True, first_seed=0):
    # inputs whose float64 scores keep a gap of 1e-4 at the top-k cut in every
    # row (the kernels' scores are within ~1e-6 of float64)
    pos = torch.arange(T)
    for seed in range(first_seed, first_seed + 50):
        gen = torch.Generator().manual_seed(seed)
        Q, K, V = (torch.randn(B, H, T, dh, generator=gen) for _ in range(3))
        slopes = 2.0 ** (-8.0 * torch.arange(1, H + 1, dtype=torch.float64) / H)
        S = torch.logsumexp(Q.double().unsqueeze(3) + K.double().unsqueeze(2), dim=-1)
        S = S - slopes.view(-1, 1, 1) * (pos[:, None] - pos[None, :]).abs()
        if causal:
            S = S.masked_fill(pos[None, :] > pos[:, None], float("-inf"))
        srt = S.sort(dim=-1, descending=True).values
        gap = (srt[..., top_k - 1] - srt[..., top_k]).abs()
        if torch.nan_to_num(gap, nan=1.0, posinf=1.0).min() > 1e-4:
            return Q, K, V, slopes.float()
    raise RuntimeError("no unambiguous case")


def _grads(cuda, Q, K, V, slopes, k, causal, gout, sparse=True):
    from mk_iii_technologies_tsrn_b200.tsrn_attention import TopKAttentionFunction
    q, kk, v = (t.to(cuda).requires_grad_(True) for t in (Q, K, V))
    # drop_p = 1e-12 takes the dense path (dropout form) with every weight kept
    out = TopKAttentionFunction.apply(q, kk, v, slopes.to(cuda), k, causal, 0,
                                      0.0 if sparse else 1e-12)
    (out * gout.to(cuda)).sum().backward()
    return out, q.grad, kk.grad, v.grad


@pytest.mark.parametrize("B,H,T,dh,k,causal", [
    (2, 3, 40, 16, 5, True),
    (1, 2, 200, 80, 16, True),      # config 5's head size, two query tiles
    (1, 2, 150, 24, 8, False),      # non-causal
    (1, 1, 70, 20, 4, True),        # dh not a multiple of 8
])
def test_sparse_backward_vs_float64(cuda, B, H, T, dh, k, causal):
    Q, K, V, slopes = _unambiguous(B, H, T, dh, k, causal)
    gout = torch.randn(B, H, T, dh, generator=torch.Generator().manual_seed(7))
    out, gq, gk, gv = _grads(cuda, Q, K, V, slopes, k, causal, gout)
    qd, kd, vd = (t.double().requires_grad_(True) for t in (Q, K, V))
    ref = tsrn_attention_torch(qd, kd, vd, slopes.double(), k, causal)
    (ref * gout.double()).sum().backward()
    _close(out, ref, rtol=1e-4)
    _close(gq, qd.grad)
    _close(gk, kd.grad)
    _close(gv, vd.grad)


def test_sparse_equals_dense_backward(cuda):
    Q, K, V, slopes = _unambiguous(1, 3, 96, 32, 8)
    gout = torch.randn(Q.shape, generator=torch.Generator().manual_seed(3))
    a = _grads(cuda, Q, K, V, slopes, 8, True, gout, sparse=True)
    b = _grads(cuda, Q, K, V, slopes, 8, True, gout, sparse=False)
    for x, y in zip(a[1:], b[1:]):
        _close(x, y, rtol=1e-4)


def test_sparse_backward_repeats_bit_for_bit(cuda):
    ops = _ops()
    g = torch.Generator(device=cuda).manual_seed(1)
    B, H, T, dh, k = 2, 4, 256, 80, 16
    Q, K, V, dO = (torch.randn(B, H, T, dh, device=cuda, generator=g) for _ in range(4))
    slopes = 2.0 ** (-8.0 * torch.arange(1, H + 1, device=cuda, dtype=torch.float32) / H)
    _, kj, kp, kl, kn = ops.tsrn_attention_train_fwd(Q, K, V, slopes, k)
    assert int(kn.min()) >= 0
    first = ops.tsrn_attention_sparse_bwd(Q, K, V, dO, kj, kp, kl, kn)
    second = ops.tsrn_attention_sparse_bwd(Q, K, V, dO, kj, kp, kl, kn)
    for x, y in zip(first, second):
        assert torch.equal(x, y)


def test_lists_match_the_forward(cuda):
    # the saved weights are the softmax over each row's kept keys: they sum to
    # one, and P @ V over the lists reproduces the forward's output
    ops = _ops()
    g = torch.Generator(device=cuda).manual_seed(2)
    B, H, T, dh, k = 1, 2, 180, 40, 8
    Q, K, V = (torch.randn(B, H, T, dh, device=cuda, generator=g) for _ in range(3))
    slopes = torch.tensor([0.5, 0.01], device=cuda)
    out, kj, kp, kl, kn = ops.tsrn_attention_train_fwd(Q, K, V, slopes, k)
    assert int(kn.min()) >= 0
    assert torch.equal((kj >= 0).sum(dim=1).to(torch.int32), kn)
    torch.testing.assert_close(kp.sum(dim=1), torch.ones(B * H * T, device=cuda),
                               rtol=1e-5, atol=1e-5)
    Vr = V.reshape(B * H, T, dh)
    rows = torch.arange(B * H * T, device=cuda) // T
    gathered = Vr[rows[:, None], kj.clamp(min=0).long()]          # [rows, 32, dh]
    recon = (kp[..., None] * gathered).sum(dim=1).reshape(B, H, T, dh)
    torch.testing.assert_close(recon, out, rtol=1e-4, atol=1e-5)
    # the saved scores before ALiBi are logsumexp_c(Q_i + K_j) of the kept pairs
    Qr, Kr = Q.reshape(B * H * T, dh).double(), K.reshape(B * H, T, dh).double()
    Kg = Kr[rows[:, None], kj.clamp(min=0).long()]                 # [rows, 32, dh]
    lse = torch.logsumexp(Qr[:, None, :] + Kg, dim=-1)
    valid = kj >= 0
    torch.testing.assert_close(kl.double()[valid], lse[valid], rtol=0, atol=2e-5)


def test_tie_overflow_falls_back_to_dense(cuda):
    # equal keys and no ALiBi: every visible key ties and is kept, more than the
    # lists hold; the count reads -1 and the backward takes the dense path
    ops = _ops()
    B, H, T, dh, k = 1, 1, 60, 16, 4
    gen = torch.Generator().manual_seed(4)
    Q = torch.randn(B, H, T, dh, generator=gen)
    K = torch.randn(B, H, 1, dh, generator=gen).expand(B, H, T, dh).contiguous()
    V = torch.randn(B, H, T, dh, generator=gen)
    slopes = torch.zeros(H)
    _, _, _, _, kn = ops.tsrn_attention_train_fwd(Q.to(cuda), K.to(cuda), V.to(cuda),
                                                  slopes.to(cuda), k)
    assert int(kn.min()) == -1
    gout = torch.randn(Q.shape, generator=torch.Generator().manual_seed(5))
    out, gq, gk, gv = _grads(cuda, Q, K, V, slopes, k, True, gout)
    qd, kd, vd = (t.double().requires_grad_(True) for t in (Q, K, V))
    ref = tsrn_attention_torch(qd, kd, vd, slopes.double(), k, True)
    (ref * gout.double()).sum().backward()
    _close(gq, qd.grad)
    _close(gk, kd.grad)
    _close(gv, vd.grad)


def test_empty(cuda):
    ops = _ops()
    z = torch.zeros(1, 2, 0, 16, device=cuda)
    out, kj, kp, kl, kn = ops.tsrn_attention_train_fwd(z, z, z, torch.ones(2, device=cuda), 4)
    assert out.shape == z.shape and kn.numel() == 0


def test_keys_out_of_range_are_empty_slots(cuda):
    # a caller's lists with keys past the slice: those slots contribute nothing
    # (and are not read), the other entries are unchanged
    ops = _ops()
    g = torch.Generator(device=cuda).manual_seed(6)
    B, H, T, dh, k = 1, 2, 140, 24, 8
    Q, K, V, dO = (torch.randn(B, H, T, dh, device=cuda, generator=g) for _ in range(4))
    slopes = torch.tensor([0.5, 0.1], device=cuda)
    _, kj, kp, kl, kn = ops.tsrn_attention_train_fwd(Q, K, V, slopes, k)
    ref = ops.tsrn_attention_sparse_bwd(Q, K, V, dO, kj, kp, kl, kn)
    bad = kj.clone()
    bad[kj < 0] = T + 1000            # padding slots pointing past the slice
    got = ops.tsrn_attention_sparse_bwd(Q, K, V, dO, bad, kp, kl, kn)
    for x, y in zip(got, ref):
        assert torch.equal(x, y)
