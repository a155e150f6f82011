"""Fused TSRN tropical top-k attention (forward) vs the oracle and the reference module."""
import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden
from test_oracle_golden import _ambiguous_rows

pytestmark = pytest.mark.gpu


def _case(B, H, T, Tc, dh, seed, scale=1.0):
    rng = np.random.default_rng(seed)
    Tkv = T + Tc
    Q = (rng.standard_normal((B, H, T, dh)) * scale).astype(np.float32)
    K = (rng.standard_normal((B, H, Tkv, dh)) * scale).astype(np.float32)
    V = rng.standard_normal((B, H, Tkv, dh)).astype(np.float32)
    slopes = (2.0 ** (-8.0 / H * (np.arange(H) + 1))).astype(np.float32)
    return Q, K, V, slopes


@pytest.mark.parametrize("B,H,T,Tc,dh,top_k,causal", [
    (2, 4, 64, 0, 16, 8, True),
    (1, 2, 200, 0, 40, 16, True),     # T not a multiple of the 32-row tile
    (2, 3, 97, 0, 24, 5, False),      # non-causal; Tkv not a multiple of 4
    (1, 2, 120, 40, 32, 8, True),     # cross-window cached keys (Tc > 0)
    (1, 1, 50, 0, 80, 64, True),      # top_k larger than the early rows' key count
    (1, 2, 40, 0, 128, 3, True),      # dh at its limit
])
def test_fused_attention_vs_oracle(cuda, B, H, T, Tc, dh, top_k, causal):
    from mk_iii_technologies_tsrn_b200 import ops
    Q, K, V, slopes = _case(B, H, T, Tc, dh, seed=B * 100 + T + dh)
    out = ops.tsrn_attention(*(torch.tensor(a, device=cuda) for a in (Q, K, V, slopes)),
                             top_k=top_k, causal=causal, Tc=Tc).cpu().numpy()
    ref, S = oracle.tsrn_attention_fwd(Q, K, V, slopes, top_k, causal, Tc)
    ok = ~_ambiguous_rows(S, top_k)
    assert ok.mean() > 0.9
    # tolerance: scores within ~1e-6 of fp64 -> softmax weights ~1e-6 relative
    np.testing.assert_allclose(out[ok], ref[ok], rtol=1e-4, atol=2e-5)


def test_fused_attention_large_dynamic_range(cuda):
    # channels far apart (scale 8): the exp-feature dot products get small and the
    # exact fallback may engage; still within tolerance
    from mk_iii_technologies_tsrn_b200 import ops
    Q, K, V, slopes = _case(1, 2, 96, 0, 32, seed=5, scale=8.0)
    out = ops.tsrn_attention(*(torch.tensor(a, device=cuda) for a in (Q, K, V, slopes)),
                             top_k=8).cpu().numpy()
    ref, S = oracle.tsrn_attention_fwd(Q, K, V, slopes, 8)
    ok = ~_ambiguous_rows(S, 8, gap=1e-3)
    np.testing.assert_allclose(out[ok], ref[ok], rtol=1e-4, atol=5e-5)


def test_module_matches_reference_output(cuda):
    from mk_iii_technologies_tsrn_b200.tsrn_attention import TropicalAttention
    g = load_golden("tsrn_attention")
    m = TropicalAttention(32, top_k=int(g["top_k"]), n_heads=4)
    keys = [k[2:] for k in g.keys() if k.startswith("p_")]
    m.load_state_dict({k: torch.tensor(g["p_" + k]) for k in keys})
    m = m.to(cuda).eval()
    with torch.no_grad():
        out = m(torch.tensor(g["x"], device=cuda)).cpu().numpy()
    _, S = oracle.tsrn_attention_fwd(g["Q"], g["K"], g["V"], g["slopes"], int(g["top_k"]))
    ok = ~_ambiguous_rows(S, int(g["top_k"]))          # [B,H,T]: rows of any head
    rows_ok = ok.all(axis=1)                            # [B,T]
    np.testing.assert_allclose(out[rows_ok], g["out"][rows_ok], rtol=1e-4, atol=2e-5)


def test_training_path_matches_fused(cuda):
    # train mode with gradients: LSE kernel + PyTorch ops (differentiable); same output
    from mk_iii_technologies_tsrn_b200.tsrn_attention import TropicalAttention
    torch.manual_seed(3)
    m = TropicalAttention(64, top_k=8, n_heads=4).to(cuda)
    x = torch.randn(2, 48, 64, device=cuda, requires_grad=True)
    m.train()
    y_train = m(x)
    y_train.sum().backward()
    assert x.grad is not None and torch.isfinite(x.grad).all()
    m.eval()
    with torch.no_grad():
        y_eval = m(x)
    torch.testing.assert_close(y_train.detach(), y_eval, rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("causal", [False, True])
def test_fused_attention_one_lane_holds_the_top_k(cuda, causal):
    # keys j = 0, 32, 64, ... (all owned by one lane of the selection warp) score
    # highest, so that lane holds more than its 4 candidates: the exact path runs;
    # integer-valued inputs also produce exact score ties
    from mk_iii_technologies_tsrn_b200 import ops
    B, H, T, dh, top_k = 1, 2, 256, 16, 8
    rng = np.random.default_rng(12)
    Q = rng.integers(-2, 3, (B, H, T, dh)).astype(np.float32)
    K = rng.integers(-2, 3, (B, H, T, dh)).astype(np.float32)
    K[:, :, ::32, :] += 6.0
    V = rng.standard_normal((B, H, T, dh)).astype(np.float32)
    slopes = np.zeros(H, np.float32)
    out = ops.tsrn_attention(*(torch.tensor(a, device=cuda) for a in (Q, K, V, slopes)),
                             top_k=top_k, causal=causal).cpu().numpy()
    ref, S = oracle.tsrn_attention_fwd(Q, K, V, slopes, top_k, causal)
    ok = ~_ambiguous_rows(S, top_k, gap=1e-5)
    assert ok.mean() > 0.5
    np.testing.assert_allclose(out[ok], ref[ok], rtol=1e-4, atol=2e-5)


def test_module_real_weights(cuda):
    # the TSRN-gist checkpoint's trained attention projections (Wq/Wk/Wv/Wo)
    from mk_iii_technologies_tsrn_b200.tsrn_attention import TropicalAttention
    g = load_golden("real_attention_gist")
    top_k, heads = int(g["top_k"]), int(g["n_heads"])
    m = TropicalAttention(g["x"].shape[-1], top_k=top_k, n_heads=heads)
    m.load_state_dict({k[2:]: torch.tensor(v) for k, v in g.items() if k.startswith("p_")})
    m = m.to(cuda).eval()
    with torch.no_grad():
        out = m(torch.tensor(g["x"], device=cuda)).cpu().numpy()
    _, S = oracle.tsrn_attention_fwd(g["Q"], g["K"], g["V"], g["slopes"], top_k)
    rows_ok = (~_ambiguous_rows(S, top_k)).all(axis=1)
    assert rows_ok.mean() > 0.9
    np.testing.assert_allclose(out[rows_ok], g["out"][rows_ok], rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("chunks", [1, 2, 3, 16])
def test_host_entry_equals_device_entry(cuda, chunks):
    # the host-pipelined entry (sequence groups' copies overlapping the
    # computation) gives the device entry's output bit for bit
    from mk_iii_technologies_tsrn_b200 import ops
    Q, K, V, slopes = _case(5, 3, 70, 6, 24, seed=9)
    hQ, hK, hV = (torch.tensor(a).pin_memory() for a in (Q, K, V))
    got = ops.tsrn_attention_host(hQ, hK, hV, torch.tensor(slopes), 6, True, 6, chunks=chunks)
    torch.cuda.synchronize()
    ref = ops.tsrn_attention(*(torch.tensor(a, device=cuda) for a in (Q, K, V, slopes)), 6, True, 6)
    assert not got.is_cuda
    assert torch.equal(got, ref.cpu())
    with pytest.raises(ValueError):
        ops.tsrn_attention_host(hQ.cuda(), hK, hV, torch.tensor(slopes), 6)
