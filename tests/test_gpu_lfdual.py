"""Tropical linear + LFDualActivation fused into the forward epilogue, and the
hybrid FFNs built on it, vs the reference (golden) and the oracle."""
import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", ["primal", "dual", "blend"])
def test_fused_lfdual_vs_reference(cuda, mode):
    from mk_iii_technologies_tsrn_b200 import ops
    g = load_golden("lfdual")
    t = lambda a: torch.tensor(a, device=cuda)
    gate = torch.sigmoid(t(g["blend_gate"])) if mode == "blend" else None
    y = ops.maxplus_lfdual(t(g["x"]), t(g["W"]), t(g["b"]), mode, t(g[f"{mode}_slopes"]),
                           t(g[f"{mode}_biases"]), t(g[f"{mode}_x_grid"]), gate).cpu().numpy()
    if mode == "blend":
        np.testing.assert_allclose(y, g[f"{mode}_out"], rtol=1e-6, atol=1e-6)
    else:
        np.testing.assert_array_equal(y, g[f"{mode}_out"])


@pytest.mark.parametrize("M,N,K", [(1024, 512, 256), (300, 130, 70)])
@pytest.mark.parametrize("mode", ["primal", "dual", "blend"])
def test_fused_lfdual_shapes(cuda, M, N, K, mode):
    # (1024, 512, 256) runs the TMA kernel's value-only epilogue, the other the generic one
    from mk_iii_technologies_tsrn_b200 import ops
    rng = np.random.default_rng(M + N + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = rng.standard_normal((N, K)).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    s = np.sort(rng.standard_normal(8)).astype(np.float32)
    pb = rng.standard_normal(8).astype(np.float32)
    xg = np.linspace(-3, 3, 8).astype(np.float32)
    bg = rng.standard_normal(N).astype(np.float32)
    t = lambda a: torch.tensor(a, device=cuda)
    gate = torch.sigmoid(t(bg)) if mode == "blend" else None
    y = ops.maxplus_lfdual(t(x), t(w), t(b), mode, t(s), t(pb), t(xg), gate).cpu().numpy()
    ref = oracle.lfdual_act(oracle.maxplus_fwd(x, w, b)[0], mode, s, pb, xg, bg)
    if mode == "blend":
        np.testing.assert_allclose(y, ref, rtol=1e-6, atol=1e-6)
    else:
        np.testing.assert_array_equal(y, ref)


@pytest.mark.parametrize("name", ["ffn_tropformer", "ffn_dtn"])
def test_hybrid_ffn_matches_reference(cuda, name):
    from mk_iii_technologies_tsrn_b200 import dtn, tropical
    g = load_golden(name)
    cls = tropical.TropicalHybridFFN if name == "ffn_tropformer" else dtn.DTNHybridFFN
    mod = cls(24, 40)
    keys = [k[2:] for k in g.keys() if k.startswith("p_")]
    mod.load_state_dict({k: torch.tensor(g["p_" + k]) for k in keys})
    mod = mod.to(cuda).eval()
    x = torch.tensor(g["x"], device=cuda)
    with torch.no_grad():                       # fused inference path
        y = mod(x).cpu().numpy()
    np.testing.assert_allclose(y, g["out"], rtol=1e-5, atol=1e-5)
    y2 = mod(x).detach().cpu().numpy()          # graph-building path (module forward)
    np.testing.assert_allclose(y2, g["out"], rtol=1e-5, atol=1e-5)


def test_hybrid_ffn_real_weights(cuda):
    # TropFormer's trained first FFN block (tropformer_best.pt), reference output
    from mk_iii_technologies_tsrn_b200 import tropical
    g = load_golden("real_ffn_tropformer")
    mod = tropical.TropicalHybridFFN(128, 256)
    mod.load_state_dict({k[2:]: torch.tensor(v) for k, v in g.items() if k.startswith("p_")})
    mod = mod.to(cuda).eval()
    with torch.no_grad():
        y = mod(torch.tensor(g["x"], device=cuda)).cpu().numpy()
    np.testing.assert_allclose(y, g["out"], rtol=1e-5, atol=1e-5)
