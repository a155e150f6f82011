"""Echo-state reservoir recurrences (GRU-gated and leaky, whole sequence in
one cluster launch) vs the oracle and vs the reference modules' outputs
(golden fixtures).  The kernel computes in fp32 with the reference loop's
operation order per element except the dot-product summation order:
tolerance 2e-5 absolute on h in (-1, 1)."""
import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden

pytestmark = pytest.mark.gpu

TOL = 2e-5


def _inputs(rng, B, T, dr, wscale=0.15):
    U = rng.standard_normal((B, T, dr)).astype(np.float32)
    Uz = (0.85 + 0.3 * rng.standard_normal((B, T, dr))).astype(np.float32)
    Ur = (2.0 + 0.3 * rng.standard_normal((B, T, dr))).astype(np.float32)
    Wzh = (wscale / np.sqrt(dr) * rng.standard_normal((dr, dr))).astype(np.float32)
    Wrh = (wscale / np.sqrt(dr) * rng.standard_normal((dr, dr))).astype(np.float32)
    Ws = (0.9 / np.sqrt(dr) * rng.standard_normal((dr, dr))).astype(np.float32)
    return U, Uz, Ur, Wzh, Wrh, Ws


def test_esn_kernel_vs_reference_golden(cuda):
    from mk_iii_technologies_tsrn_b200 import ops
    g = load_golden("esn")
    t = lambda a: torch.tensor(a, device=cuda)
    H = ops.esn_gru_fwd(*(t(g[k]) for k in ("U", "Uz", "Ur", "Wzh", "Wrh", "Ws")))
    np.testing.assert_allclose(H.cpu().numpy(), g["H"], rtol=0, atol=TOL)


def test_esn_module_vs_reference_golden(cuda):
    from mk_iii_technologies_tsrn_b200.reservoir import EchoStateReservoir
    g = load_golden("esn")
    d = g["x"].shape[-1]
    mod = EchoStateReservoir(d, d).to(cuda).eval()
    mod.load_state_dict({k[2:]: torch.tensor(v) for k, v in g.items() if k.startswith("p_")})
    with torch.no_grad():
        y = mod(torch.tensor(g["x"], device=cuda))
    np.testing.assert_allclose(y.cpu().numpy(), g["H"], rtol=0, atol=TOL)


# shapes: tiny, ragged dr (not a multiple of 4), one CTA per cluster, weights
# in shared memory with 8 and 16 CTAs per cluster, weights read from L2
# (dr 1024 and 640 GRU), many batch groups
SHAPES = [(1, 1, 1), (3, 17, 150), (2, 5, 37), (8, 64, 640), (64, 8, 256), (4, 12, 1024),
          (130, 6, 96), (5, 9, 513)]


@pytest.mark.parametrize("B,T,dr", SHAPES)
def test_esn_kernel_vs_oracle(cuda, B, T, dr):
    from mk_iii_technologies_tsrn_b200 import ops
    rng = np.random.default_rng(B * 1000 + T + dr)
    arrs = _inputs(rng, B, T, dr)
    H = ops.esn_gru_fwd(*(torch.tensor(a, device=cuda) for a in arrs)).cpu().numpy()
    ref = oracle.esn_gru_fwd(*arrs)
    np.testing.assert_allclose(H, ref, rtol=0, atol=TOL)


@pytest.mark.parametrize("B,T,dr", SHAPES)
def test_esn_leaky_kernel_vs_oracle(cuda, B, T, dr):
    from mk_iii_technologies_tsrn_b200 import ops
    rng = np.random.default_rng(B * 1000 + T + dr + 7)
    U, _, _, _, _, Ws = _inputs(rng, B, T, dr)
    lk = np.float32(0.37)
    H = ops.esn_leaky_fwd(torch.tensor(U, device=cuda), torch.tensor(Ws, device=cuda),
                          torch.tensor(lk, device=cuda)).cpu().numpy()
    np.testing.assert_allclose(H, oracle.esn_leaky_fwd(U, Ws, lk), rtol=0, atol=TOL)


def test_esn_gru_strided_weights(cuda):
    # W_z.weight[:, :dr] passed in place (row stride 2 dr)
    from mk_iii_technologies_tsrn_b200 import ops
    rng = np.random.default_rng(5)
    B, T, dr = 6, 20, 96
    U, Uz, Ur, Wzh, Wrh, Ws = _inputs(rng, B, T, dr)
    t = lambda a: torch.tensor(a, device=cuda)
    Wz_full = torch.cat([t(Wzh), t(rng.standard_normal((dr, dr)).astype(np.float32))], 1)
    Wr_full = torch.cat([t(Wrh), t(rng.standard_normal((dr, dr)).astype(np.float32))], 1)
    H = ops.esn_gru_fwd(t(U), t(Uz), t(Ur), Wz_full[:, :dr], Wr_full[:, :dr], t(Ws))
    np.testing.assert_allclose(H.cpu().numpy(), oracle.esn_gru_fwd(U, Uz, Ur, Wzh, Wrh, Ws),
                               rtol=0, atol=TOL)


def test_esn_leaky_vs_reference_golden(cuda):
    from mk_iii_technologies_tsrn_b200 import ops
    from mk_iii_technologies_tsrn_b200.reservoir import LeakyEchoStateReservoir
    g = load_golden("esn_leaky")
    t = lambda a: torch.tensor(a, device=cuda)
    H = ops.esn_leaky_fwd(t(g["U"]), t(g["Ws"]), t(g["lk"]))
    np.testing.assert_allclose(H.cpu().numpy(), g["H"], rtol=0, atol=TOL)
    d = g["x"].shape[-1]
    mod = LeakyEchoStateReservoir(d, d).to(cuda).eval()
    mod.load_state_dict({k[2:]: torch.tensor(v) for k, v in g.items() if k.startswith("p_")})
    with torch.no_grad():
        y = mod(t(g["x"]))
    np.testing.assert_allclose(y.cpu().numpy(), g["H"], rtol=0, atol=TOL)


def test_esn_empty_sequence(cuda):
    from mk_iii_technologies_tsrn_b200 import ops
    z = torch.zeros(2, 0, 16, device=cuda)
    w = torch.zeros(16, 16, device=cuda)
    assert ops.esn_gru_fwd(z, z, z, w, w, w).shape == (2, 0, 16)


def test_esn_module_matches_training_loop(cuda):
    # the fused inference path and the autograd loop of the same module agree
    from mk_iii_technologies_tsrn_b200.reservoir import EchoStateReservoir
    torch.manual_seed(3)
    mod = EchoStateReservoir(96, 48).to(cuda)
    with torch.no_grad():
        mod.W_z.weight.normal_(0.0, 0.1)
        mod.W_r.weight.normal_(0.0, 0.1)
        mod.readout.weight.normal_(0.0, 0.1)
        mod._cached_v.normal_()
    x = torch.randn(4, 40, 96, device=cuda)
    v0 = mod._cached_v.clone()
    y_loop = mod(x)
    mod._cached_v.copy_(v0)
    with torch.no_grad():
        y_fused = mod(x)
    torch.testing.assert_close(y_fused, y_loop.detach(), rtol=0, atol=1e-4)


def test_esn_rejects_cpu_inputs():
    from mk_iii_technologies_tsrn_b200 import ops
    z = torch.zeros(1, 2, 4)
    w = torch.zeros(4, 4)
    with pytest.raises((RuntimeError, ValueError)):
        ops.esn_gru_fwd(z, z, z, w, w, w)


@pytest.mark.parametrize("gru", [True, False])
@pytest.mark.parametrize("B,T,dr", [(9, 40, 96), (64, 30, 320)])
def test_esn_segments_continue_bit_for_bit(cuda, gru, B, T, dr):
    # a sequence run as consecutive segments, each from the previous segment's
    # last state (h0), equals one launch over the whole sequence bit for bit;
    # h0 against the oracle
    from mk_iii_technologies_tsrn_b200 import ops
    rng = np.random.default_rng(B + T + dr)
    U, Uz, Ur, Wzh, Wrh, Ws = (torch.tensor(a, device=cuda) for a in _inputs(rng, B, T, dr))
    lk = torch.tensor([0.3], device=cuda)

    def run(sl, h0=None):
        if gru:
            return ops.esn_gru_fwd(U[:, sl], Uz[:, sl], Ur[:, sl], Wzh, Wrh, Ws, h0=h0)
        return ops.esn_leaky_fwd(U[:, sl], Ws, lk, h0=h0)

    whole = run(slice(0, T))
    parts, h0 = [], None
    for a, b in ((0, 7), (7, 8), (8, 25), (25, T)):
        parts.append(run(slice(a, b), h0))
        h0 = parts[-1][:, -1]
    assert torch.equal(torch.cat(parts, dim=1), whole)
    h0 = torch.tensor(rng.uniform(-0.9, 0.9, (B, dr)).astype(np.float32), device=cuda)
    got = run(slice(0, T), h0).cpu().numpy()
    if gru:
        ref = oracle.esn_gru_fwd(*(t.cpu().numpy() for t in (U, Uz, Ur, Wzh, Wrh, Ws)),
                                 h0=h0.cpu().numpy())
    else:
        ref = oracle.esn_leaky_fwd(U.cpu().numpy(), Ws.cpu().numpy(), 0.3, h0=h0.cpu().numpy())
    np.testing.assert_allclose(got, ref, rtol=0, atol=TOL)


@pytest.mark.parametrize("gru", [True, False])
@pytest.mark.parametrize("segments", [1, 3, 4])
def test_esn_host_entry_equals_device(cuda, gru, segments):
    # host-resident inputs, time windows' copies overlapping the recurrence
    from mk_iii_technologies_tsrn_b200 import ops
    rng = np.random.default_rng(21)
    U, Uz, Ur, Wzh, Wrh, Ws = _inputs(rng, 17, 50, 72)
    hU, hUz, hUr = (torch.tensor(a).pin_memory() for a in (U, Uz, Ur))
    dW = [torch.tensor(a, device=cuda) for a in (Wzh, Wrh, Ws)]
    lk = torch.tensor([0.25], device=cuda)
    if gru:
        got = ops.esn_fwd_host(hU, dW[2], Uz=hUz, Ur=hUr, Wzh=dW[0], Wrh=dW[1],
                               segments=segments)
        ref = ops.esn_gru_fwd(hU.to(cuda), hUz.to(cuda), hUr.to(cuda), *dW)
    else:
        got = ops.esn_fwd_host(hU, dW[2], lk=lk, segments=segments)
        ref = ops.esn_leaky_fwd(hU.to(cuda), dW[2], lk)
    torch.cuda.synchronize()
    assert not got.is_cuda
    assert torch.equal(got, ref.cpu())
