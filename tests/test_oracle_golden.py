"""Pin the numpy oracle against golden vectors produced by the reference's own
PyTorch code (tests/golden/gen_golden.py) and its hand-computed KAT."""
import numpy as np
import pytest

import oracle
from oracle import scan as oscan

from conftest import load_golden


def test_kat_2x2():
    # cuda/test_kernel.py:117-136: C = A (x) B with B stored [K, N]
    g = load_golden("kat_2x2")
    y, idx = oracle.maxplus_fwd(g["A"], g["B"].T.copy())
    np.testing.assert_array_equal(y, g["expected"])
    np.testing.assert_array_equal(y, g["C"])
    np.testing.assert_array_equal(idx, g["idx"])


def test_kat_2x2_matmul_oracle():
    # the same KAT through the A (x) B restatement (B stored [K, N])
    g = load_golden("kat_2x2")
    y, idx = oracle.maxplus_matmul(g["A"], g["B"])
    np.testing.assert_array_equal(y, g["expected"])
    np.testing.assert_array_equal(idx, g["idx"])
    # the eigenvalue iteration on the KAT matrix, against a direct loop
    Ak, lam = oracle.tropical_power_chain(g["A"], 3)
    direct = g["A"].astype(np.float32)
    for _ in range(3):
        direct = (direct[:, :, None] + g["A"][None, :, :]).max(axis=1)
    np.testing.assert_array_equal(Ak, direct)
    assert lam == float(np.diag(direct).max() / 4)


def test_bf16_checkers_agree():
    # the large-size bf16 checker (the reference expression run by torch on
    # bf16 tensors, oracle.torch_ref) agrees with the numpy restatement, which
    # the reference fixtures pin
    import torch
    from oracle.torch_ref import maxplus_fwd_torch
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((24, 700)) * 3).astype(np.float32)
    w = (rng.standard_normal((300, 700)) * 3).astype(np.float32)
    w[rng.random(w.shape) < 0.05] = -np.inf
    ry, ri = oracle.maxplus_fwd_bf16(x, w)
    tv, ti = maxplus_fwd_torch(torch.tensor(x).bfloat16(), torch.tensor(w).bfloat16())
    np.testing.assert_array_equal(tv.float().numpy(), ry)
    np.testing.assert_array_equal(ti.numpy(), ri)


@pytest.mark.parametrize("name", ["linear_seed42", "linear_gauss", "linear_ties",
                                  "linear_neginf", "linear_nan"])
def test_forward_bit_exact(name):
    g = load_golden(name)
    y, idx = oracle.maxplus_fwd(g["x"], g["W"])
    np.testing.assert_array_equal(y, g["max"])          # NaN positions equal too
    np.testing.assert_array_equal(idx, g["idx"])


@pytest.mark.parametrize("name", ["linear_seed42", "linear_gauss", "linear_ties"])
def test_eval_forward_with_bias(name):
    g = load_golden(name)
    y, _ = oracle.maxplus_fwd(g["x"], g["W"], g.get("bias"))
    np.testing.assert_array_equal(y, g["y_eval"])
    np.testing.assert_array_equal(y, g["y_train"])     # train value = hard max too


@pytest.mark.parametrize("name", ["linear_seed42", "linear_gauss", "linear_ties"])
def test_argmax_backward(name):
    g = load_golden(name)
    _, idx = oracle.maxplus_fwd(g["x"], g["W"])
    gx, gw, gb = oracle.maxplus_bwd_argmax(idx, g["g"], g["x"].shape[1])
    np.testing.assert_allclose(gx, g["gx_eval"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(gw, g["gw_eval"], rtol=1e-6, atol=1e-5)
    if "gb_eval" in g:
        np.testing.assert_allclose(gb, g["gb_eval"], rtol=1e-6, atol=1e-5)


@pytest.mark.parametrize("name", ["linear_seed42", "linear_gauss", "linear_gauss_tau05",
                                  "linear_ties"])
def test_ste_backward(name):
    g = load_golden(name)
    tau = float(g["ste_temp"])
    gx, gw, gb = oracle.maxplus_bwd_smooth("ste", tau, g["x"], g["W"], g["g"])
    np.testing.assert_allclose(gx, g["gx_train"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(gw, g["gw_train"], rtol=1e-4, atol=1e-5)
    if "gb_train" in g:
        np.testing.assert_allclose(gb, g["gb_train"], rtol=1e-5, atol=1e-5)


def test_scores_hard_and_smooth():
    g = load_golden("dtn_scores")
    Q, K, gS, scale = g["Q"], g["K"], g["gS"], float(g["scale"])
    B, H, L, d = Q.shape
    S = np.empty((B, H, L, L), np.float32)
    gQh = np.zeros_like(Q, dtype=np.float64)
    gKh = np.zeros_like(K, dtype=np.float64)
    gQs = np.zeros_like(gQh)
    gKs = np.zeros_like(gKh)
    T = float(g["smooth_temp"])
    for b in range(B):
        for h in range(H):
            y, idx = oracle.maxplus_fwd(Q[b, h], K[b, h], scale=scale)
            S[b, h] = y
            np.testing.assert_array_equal(idx, g["idx"][b, h])
            gq, gk, _ = oracle.maxplus_bwd_argmax(idx, gS[b, h], d, scale=scale)
            gQh[b, h], gKh[b, h] = gq, gk
            gq, gk, _ = oracle.maxplus_bwd_smooth("lse", T, Q[b, h], K[b, h],
                                                  gS[b, h] * scale)
            gQs[b, h], gKs[b, h] = gq, gk
    np.testing.assert_array_equal(S, g["S_hard"])
    np.testing.assert_array_equal(S, g["S_smooth"])      # smooth STE keeps the hard value
    np.testing.assert_allclose(gQh, g["gQ_hard"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(gKh, g["gK_hard"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(gQs, g["gQ_smooth"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(gKs, g["gK_smooth"], rtol=1e-5, atol=1e-6)


def test_tsrn_lse_scores():
    g = load_golden("tsrn_scores")
    Q, K = g["Q"], g["K"]
    B, H, T, dh = Q.shape
    for b in range(B):
        for h in range(H):
            y = oracle.maxplus_lse_fwd(Q[b, h], K[b, h], 1.0)
            np.testing.assert_allclose(y, g["S64"][b, h], rtol=1e-6, atol=1e-6)
            np.testing.assert_allclose(y, g["S"][b, h], rtol=1e-5, atol=1e-5)


def test_scan_closed_form_matches_reference():
    g = load_golden("tsrn_ssm")
    H = oscan.scan_closed_form(g["u"], g["p_A"])
    np.testing.assert_array_equal(H, g["H"])


def test_scan_recurrence_vs_closed_form():
    # the reference evaluates h_t = max(A_c + h_{t-1}, u_t), h_{-1} = 0, by a closed
    # form; the sequential recurrence agrees up to O(T ulp)
    g = load_golden("tsrn_ssm")
    h, _ = oscan.scan_fwd(g["u"], g["A_c"], h_init=0.0)
    T = g["u"].shape[1]
    np.testing.assert_allclose(h, g["H"], rtol=0, atol=4 * T * np.finfo(np.float32).eps *
                               max(1.0, float(np.abs(g["H"]).max())))


def test_scan_backward_matches_torch_cummax_rule():
    # gradient of the closed form through cummax (last index on ties) equals the
    # recurrence's argmax-path gradient when the input wins ties
    import torch

    g = load_golden("tsrn_ssm")
    u = torch.tensor(g["u"], dtype=torch.float64, requires_grad=True)
    A = torch.tensor(g["A_c"], dtype=torch.float64, requires_grad=True)
    B, T, C = u.shape
    t_idx = torch.arange(T, dtype=torch.float64).unsqueeze(-1)
    G = torch.cat([A.unsqueeze(0).expand(B, -1).unsqueeze(1), u - t_idx * A], dim=1)
    H = t_idx.unsqueeze(0) * A + G.cummax(dim=1).values[:, 1:, :]
    rng = np.random.default_rng(0)
    gh = rng.standard_normal((B, T, C))
    (H * torch.tensor(gh)).sum().backward()
    hh, win = oscan.scan_fwd(g["u"].astype(np.float64), g["A_c"].astype(np.float64), 0.0)
    gu, ga, _ = oscan.scan_bwd(gh, win)
    np.testing.assert_allclose(gu, u.grad.numpy(), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(ga, A.grad.numpy(), rtol=1e-10, atol=1e-10)


def test_scan_tie_rule_input_wins():
    u = np.array([[[1.0], [0.5], [1.0], [0.0]]], np.float32)  # a = 0: ties at t=2
    a = np.zeros(1, np.float32)
    h, win = oscan.scan_fwd(u, a, -np.inf)
    np.testing.assert_array_equal(h[0, :, 0], [1.0, 1.0, 1.0, 1.0])
    np.testing.assert_array_equal(win[0, :, 0], [True, False, True, False])


def test_win_mask_packing():
    rng = np.random.default_rng(1)
    win = rng.random((2, 70, 3)) < 0.5
    words = oscan.win_mask_words(win)
    assert words.shape == (2, 3, 3)
    for t in range(70):
        bit = (words[:, t // 32, :] >> (t % 32)) & 1
        np.testing.assert_array_equal(bit.astype(bool), win[:, t, :])


@pytest.mark.parametrize("name", ["linear_bf16_gauss", "linear_bf16_ties"])
def test_bf16_arith_forward(name):
    # the reference TropicalLinear evaluated on bf16 tensors: sums rounded to bf16
    g = load_golden(name)
    y, idx = oracle.maxplus_fwd_bf16(g["x"], g["W"])
    np.testing.assert_array_equal(y, g["max"])
    np.testing.assert_array_equal(idx, g["idx"])
    # and it differs from fp32 arithmetic on the same inputs (the mode matters)
    if name == "linear_bf16_gauss":
        assert not np.array_equal(oracle.maxplus_fwd(g["x"], g["W"])[0], g["max"])


def test_round_bf16_rule():
    vals = np.array([1.0, 1.00390625, 1.005859375, 1.0078125, -2.0, np.inf, -np.inf,
                     3.4e38, 1e-40], dtype=np.float32)
    r = oracle.round_bf16(vals)
    # 1 + 2^-8 is halfway between 1 and 1 + 2^-7: ties to even -> 1
    assert r[1] == 1.0
    assert r[2] == np.float32(1.0078125)      # above halfway rounds up
    assert np.isinf(r[7])                     # beyond the largest bf16 -> inf
    assert np.isnan(oracle.round_bf16(np.array([np.nan], np.float32)))[0]


def _ambiguous_rows(S, top_k, gap=1e-4):
    """Rows whose top_k-th and next score are closer than ``gap`` (fp32 score rounding
    may then select differently) -- excluded from exact selection checks."""
    Tkv = S.shape[-1]
    k = min(top_k, Tkv)
    srt = -np.sort(-S, axis=-1)
    if k >= Tkv:
        return np.zeros(S.shape[:-1], bool)
    a, b = srt[..., k - 1], srt[..., k]
    with np.errstate(invalid="ignore"):
        return np.isfinite(a) & np.isfinite(b) & (np.abs(a - b) < gap)


def test_tsrn_attention_oracle_pinned():
    # the reference module's own attention context (Wo input), fp32
    g = load_golden("tsrn_attention")
    out, S = oracle.tsrn_attention_fwd(g["Q"], g["K"], g["V"], g["slopes"], int(g["top_k"]))
    amb = _ambiguous_rows(S, int(g["top_k"]))
    assert amb.mean() < 0.05
    ok = ~amb
    np.testing.assert_allclose(out[ok], g["ctx"][ok], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("mode", ["primal", "dual", "blend"])
def test_lfdual_oracle_pinned(mode):
    g = load_golden("lfdual")
    y, _ = oracle.maxplus_fwd(g["x"], g["W"], g["b"])
    out = oracle.lfdual_act(y, mode, g[f"{mode}_slopes"], g[f"{mode}_biases"],
                            g[f"{mode}_x_grid"], g.get("blend_gate"))
    if mode == "blend":      # sigmoid: numpy vs torch may differ in the last place
        np.testing.assert_allclose(out, g[f"{mode}_out"], rtol=1e-6, atol=1e-6)
    else:
        np.testing.assert_array_equal(out, g[f"{mode}_out"])


def test_esn_oracle_pinned():
    g = load_golden("esn")
    H = oracle.esn_gru_fwd(g["U"], g["Uz"], g["Ur"], g["Wzh"], g["Wrh"], g["Ws"])
    np.testing.assert_allclose(H, g["H"], rtol=0, atol=1e-6)


def test_esn_leaky_oracle_pinned():
    g = load_golden("esn_leaky")
    H = oracle.esn_leaky_fwd(g["U"], g["Ws"], g["lk"])
    np.testing.assert_allclose(H, g["H"], rtol=0, atol=1e-6)


def test_tsrn_block_cpu_port_pinned():
    # the CPU port timed as the config-5 block baseline reproduces the reference
    # TSRNBlock's tropical branches (fixture from the reference module)
    import torch
    from oracle.torch_ref import tsrn_block_torch
    g = load_golden("tsrn_block")
    sd = {k[2:]: torch.tensor(v) for k, v in g.items() if k.startswith("p_")}
    y = tsrn_block_torch(torch.tensor(g["x"]), sd, int(g["heads"]), int(g["top_k"]))
    np.testing.assert_allclose(y.numpy(), g["y"], rtol=1e-6, atol=1e-6)
