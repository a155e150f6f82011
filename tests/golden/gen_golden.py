"""Generate golden vectors by running the reference's own PyTorch code.

Run in a container that has the reference checkout (default
/root/reference, override with TSRN_REFERENCE):

    python tests/golden/gen_golden.py [generator ...]

Writes ``tests/golden/*.npz``.  Each fixture stores its inputs and the outputs
of the reference expression, so the tests (and the oracle pin) need nothing
but numpy at run time.  Reference modules are loaded by file path because the
installed ``cuda-python`` package shadows the reference's ``cuda/`` directory
and ``research/tsrn_dml.py`` clashes by name with the top-level ``tsrn_dml.py``.
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import torch

REF = os.environ.get("TSRN_REFERENCE", "/root/reference")
OUT = os.path.dirname(os.path.abspath(__file__))


def _load(name: str, rel: str):
    path = os.path.join(REF, rel)
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _np(t):
    return t.detach().cpu().numpy()


def _save(name: str, **arrays):
    path = os.path.join(OUT, f"{name}.npz")
    np.savez_compressed(path, **{k: (v if isinstance(v, np.ndarray) else np.asarray(v))
                                 for k, v in arrays.items()})
    print(f"wrote {path}")


def gen_kat(trop):
    # cuda/test_kernel.py:117-136, computed with the reference broadcast expression
    A = torch.tensor([[1.0, 2.0], [3.0, 0.0]])
    B = torch.tensor([[0.0, 1.0], [2.0, 0.0]])
    C = (A.unsqueeze(2) + B.unsqueeze(0)).max(dim=1)
    _save("kat_2x2", A=_np(A), B=_np(B), C=_np(C.values), idx=_np(C.indices),
          expected=np.array([[4.0, 2.0], [3.0, 4.0]], np.float32))


def _linear_case(trop, name, x, W, bias, g, ste_temp=1.0):
    layer = trop.TropicalLinear(W.shape[1], W.shape[0], bias=bias is not None)
    with torch.no_grad():
        layer.weight.copy_(W)
        if bias is not None:
            layer.bias.copy_(bias)
    old = trop.TropicalLinear._ste_temp
    trop.TropicalLinear._ste_temp = ste_temp
    try:
        out = {}
        for mode in ("eval", "train"):
            layer.train(mode == "train")
            layer.zero_grad()
            xx = x.clone().requires_grad_(True)
            y = layer(xx)
            (y * g).sum().backward()
            out[f"y_{mode}"] = _np(y)
            out[f"gx_{mode}"] = _np(xx.grad)
            out[f"gw_{mode}"] = _np(layer.weight.grad)
            if bias is not None:
                out[f"gb_{mode}"] = _np(layer.bias.grad)
        scores = W.unsqueeze(0) + x.unsqueeze(1)          # tropformer.py:131
        mx = scores.max(dim=-1)                             # tropformer.py:141
        out["max"] = _np(mx.values)
        out["idx"] = _np(mx.indices)
    finally:
        trop.TropicalLinear._ste_temp = old
    arrays = dict(x=_np(x), W=_np(W), g=_np(g), ste_temp=np.float32(ste_temp), **out)
    if bias is not None:
        arrays["bias"] = _np(bias)
    _save(name, **arrays)


def gen_linear(trop):
    # the reference's own op-level test setup (cuda/test_kernel.py:15-65): seed 42,
    # batch 8, in 64, out 32, TropicalLinear weights U(-0.5, 0.5), zero bias
    torch.manual_seed(42)
    ref = trop.TropicalLinear(64, 32, bias=True)
    torch.empty(32, 64).uniform_(-0.5, 0.5)  # the second layer's init in that test
    x = torch.randn(8, 64)
    g = torch.ones(8, 32)                    # y.sum().backward()
    _linear_case(trop, "linear_seed42", x, ref.weight.detach().clone(),
                 ref.bias.detach().clone(), g)

    # config-1 distribution at a small size, non-zero bias, random upstream grad
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(48, 40, generator=gen)
    W = torch.randn(24, 40, generator=gen)
    b = torch.randn(24, generator=gen)
    g = torch.randn(48, 24, generator=gen)
    _linear_case(trop, "linear_gauss", x, W, b, g)
    _linear_case(trop, "linear_gauss_tau05", x, W, b, g, ste_temp=0.5)

    # tie-rich: small integers, many equal sums
    gen = torch.Generator().manual_seed(1)
    x = torch.randint(-3, 4, (37, 45), generator=gen).float()
    W = torch.randint(-3, 4, (29, 45), generator=gen).float()
    g = torch.randn(37, 29, generator=gen)
    _linear_case(trop, "linear_ties", x, W, None, g)

    # -inf rich: 5% of W is -inf, one x row all -inf, one W row all -inf
    gen = torch.Generator().manual_seed(2)
    x = torch.randn(20, 33, generator=gen)
    W = torch.randn(18, 33, generator=gen)
    W[torch.rand(18, 33, generator=gen) < 0.05] = float("-inf")
    x[3] = float("-inf")
    W[5] = float("-inf")
    scores = W.unsqueeze(0) + x.unsqueeze(1)
    mx = scores.max(dim=-1)
    _save("linear_neginf", x=_np(x), W=_np(W), max=_np(mx.values), idx=_np(mx.indices))

    # NaN and +inf/-inf pairs: torch.max propagates NaN and reports the first NaN
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(9, 70, generator=gen)
    W = torch.randn(7, 70, generator=gen)
    x[1, 5] = float("nan")
    x[2, 40] = float("inf")
    W[3, 40] = float("-inf")      # inf + -inf = NaN at (2, 3, 40)
    x[4, 10] = float("nan")
    x[4, 60] = float("nan")
    W[6, 0] = float("nan")
    scores = W.unsqueeze(0) + x.unsqueeze(1)
    mx = scores.max(dim=-1)
    _save("linear_nan", x=_np(x), W=_np(W), max=_np(mx.values), idx=_np(mx.indices))


def gen_bf16(trop):
    # eval-mode TropicalLinear on bf16 weight and input (tropformer.py:131,141):
    # the reference's own bf16 arithmetic (each sum rounded to bf16).  No bias,
    # so the module output is the bf16 max itself.
    for name, seed, kind in (("linear_bf16_gauss", 10, "gauss"), ("linear_bf16_ties", 11, "ties")):
        gen = torch.Generator().manual_seed(seed)
        if kind == "gauss":
            x = torch.randn(40, 72, generator=gen) * 3.0
            w = torch.randn(24, 72, generator=gen) * 3.0
            x[2, 5] = float("nan")
            w[3, :] = float("-inf")
        else:
            x = torch.randint(-4, 5, (33, 50), generator=gen).float() * 0.25
            w = torch.randint(-4, 5, (21, 50), generator=gen).float() * 0.25
        layer = trop.TropicalLinear(x.shape[1], w.shape[0], bias=False)
        with torch.no_grad():
            layer.weight.copy_(w)
        layer = layer.bfloat16().eval()
        xb = x.bfloat16()
        with torch.no_grad():
            y = layer(xb)
            idx = (layer.weight.unsqueeze(0) + xb.unsqueeze(1)).max(dim=-1).indices
        _save(name, x=_np(xb.float()), W=_np(layer.weight.float()), max=_np(y.float()),
              idx=_np(idx))


def gen_scores(trop, dtn):
    # DTNAttention tropical score (deep_tropical_net.py:148-150): hard and smooth
    gen = torch.Generator().manual_seed(4)
    Bz, H, L, dk = 2, 4, 6, 8
    Q = torch.randn(Bz, H, L, dk, generator=gen)
    K = torch.randn(Bz, H, L, dk, generator=gen)
    gS = torch.randn(Bz, H, L, L, generator=gen)
    scale = dk ** -0.5
    out = {}
    for smooth in (False, True):
        old = trop._USE_SMOOTH_MAX
        trop._USE_SMOOTH_MAX = smooth
        try:
            q = Q.clone().requires_grad_(True)
            k = K.clone().requires_grad_(True)
            S = trop._tropical_max(q.unsqueeze(3) + k.unsqueeze(2), dim=-1) * scale
            (S * gS).sum().backward()
        finally:
            trop._USE_SMOOTH_MAX = old
        tag = "smooth" if smooth else "hard"
        out[f"S_{tag}"] = _np(S)
        out[f"gQ_{tag}"] = _np(q.grad)
        out[f"gK_{tag}"] = _np(k.grad)
    idx = (Q.unsqueeze(3) + K.unsqueeze(2)).max(dim=-1).indices
    _save("dtn_scores", Q=_np(Q), K=_np(K), gS=_np(gS), scale=np.float32(scale),
          smooth_temp=np.float32(trop._SMOOTH_MAX_TEMP), idx=_np(idx), **out)

    # full DTNAttention block (train mode: STE in the tropical Q/K projections)
    torch.manual_seed(5)
    d, heads = 32, 4
    attn = dtn.DTNAttention(d, heads, dropout=0.0)
    with torch.no_grad():
        attn.q_proj.weight.normal_(0.0, 0.02)
        attn.k_proj.weight.normal_(0.0, 0.02)
        attn.maslov.log_temps.copy_(torch.log(torch.rand(heads) * 0.9 + 0.1))
    attn.train()
    x = torch.randn(3, 7, d, requires_grad=True)
    gout = torch.randn(3, 7, d)
    out_t, w_t = attn(x)
    (out_t * gout).sum().backward()
    state = {f"p_{k}": _np(v) for k, v in attn.state_dict().items()}
    grads = {f"g_{n}": _np(p.grad) for n, p in attn.named_parameters()}
    _save("dtn_block", x=_np(x), gout=_np(gout), out=_np(out_t), attn=_np(w_t),
          gx=_np(x.grad), **state, **grads)


def gen_tsrn(research):
    # research TropicalAttention._channel_chunked_scores (research/tsrn_dml.py:438-460)
    gen = torch.Generator().manual_seed(6)
    Bz, H, T, dh = 2, 2, 12, 10
    Q = torch.randn(Bz, H, T, dh, generator=gen)
    K = torch.randn(Bz, H, T, dh, generator=gen)
    attn = research.TropicalAttention(H * dh, top_k=4, n_heads=H)
    S = attn._channel_chunked_scores(Q, K, Bz, H, T, dh)
    S64 = torch.logsumexp(Q.double().unsqueeze(3) + K.double().unsqueeze(2), dim=-1)
    _save("tsrn_scores", Q=_np(Q), K=_np(K), S=_np(S), S64=_np(S64))

    # TropicalSSM (research/tsrn_dml.py:917-980) module forward/backward with a
    # non-zero C_proj so the scan reaches the output
    torch.manual_seed(7)
    d, ds, T = 16, 8, 40
    ssm = research.TropicalSSM(d, ds)
    with torch.no_grad():
        ssm.C_proj.weight.normal_(0.0, 0.3)
        ssm.A.copy_(torch.linspace(-0.3, 0.05, ds))   # includes A > 0 (clamped to 0)
        ssm.gate_B.weight.normal_(0.0, 0.2)
    x = torch.randn(2, T, d, requires_grad=True)
    gout = torch.randn(2, T, d)
    y = ssm(x)
    (y * gout).sum().backward()
    # the scan input u and its closed-form output, for the scan-level pin
    with torch.no_grad():
        u = torch.sigmoid(ssm.gate_B(x)) * ssm.B_proj(x)
        A_c = ssm.A.clamp(max=0)
        t_idx = torch.arange(T, dtype=x.dtype).unsqueeze(-1)
        G = torch.cat([A_c.unsqueeze(0).expand(2, -1).unsqueeze(1), u - t_idx * A_c], dim=1)
        Hs = t_idx.unsqueeze(0) * A_c + G.cummax(dim=1).values[:, 1:, :]
    state = {f"p_{k}": _np(v) for k, v in ssm.state_dict().items()}
    grads = {f"g_{n}": _np(p.grad) for n, p in ssm.named_parameters()}
    _save("tsrn_ssm", x=_np(x), gout=_np(gout), y=_np(y), gx=_np(x.grad), u=_np(u),
          H=_np(Hs), A_c=_np(A_c), **state, **grads)


def gen_lfdual(trop, dtn):
    # TropicalLinear (eval, with bias) followed by LFDualActivation in each mode
    # (tropformer.py:224-289), and the two hybrid FFNs (tropformer.py:407-456,
    # deep_tropical_net.py:172-211) in eval mode with non-default parameters
    torch.manual_seed(9)
    d, ffn, M = 24, 40, 30
    x = torch.randn(M, d)
    out = {"x": _np(x)}
    lin = trop.TropicalLinear(d, ffn)
    with torch.no_grad():
        lin.weight.normal_(0.0, 0.7)
        lin.bias.normal_(0.0, 0.5)
    lin.eval()
    out["W"], out["b"] = _np(lin.weight), _np(lin.bias)
    with torch.no_grad():
        y = lin(x)
    for mode in ("primal", "dual", "blend"):
        act = trop.LFDualActivation(ffn, num_pieces=8, mode=mode)
        with torch.no_grad():
            act.slopes.add_(torch.randn(8) * 0.3)
            act.biases.normal_(0.0, 0.4)
            act.x_grid.add_(torch.randn(8) * 0.2)
            if mode == "blend":
                act.blend_gate.normal_(0.0, 1.0)
            out[f"{mode}_out"] = _np(act(y))
        out[f"{mode}_slopes"] = _np(act.slopes)
        out[f"{mode}_biases"] = _np(act.biases)
        out[f"{mode}_x_grid"] = _np(act.x_grid)
        if mode == "blend":
            out["blend_gate"] = _np(act.blend_gate)
    _save("lfdual", **out)
    for name, cls in (("ffn_tropformer", trop.TropicalHybridFFN),
                      ("ffn_dtn", dtn.DTNHybridFFN)):
        torch.manual_seed(10)
        ffn_mod = cls(d, ffn)
        with torch.no_grad():
            for pname, prm in ffn_mod.named_parameters():
                if "lf_act" in pname or "gate_proj" in pname:
                    prm.add_(torch.randn_like(prm) * 0.3)
        ffn_mod.eval()
        xx = torch.randn(2, 7, d)
        with torch.no_grad():
            yy = ffn_mod(xx)
        state = {f"p_{k}": _np(v) for k, v in ffn_mod.state_dict().items()}
        _save(name, x=_np(xx), out=_np(yy), **state)


def gen_esn(research):
    # research EchoStateReservoir (research/tsrn_dml.py:736-843), eval: d_model =
    # d_reservoir and readout = identity, so the output is the state sequence H.
    # _cached_v is set before the forward so the power iteration draws no
    # random numbers; the recurrence inputs are computed by the module's own parts.
    import copy
    torch.manual_seed(11)
    d = 24
    esn = research.EchoStateReservoir(d, d)
    with torch.no_grad():
        esn.W_z.weight.normal_(0.0, 0.15)
        esn.W_r.weight.normal_(0.0, 0.15)
        esn.log_rho.fill_(0.4)
        esn.readout.weight.copy_(torch.eye(d))
        esn._cached_v.copy_(torch.randn(d))
    esn.eval()
    x = torch.randn(2, 30, d)
    # copies: the forward updates _cached_v in place
    state = {f"p_{k}": _np(v).copy() for k, v in esn.state_dict().items()}
    with torch.no_grad():
        probe = copy.deepcopy(esn)
        rho_target = torch.sigmoid(probe.log_rho) * 1.5
        rho_current = probe._power_iter_spectral_radius(probe.W_res)
        W_scaled = probe.W_res * (rho_target / rho_current.clamp(min=1e-6))
        U = probe.W_in(x)
        Uz = U @ probe.W_z.weight[:, d:].T + probe.W_z.bias
        Ur = U @ probe.W_r.weight[:, d:].T + probe.W_r.bias
        H = esn(x)
    _save("esn", x=_np(x), H=_np(H), U=_np(U), Uz=_np(Uz), Ur=_np(Ur),
          Wzh=_np(esn.W_z.weight[:, :d]), Wrh=_np(esn.W_r.weight[:, :d]), Ws=_np(W_scaled),
          **state)


def gen_esn_leaky(tsrn_gpu):
    # leaky EchoStateReservoir of tsrn_gpu.py (:435-487), eval; d_model =
    # d_reservoir, readout = identity, so the output is the state sequence H.
    torch.manual_seed(12)
    d = 24
    esn = tsrn_gpu.EchoStateReservoir(d, d)
    with torch.no_grad():
        esn.log_rho.fill_(0.4)
        esn.leak.fill_(-0.6)
        esn.readout.weight.copy_(torch.eye(d))
    esn.eval()
    x = torch.randn(2, 30, d)
    state = {f"p_{k}": _np(v).copy() for k, v in esn.state_dict().items()}
    with torch.no_grad():
        rho = torch.sigmoid(esn.log_rho) * 1.5
        eigs = torch.linalg.eigvals(esn.W_res).abs()
        W_scaled = esn.W_res * (rho / (eigs.max().real.clamp(min=1e-6)))
        lk = torch.sigmoid(esn.leak)
        U = esn.W_in(x)
        H = esn(x)
    _save("esn_leaky", x=_np(x), H=_np(H), U=_np(U), Ws=_np(W_scaled), lk=_np(lk), **state)


def gen_real_weights(trop, research):
    # Trained weights shipped with the reference: TropFormer's first hybrid FFN
    # block (tropformer_best.pt, all parameters) and the TSRN-gist attention
    # projections (checkpoints/tsrn_gist_best.pt: Wq/Wk/Wv/Wo; that checkpoint
    # predates the QK-norm, which keeps its initial identity affine).  Inputs
    # seeded; outputs from the reference modules in eval mode.
    ck = torch.load(os.path.join(REF, "tropformer_best.pt"), map_location="cpu",
                    weights_only=False)
    pre = "blocks.0.ffn."
    sub = {k[len(pre):]: v for k, v in ck.items() if k.startswith(pre)}
    torch.manual_seed(13)
    ffn = trop.TropicalHybridFFN(128, 256)
    ffn.load_state_dict(sub, strict=True)
    ffn.eval()
    x = torch.randn(4, 17, 128)
    with torch.no_grad():
        out = ffn(x)
    _save("real_ffn_tropformer", x=_np(x), out=_np(out),
          **{f"p_{k}": _np(v).copy() for k, v in ffn.state_dict().items()})

    gk = torch.load(os.path.join(REF, "checkpoints", "tsrn_gist_best.pt"), map_location="cpu",
                    weights_only=False)
    pre = "s1_blocks.0.attn."
    sub = {k[len(pre):]: v for k, v in gk["model_state_dict"].items() if k.startswith(pre)}
    cfg = gk["config"]
    torch.manual_seed(14)
    d, heads, top_k = cfg["d_model"], cfg["n_heads"], cfg["top_k"]
    attn = research.TropicalAttention(d, top_k=top_k, n_heads=heads)
    missing, unexpected = attn.load_state_dict(sub, strict=False)
    assert not unexpected and {"Wq.weight", "Wk.weight", "Wv.weight", "Wo.weight"} & set(sub)
    attn.eval()
    B, T = 2, cfg["context_len"]
    x = torch.randn(B, T, d)
    with torch.no_grad():
        out = attn(x)
        dh = d // heads
        Q = attn.q_norm(attn.Wq(x).view(B, T, heads, dh).permute(0, 2, 1, 3))
        K = attn.k_norm(attn.Wk(x).view(B, T, heads, dh).permute(0, 2, 1, 3))
        V = attn.Wv(x).view(B, T, heads, dh).permute(0, 2, 1, 3)
        Q, K = attn.rope(Q, K)
    _save("real_attention_gist", x=_np(x), out=_np(out), Q=_np(Q), K=_np(K), V=_np(V),
          slopes=_np(attn.alibi_slopes), top_k=np.int64(top_k), n_heads=np.int64(heads),
          **{f"p_{k}": _np(v).copy() for k, v in attn.state_dict().items()})


def gen_dropin(dropin):
    # tropformer_dropin.py modules in eval mode (dropout 0): the hybrid
    # attention (self and cross, masks, KV-cache decoding), an encoder-decoder
    # transformer, a causal LM; and training-mode gradients of an encoder layer
    torch.manual_seed(15)
    d, heads = 32, 4

    def liven(mod):   # gates away from their initial constants, so both score kinds count
        with torch.no_grad():
            for name, prm in mod.named_parameters():
                if "score_gate" in name or "gate_proj" in name or "lf_act" in name:
                    prm.add_(torch.randn_like(prm) * 0.5)
        return mod

    out = {}
    sa = liven(dropin.TropicalMultiHeadAttention(d, heads, dropout=0.0)).eval()
    ca = liven(dropin.TropicalMultiHeadAttention(d, heads, dropout=0.0,
                                                 is_cross_attention=True)).eval()
    x = torch.randn(2, 7, d)
    mem = torch.randn(2, 5, d)
    mask = dropin.make_causal_mask(7, torch.device("cpu"))
    pad = torch.zeros(2, 7, dtype=torch.bool)
    pad[1, 5:] = True
    with torch.no_grad():
        out["sa_out"] = _np(sa(x, x, x, attn_mask=mask, key_padding_mask=pad)[0])
        out["ca_out"] = _np(ca(x, mem, mem)[0])
        cache = dropin.TropicalKVCache()
        out["kv_out1"] = _np(sa(x[:, :4], x[:, :4], x[:, :4], cache=cache)[0])
        out["kv_out2"] = _np(sa(x[:, 4:5], x[:, 4:5], x[:, 4:5], cache=cache)[0])
    out.update({f"psa_{k}": _np(v).copy() for k, v in sa.state_dict().items()})
    out.update({f"pca_{k}": _np(v).copy() for k, v in ca.state_dict().items()})
    _save("dropin_attention", x=_np(x), mem=_np(mem), pad=pad.numpy(), **out)

    torch.manual_seed(16)
    tr = liven(dropin.TropicalTransformer(d_model=d, nhead=heads, num_encoder_layers=2,
                                          num_decoder_layers=2, dim_feedforward=64,
                                          dropout=0.0)).eval()
    src, tgt = torch.randn(2, 6, d), torch.randn(2, 5, d)
    with torch.no_grad():
        y = tr(src, tgt, tgt_mask=dropin.make_causal_mask(5, torch.device("cpu")))
    _save("dropin_transformer", src=_np(src), tgt=_np(tgt), out=_np(y),
          **{f"p_{k}": _np(v).copy() for k, v in tr.state_dict().items()})

    torch.manual_seed(17)
    lm = liven(dropin.TropicalDecoderModel(50, d_model=d, nhead=heads, num_layers=2,
                                           dim_feedforward=64, dropout=0.0,
                                           max_seq_len=16)).eval()
    ids = torch.randint(0, 50, (2, 9))
    with torch.no_grad():
        logits = lm(ids)
    _save("dropin_lm", ids=ids.numpy(), logits=_np(logits),
          **{f"p_{k}": _np(v).copy() for k, v in lm.state_dict().items()})

    torch.manual_seed(18)
    enc = liven(dropin.TropicalEncoderLayer(d, heads, dim_feedforward=64, dropout=0.0))
    enc.train()
    xe = torch.randn(2, 6, d)
    state = {f"p_{k}": _np(v).copy() for k, v in enc.state_dict().items()}
    enc(xe).square().sum().backward()
    grads = {f"g_{k}": _np(p.grad) for k, p in enc.named_parameters()}
    _save("dropin_encoder_grad", x=_np(xe), **state, **grads)


def gen_tsrn_attention(research):
    # research TropicalAttention (research/tsrn_dml.py:355-548), eval, causal,
    # fast path: the module output, the Wo input (the attention context) and
    # the rotated Q/K/V computed by the module's own sub-modules
    torch.manual_seed(8)
    d, heads, top_k, B, T = 32, 4, 6, 2, 40
    attn = research.TropicalAttention(d, top_k=top_k, n_heads=heads)
    with torch.no_grad():
        attn.q_norm.weight.uniform_(0.5, 1.5)
        attn.k_norm.bias.uniform_(-0.2, 0.2)
    attn.eval()
    x = torch.randn(B, T, d)
    with torch.no_grad():
        out = attn(x).clone()
        # the attention context (Wo's input): the same forward with Wo = identity
        wo = attn.Wo.weight.detach().clone()
        attn.Wo.weight.copy_(torch.eye(d))
        ctx = attn(x).clone()
        attn.Wo.weight.copy_(wo)
        dh = d // heads
        Q = attn.q_norm(attn.Wq(x).view(B, T, heads, dh).permute(0, 2, 1, 3))
        K = attn.k_norm(attn.Wk(x).view(B, T, heads, dh).permute(0, 2, 1, 3))
        V = attn.Wv(x).view(B, T, heads, dh).permute(0, 2, 1, 3)
        Q, K = attn.rope(Q, K)
    ctx = ctx.view(B, T, heads, dh).permute(0, 2, 1, 3)
    state = {f"p_{k}": _np(v) for k, v in attn.state_dict().items()}
    _save("tsrn_attention", x=_np(x), out=_np(out), Q=_np(Q), K=_np(K), V=_np(V),
          ctx=_np(ctx), slopes=_np(attn.alibi_slopes), top_k=np.int64(top_k), **state)


def gen_tsrn_block(research):
    # the tropical branches of research TSRNBlock (research/tsrn_dml.py:1050-1110),
    # eval: x + attn(ln_attn(x)), then + reservoir(ln_res(.)), then
    # + tropical_ssm(ln_ssm(.)) -- the block's order without the sheaf, FFN and
    # p-adic branches between them -- each by the block's own sub-modules.
    # Inputs are redrawn until no attention row has a near-tie at its top-k cut.
    import copy
    d, heads, top_k, B, T = 48, 4, 4, 2, 36
    for seed in range(12, 40):
        torch.manual_seed(seed)
        blk = research.TSRNBlock(d, top_k=top_k, n_heads=heads, sheaf_window=4, mem_depth=3,
                                 use_reservoir=True, use_padic_attn=False, use_memory=False,
                                 use_tropical_ssm=True, dropout=0.0)
        with torch.no_grad():
            for ln in (blk.ln_attn, blk.ln_res, blk.ln_ssm):
                ln.weight.uniform_(0.6, 1.4)
                ln.bias.uniform_(-0.2, 0.2)
            blk.attn.Wo.weight.normal_(0.0, 0.2)
            r = blk.reservoir
            r.W_z.weight.normal_(0.0, 0.15)
            r.W_r.weight.normal_(0.0, 0.15)
            r.log_rho.fill_(0.4)
            r.readout.weight.normal_(0.0, 0.3)
            r._cached_v.copy_(torch.randn(r.dr if hasattr(r, "dr") else r.W_res.shape[0]))
            m = blk.tropical_ssm
            m.C_proj.weight.normal_(0.0, 0.3)
            m.A.copy_(torch.linspace(-0.3, 0.05, m.A.numel()))
            m.gate_B.weight.normal_(0.0, 0.2)
            m.gate_out.weight.normal_(0.0, 0.2)
        blk.eval()
        x = torch.randn(B, T, d)
        state = {f"p_{k}": _np(v).copy() for k, v in blk.state_dict().items()}
        with torch.no_grad():
            probe = copy.deepcopy(blk)
            xa = probe.ln_attn(x)
            Bq, H, dh = B, heads, d // heads
            Q = probe.attn.q_norm(probe.attn.Wq(xa).view(Bq, T, H, dh).permute(0, 2, 1, 3))
            K = probe.attn.k_norm(probe.attn.Wk(xa).view(Bq, T, H, dh).permute(0, 2, 1, 3))
            Q, K = probe.attn.rope(Q, K)
            S = torch.logsumexp(Q.double().unsqueeze(3) + K.double().unsqueeze(2), dim=-1)
            pos = torch.arange(T)
            S = S - probe.attn.alibi_slopes.double().view(-1, 1, 1) * \
                (pos[:, None] - pos[None, :]).abs()
            S = S.masked_fill((pos[None, :] > pos[:, None])[None, None], float("-inf"))
            srt = S.sort(dim=-1, descending=True).values
            kk = min(top_k, T)
            gap = (srt[..., kk - 1] - srt[..., kk]).abs()
            if torch.nan_to_num(gap, nan=1.0, posinf=1.0).min() < 2e-4:
                continue
            y1 = x + blk.attn(blk.ln_attn(x))
            y2 = y1 + blk.reservoir(blk.ln_res(y1))
            y3 = y2 + blk.tropical_ssm(blk.ln_ssm(y2))
        _save("tsrn_block", x=_np(x), y_attn=_np(y1), y_res=_np(y2), y=_np(y3),
              d=np.int64(d), heads=np.int64(heads), top_k=np.int64(top_k), seed=np.int64(seed),
              **state)
        return
    raise RuntimeError("no seed without a top-k near-tie")


GENERATORS = ("kat", "linear", "bf16", "lfdual", "scores", "tsrn", "tsrn_attention", "esn",
              "esn_leaky", "real_weights", "dropin", "tsrn_block")


def main():
    only = set(sys.argv[1:])
    if only - set(GENERATORS):
        raise SystemExit(f"unknown generators {sorted(only - set(GENERATORS))}; "
                         f"choose from {GENERATORS}")
    sys.path.insert(0, REF)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    trop = _load("tropformer", "tropformer.py")
    dtn = _load("deep_tropical_net", "deep_tropical_net.py")
    research = _load("research_tsrn_dml", "research/tsrn_dml.py")
    tsrn_gpu = _load("tsrn_gpu", "tsrn_gpu.py")
    dropin = _load("tropformer_dropin", "tropformer_dropin.py")
    jobs = {"kat": lambda: gen_kat(trop), "linear": lambda: gen_linear(trop),
            "bf16": lambda: gen_bf16(trop), "lfdual": lambda: gen_lfdual(trop, dtn),
            "scores": lambda: gen_scores(trop, dtn), "tsrn": lambda: gen_tsrn(research),
            "tsrn_attention": lambda: gen_tsrn_attention(research),
            "esn": lambda: gen_esn(research), "esn_leaky": lambda: gen_esn_leaky(tsrn_gpu),
            "real_weights": lambda: gen_real_weights(trop, research),
            "dropin": lambda: gen_dropin(dropin),
            "tsrn_block": lambda: gen_tsrn_block(research)}
    for name in GENERATORS:          # every fixture unless some are named
        if not only or name in only:
            jobs[name]()


if __name__ == "__main__":
    main()
