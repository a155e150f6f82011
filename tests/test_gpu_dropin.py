"""tropformer_dropin.py drop-ins (dropin.py) vs the reference modules' outputs
(golden fixtures): hybrid attention with masks and KV-cache decoding, a full
encoder-decoder transformer, a causal LM, and training-mode gradients of an
encoder layer.  The tropical scores and max-plus projections are exact; the
classical matmuls, softmax and layer norms differ from the CPU reference in
summation order only: tolerance 1e-4 (outputs), 1e-3 relative (gradients)."""
import numpy as np
import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu


def _state(g, prefix):
    return {k[len(prefix):]: torch.tensor(v) for k, v in g.items() if k.startswith(prefix)}


def test_attention_self_cross_and_kv_cache(cuda):
    from mk_iii_technologies_tsrn_b200 import dropin
    g = load_golden("dropin_attention")
    t = lambda a: torch.tensor(a, device=cuda)
    sa = dropin.TropicalMultiHeadAttention(32, 4, dropout=0.0)
    sa.load_state_dict(_state(g, "psa_"))
    ca = dropin.TropicalMultiHeadAttention(32, 4, dropout=0.0, is_cross_attention=True)
    ca.load_state_dict(_state(g, "pca_"))
    sa, ca = sa.to(cuda).eval(), ca.to(cuda).eval()
    x, mem, pad = t(g["x"]), t(g["mem"]), t(g["pad"])
    mask = dropin.make_causal_mask(7, cuda)
    with torch.no_grad():
        y = sa(x, x, x, attn_mask=mask, key_padding_mask=pad)[0]
        yc = ca(x, mem, mem)[0]
        cache = dropin.TropicalKVCache()
        y1 = sa(x[:, :4], x[:, :4], x[:, :4], cache=cache)[0]
        y2 = sa(x[:, 4:5], x[:, 4:5], x[:, 4:5], cache=cache)[0]
    assert cache.k.shape[2] == 5
    for got, key in ((y, "sa_out"), (yc, "ca_out"), (y1, "kv_out1"), (y2, "kv_out2")):
        np.testing.assert_allclose(got.cpu().numpy(), g[key], rtol=1e-4, atol=1e-4, err_msg=key)


def test_transformer_matches_reference(cuda):
    from mk_iii_technologies_tsrn_b200 import dropin
    g = load_golden("dropin_transformer")
    tr = dropin.TropicalTransformer(d_model=32, nhead=4, num_encoder_layers=2,
                                    num_decoder_layers=2, dim_feedforward=64, dropout=0.0)
    tr.load_state_dict(_state(g, "p_"))
    tr = tr.to(cuda).eval()
    with torch.no_grad():
        y = tr(torch.tensor(g["src"], device=cuda), torch.tensor(g["tgt"], device=cuda),
               tgt_mask=dropin.make_causal_mask(5, cuda))
    np.testing.assert_allclose(y.cpu().numpy(), g["out"], rtol=1e-4, atol=1e-4)


def test_decoder_lm_matches_reference(cuda):
    from mk_iii_technologies_tsrn_b200 import dropin
    g = load_golden("dropin_lm")
    lm = dropin.TropicalDecoderModel(50, d_model=32, nhead=4, num_layers=2,
                                     dim_feedforward=64, dropout=0.0, max_seq_len=16)
    lm.load_state_dict(_state(g, "p_"))
    lm = lm.to(cuda).eval()
    with torch.no_grad():
        logits = lm(torch.tensor(g["ids"], device=cuda))
    np.testing.assert_allclose(logits.cpu().numpy(), g["logits"], rtol=1e-4, atol=1e-4)


def test_encoder_layer_training_gradients(cuda):
    # train mode: STE backward of the tropical projection, argmax backward of the
    # tropical score, autograd for the rest
    from mk_iii_technologies_tsrn_b200 import dropin
    g = load_golden("dropin_encoder_grad")
    enc = dropin.TropicalEncoderLayer(32, 4, dim_feedforward=64, dropout=0.0)
    enc.load_state_dict(_state(g, "p_"))
    enc = enc.to(cuda).train()
    enc(torch.tensor(g["x"], device=cuda)).square().sum().backward()
    for name, p in enc.named_parameters():
        ref = g["g_" + name]
        np.testing.assert_allclose(p.grad.cpu().numpy(), ref, rtol=1e-3,
                                   atol=1e-3 * max(1.0, float(np.abs(ref).max())), err_msg=name)
