"""Host-side checks of the drop-in modules (no GPU): names, parameters and
state-dict layout match the reference's (from the golden fixtures), and CPU
inputs are refused rather than silently computed on the CPU."""
import numpy as np
import pytest
import torch

from conftest import load_golden


def _golden_state(name):
    g = load_golden(name)
    return {k[2:]: v for k, v in g.items() if k.startswith("p_")}


def test_dtn_state_dict_matches_reference():
    from mk_iii_technologies_tsrn_b200.dtn import DTNAttention
    ref = _golden_state("dtn_block")
    mod = DTNAttention(32, 4, dropout=0.0)
    ours = mod.state_dict()
    assert set(ours) == set(ref)
    for k, v in ref.items():
        assert tuple(ours[k].shape) == v.shape, k
    mod.load_state_dict({k: torch.tensor(v) for k, v in ref.items()})


def test_ssm_state_dict_matches_reference():
    from mk_iii_technologies_tsrn_b200.ssm import TropicalSSM
    ref = _golden_state("tsrn_ssm")
    mod = TropicalSSM(16, 8)
    ours = mod.state_dict()
    assert set(ours) == set(ref)
    for k, v in ref.items():
        assert tuple(ours[k].shape) == v.shape, k


def test_tropical_linear_surface():
    from mk_iii_technologies_tsrn_b200.tropical import TropicalLinear
    from mk_iii_technologies_tsrn_b200.maxplus_binding import CUDATropicalLinear
    assert TropicalLinear._ste_temp == 1.0
    for cls, kw in ((TropicalLinear, {}), (CUDATropicalLinear, {"ste_temp": 1.0})):
        layer = cls(64, 32, bias=True, **kw)
        assert set(layer.state_dict()) == {"weight", "bias"}
        assert layer.weight.shape == (32, 64) and layer.bias.shape == (32,)
        assert float(layer.weight.min()) >= -0.5 and float(layer.weight.max()) <= 0.5
        assert torch.all(layer.bias == 0)
        assert cls(8, 4, bias=False).bias is None


def test_cpu_inputs_are_refused():
    from mk_iii_technologies_tsrn_b200.tropical import TropicalLinear
    layer = TropicalLinear(8, 4)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        layer(torch.randn(2, 8))


def test_is_cuda_kernel_available_without_gpu():
    from mk_iii_technologies_tsrn_b200.maxplus_binding import is_cuda_kernel_available
    assert is_cuda_kernel_available() == torch.cuda.is_available()


def test_tsrn_attention_state_dict_matches_reference():
    # same parameter and buffer names as research TropicalAttention
    from conftest import load_golden
    from mk_iii_technologies_tsrn_b200.tsrn_attention import TropicalAttention
    g = load_golden("tsrn_attention")
    ref_keys = sorted(k[2:] for k in g.keys() if k.startswith("p_"))
    m = TropicalAttention(32, top_k=6, n_heads=4)
    assert sorted(m.state_dict().keys()) == ref_keys
    m.load_state_dict({k: torch.tensor(g["p_" + k]) for k in ref_keys})
    np.testing.assert_allclose(m.alibi_slopes.numpy(), g["slopes"])


@pytest.mark.parametrize("name,cls", [("ffn_tropformer", "TropicalHybridFFN"),
                                      ("ffn_dtn", "DTNHybridFFN")])
def test_hybrid_ffn_state_dict_matches_reference(name, cls):
    from conftest import load_golden
    from mk_iii_technologies_tsrn_b200 import dtn, tropical
    g = load_golden(name)
    mod = (tropical.TropicalHybridFFN if cls == "TropicalHybridFFN" else dtn.DTNHybridFFN)(24, 40)
    ref_keys = sorted(k[2:] for k in g.keys() if k.startswith("p_"))
    assert sorted(mod.state_dict().keys()) == ref_keys
    mod.load_state_dict({k: torch.tensor(g["p_" + k]) for k in ref_keys})


def test_reservoir_state_dict_matches_reference():
    from mk_iii_technologies_tsrn_b200.reservoir import EchoStateReservoir
    ref = _golden_state("esn")
    d = ref["W_in.weight"].shape[1]
    mod = EchoStateReservoir(d, d)
    ours = mod.state_dict()
    assert set(ours) == set(ref)
    for k, v in ref.items():
        assert tuple(ours[k].shape) == v.shape, k
    mod.load_state_dict({k: torch.tensor(v) for k, v in ref.items()})


def test_leaky_reservoir_state_dict_matches_reference():
    from mk_iii_technologies_tsrn_b200.reservoir import LeakyEchoStateReservoir
    ref = _golden_state("esn_leaky")
    d = ref["W_in.weight"].shape[1]
    mod = LeakyEchoStateReservoir(d, d)
    assert set(mod.state_dict()) == set(ref)
    mod.load_state_dict({k: torch.tensor(v) for k, v in ref.items()})


@pytest.mark.parametrize("which", ["gru", "leaky", "attention"])
def test_tsrn_modules_refuse_cpu_inputs(which):
    # the reservoirs and the attention run only on the CUDA kernels, in training too
    from mk_iii_technologies_tsrn_b200.reservoir import (EchoStateReservoir,
                                                          LeakyEchoStateReservoir)
    from mk_iii_technologies_tsrn_b200.tsrn_attention import TropicalAttention
    mod = {"gru": lambda: EchoStateReservoir(8, 8), "leaky": lambda: LeakyEchoStateReservoir(8, 8),
           "attention": lambda: TropicalAttention(8, top_k=2, n_heads=2)}[which]()
    x = torch.randn(1, 5, 8)
    for grad in (False, True):
        with torch.set_grad_enabled(grad), pytest.raises(RuntimeError):
            mod(x)


def test_real_weight_state_dicts_load():
    # the reference's trained checkpoints (via the fixtures) load into the drop-ins
    from mk_iii_technologies_tsrn_b200.tropical import TropicalHybridFFN
    from mk_iii_technologies_tsrn_b200.tsrn_attention import TropicalAttention
    ffn = _golden_state("real_ffn_tropformer")
    mod = TropicalHybridFFN(128, 256)
    assert set(mod.state_dict()) == set(ffn)
    mod.load_state_dict({k: torch.tensor(v) for k, v in ffn.items()})
    att = _golden_state("real_attention_gist")
    m = TropicalAttention(128, top_k=8, n_heads=2)
    assert set(m.state_dict()) == set(att)
    m.load_state_dict({k: torch.tensor(v) for k, v in att.items()})


@pytest.mark.parametrize("name,build", [
    ("dropin_transformer", lambda d: d.TropicalTransformer(
        d_model=32, nhead=4, num_encoder_layers=2, num_decoder_layers=2,
        dim_feedforward=64, dropout=0.0)),
    ("dropin_lm", lambda d: d.TropicalDecoderModel(
        50, d_model=32, nhead=4, num_layers=2, dim_feedforward=64, dropout=0.0, max_seq_len=16)),
    ("dropin_encoder_grad", lambda d: d.TropicalEncoderLayer(32, 4, dim_feedforward=64,
                                                            dropout=0.0)),
])
def test_dropin_state_dicts_match_reference(name, build):
    from mk_iii_technologies_tsrn_b200 import dropin
    ref = _golden_state(name)
    mod = build(dropin)
    assert set(mod.state_dict()) == set(ref)
    mod.load_state_dict({k: torch.tensor(v) for k, v in ref.items()})


def test_dropin_kv_cache_appends():
    from mk_iii_technologies_tsrn_b200.dropin import TropicalKVCache
    c = TropicalKVCache()
    k1, v1 = c.update(torch.zeros(1, 2, 3, 4), torch.ones(1, 2, 3, 4))
    k2, v2 = c.update(torch.zeros(1, 2, 1, 4), torch.ones(1, 2, 1, 4))
    assert k2.shape == (1, 2, 4, 4) and v2.shape == (1, 2, 4, 4)
    c.reset()
    assert c.k is None and c.v is None


def test_swap_into_replaces_foreign_branches():
    # a block whose attn / reservoir / tropical_ssm are foreign classes with the
    # reference attribute layout: swap_into installs this library's modules with
    # the same parameters and buffers, and leaves other attributes alone
    import copy
    import torch.nn as nn
    from mk_iii_technologies_tsrn_b200.tsrn_block import TSRNTropicalPath, swap_into
    from mk_iii_technologies_tsrn_b200.tsrn_attention import TropicalAttention
    from mk_iii_technologies_tsrn_b200.reservoir import EchoStateReservoir
    from mk_iii_technologies_tsrn_b200.ssm import TropicalSSM
    torch.manual_seed(0)
    src = TSRNTropicalPath(32, top_k=4, n_heads=4)
    blk = nn.Module()
    for name in ("attn", "reservoir", "tropical_ssm"):
        foreign = copy.deepcopy(getattr(src, name))
        foreign.__class__ = type("Foreign" + name, (nn.Module,), {})
        setattr(blk, name, foreign)
    blk.sheaf = nn.Linear(3, 3)
    sheaf = blk.sheaf
    with torch.no_grad():
        blk.attn.Wq.weight.add_(1.0)
    swap_into(blk)
    assert isinstance(blk.attn, TropicalAttention)
    assert isinstance(blk.reservoir, EchoStateReservoir)
    assert isinstance(blk.tropical_ssm, TropicalSSM)
    assert blk.sheaf is sheaf
    assert torch.equal(blk.attn.Wq.weight, src.attn.Wq.weight + 1.0)
    for name in ("reservoir", "tropical_ssm"):
        for k, v in getattr(src, name).state_dict().items():
            assert torch.equal(getattr(blk, name).state_dict()[k], v), (name, k)
