"""Drop-in modules on the GPU vs the reference modules' own outputs (golden)."""
import numpy as np
import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu


def _state(g):
    return {k[2:]: torch.tensor(v) for k, v in g.items() if k.startswith("p_")}


@pytest.mark.parametrize("cls_name", ["tropical.TropicalLinear",
                                      "maxplus_binding.CUDATropicalLinear"])
@pytest.mark.parametrize("train", [False, True])
def test_linear_modules_golden(cuda, cls_name, train):
    import importlib
    mod_name, cls = cls_name.split(".")
    cls = getattr(importlib.import_module(f"mk_iii_technologies_tsrn_b200.{mod_name}"), cls)
    g = load_golden("linear_seed42")
    layer = cls(64, 32, bias=True).to(cuda)
    with torch.no_grad():
        layer.weight.copy_(torch.tensor(g["W"]))
        layer.bias.copy_(torch.tensor(g["bias"]))
    layer.train(train)
    x = torch.tensor(g["x"], device=cuda, requires_grad=True)
    y = layer(x)
    (y * torch.tensor(g["g"], device=cuda)).sum().backward()
    tag = "train" if train else "eval"
    np.testing.assert_array_equal(y.detach().cpu().numpy(), g[f"y_{tag}"])
    np.testing.assert_allclose(x.grad.cpu().numpy(), g[f"gx_{tag}"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(layer.weight.grad.cpu().numpy(), g[f"gw_{tag}"],
                               rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(layer.bias.grad.cpu().numpy(), g[f"gb_{tag}"],
                               rtol=1e-5, atol=1e-5)


def test_leading_dims(cuda):
    # cuda/test_kernel.py:68-90
    from mk_iii_technologies_tsrn_b200.maxplus_binding import CUDATropicalLinear
    layer = CUDATropicalLinear(32, 16).to(cuda)
    for shape in ((4, 32), (4, 10, 32), (2, 3, 5, 32)):
        assert layer(torch.randn(*shape, device=cuda)).shape == shape[:-1] + (16,)


def test_dtn_block_golden(cuda):
    from mk_iii_technologies_tsrn_b200.dtn import DTNAttention
    g = load_golden("dtn_block")
    attn = DTNAttention(32, 4, dropout=0.0).to(cuda)
    attn.load_state_dict(_state(g))
    attn.train()
    x = torch.tensor(g["x"], device=cuda, requires_grad=True)
    out, w = attn(x)
    (out * torch.tensor(g["gout"], device=cuda)).sum().backward()
    np.testing.assert_allclose(out.detach().cpu().numpy(), g["out"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(w.detach().cpu().numpy(), g["attn"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(x.grad.cpu().numpy(), g["gx"], rtol=1e-4, atol=1e-5)
    for n, p in attn.named_parameters():
        np.testing.assert_allclose(p.grad.cpu().numpy(), g[f"g_{n}"], rtol=1e-3, atol=1e-5,
                                   err_msg=n)


def test_ssm_module_golden(cuda):
    # the reference evaluates the scan by a closed form; ours is the exact
    # recurrence, equal up to O(T ulp)
    from mk_iii_technologies_tsrn_b200.ssm import TropicalSSM
    g = load_golden("tsrn_ssm")
    ssm = TropicalSSM(16, 8).to(cuda)
    ssm.load_state_dict(_state(g))
    x = torch.tensor(g["x"], device=cuda, requires_grad=True)
    y = ssm(x)
    (y * torch.tensor(g["gout"], device=cuda)).sum().backward()
    np.testing.assert_allclose(y.detach().cpu().numpy(), g["y"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(x.grad.cpu().numpy(), g["gx"], rtol=1e-4, atol=1e-5)
    for n, p in ssm.named_parameters():
        np.testing.assert_allclose(p.grad.cpu().numpy(), g[f"g_{n}"], rtol=1e-3, atol=1e-5,
                                   err_msg=n)
