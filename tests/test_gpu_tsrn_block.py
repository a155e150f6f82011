"""The tropical branches of a TSRN block (research/tsrn_dml.py:1050-1110) --
attention, echo-state reservoir, tropical SSM, each a pre-LayerNorm residual
branch in the block's order -- against the reference TSRNBlock's own
sub-modules (golden fixture tsrn_block.npz, made by tests/golden/gen_golden.py
from the reference block's state dict).  The fixture's inputs have no
attention row with a near-tie at its top-k cut."""
import numpy as np
import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu


def _path(g, dev):
    from mk_iii_technologies_tsrn_b200.tsrn_block import TSRNTropicalPath
    m = TSRNTropicalPath(int(g["d"]), int(g["top_k"]), int(g["heads"]))
    sd = m.state_dict()
    missing = [k for k in sd if "p_" + k not in g]
    assert not missing, missing
    m.load_state_dict({k: torch.tensor(g["p_" + k]) for k in sd})
    return m.to(dev).eval()


def test_tropical_path_matches_reference_block(cuda):
    g = load_golden("tsrn_block")
    m = _path(g, cuda)
    x = torch.tensor(g["x"], device=cuda)
    with torch.no_grad():
        y1 = x + m.attn(m.ln_attn(x))
        y2 = y1 + m.reservoir(m.ln_res(y1))
        y3 = y2 + m.tropical_ssm(m.ln_ssm(y2))
        y = _path(g, cuda)(x)
    np.testing.assert_allclose(y1.cpu().numpy(), g["y_attn"], rtol=1e-4, atol=5e-5)
    np.testing.assert_allclose(y2.cpu().numpy(), g["y_res"], rtol=1e-4, atol=5e-5)
    np.testing.assert_allclose(y3.cpu().numpy(), g["y"], rtol=1e-4, atol=5e-5)
    torch.testing.assert_close(y, y3, rtol=0, atol=0)


def test_branch_events(cuda):
    g = load_golden("tsrn_block")
    m = _path(g, cuda)
    ev = {n: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for n in ("attn", "reservoir", "tropical_ssm")}
    with torch.no_grad():
        m(torch.tensor(g["x"], device=cuda), events=ev)
    torch.cuda.synchronize()
    assert all(a.elapsed_time(b) > 0 for a, b in ev.values())
