"""The tropical ops are CUDA-graph safe: a captured DTNAttention training step
(forward + backward: tropical projections with the STE backward, tropical
score, gated Maslov softmax) replayed on new inputs gives the eager step's
outputs and gradients."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("pointer_checks", [0, 1])
def test_dtn_step_graph_replay_matches_eager(cuda, pointer_checks):
    from mk_iii_technologies_tsrn_b200 import _lib
    from mk_iii_technologies_tsrn_b200.dtn import DTNAttention
    _lib.load().tp_set_pointer_checks(pointer_checks)
    try:
        torch.manual_seed(0)
        attn = DTNAttention(64, 4, dropout=0.0).to(cuda).train()
        gen = torch.Generator(device=cuda).manual_seed(1)
        x = torch.randn(8, 32, 64, device=cuda, generator=gen, requires_grad=True)
        g = torch.randn(8, 32, 64, device=cuda, generator=gen)
        static_out = {}

        def step():
            out, w = attn(x)
            out.backward(g)
            static_out["out"], static_out["w"] = out, w

        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                attn.zero_grad(set_to_none=True)
                x.grad = None
                step()
        torch.cuda.current_stream().wait_stream(side)
        attn.zero_grad(set_to_none=True)
        x.grad = None
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()

        for seed in (2, 3):
            xn = torch.randn(8, 32, 64, device=cuda,
                             generator=torch.Generator(device=cuda).manual_seed(seed))
            with torch.no_grad():
                x.copy_(xn)
            graph.replay()
            torch.cuda.synchronize()
            got = {"out": static_out["out"].detach().clone(), "w": static_out["w"].detach().clone(),
                   "gx": x.grad.clone()}
            got.update({n: p.grad.clone() for n, p in attn.named_parameters()})
            # eager reference on the same input
            xe = xn.clone().requires_grad_(True)
            params = [p for _, p in attn.named_parameters()]
            out, w = attn(xe)
            grads = torch.autograd.grad(out, [xe] + params, g)
            torch.testing.assert_close(got["out"], out.detach(), rtol=1e-5, atol=1e-6)
            torch.testing.assert_close(got["w"], w.detach(), rtol=1e-5, atol=1e-6)
            torch.testing.assert_close(got["gx"], grads[0], rtol=1e-4, atol=1e-5)
            for (n, _), gr in zip(attn.named_parameters(), grads[1:]):
                torch.testing.assert_close(got[n], gr, rtol=1e-4, atol=1e-5, msg=n)
        del graph
    finally:
        _lib.load().tp_set_pointer_checks(1)
