"""Host-to-host max-plus with the PCIe transfers overlapped (ops.maxplus_host):
results equal the device entry point's bit for bit."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,blocks,with_bias,argmax", [
    (1000, 300, 200, 4, False, True),    # ragged last block
    (2048, 512, 384, 3, True, True),
    (4096, 1024, 1024, 4, False, True),  # blocks large enough for the TMA kernel
    (777, 129, 65, 2, True, False),      # value only
])
def test_maxplus_host_equals_device(cuda, M, N, K, blocks, with_bias, argmax):
    from mk_iii_technologies_tsrn_b200 import ops
    g = torch.Generator().manual_seed(M + N + K)
    x = torch.randn(M, K, generator=g).pin_memory()
    w = torch.randn(N, K, generator=g)
    w[torch.rand(N, K, generator=g) < 0.05] = float("-inf")
    w = w.pin_memory()
    b = torch.randn(N, generator=g) if with_bias else None
    y, am = ops.maxplus_host(x, w, b, argmax=argmax, blocks=blocks)
    torch.cuda.current_stream().synchronize()
    yd, ad = ops.maxplus(x.to(cuda), w.to(cuda), b.to(cuda) if b is not None else None,
                         argmax=argmax)
    assert torch.equal(y.view(torch.int32), yd.cpu().view(torch.int32))
    if argmax:
        assert torch.equal(am, ad.cpu())
    else:
        assert am is None


def test_maxplus_host_into_given_buffers_twice(cuda):
    from mk_iii_technologies_tsrn_b200 import ops
    g = torch.Generator().manual_seed(1)
    x = torch.randn(512, 96, generator=g).pin_memory()
    w = torch.randn(200, 96, generator=g).pin_memory()
    y = torch.empty(512, 200).pin_memory()
    am = torch.empty(512, 200, dtype=torch.int32).pin_memory()
    for _ in range(2):
        ops.maxplus_host(x, w, out=y, out_argmax=am)
        torch.cuda.current_stream().synchronize()
        yd, ad = ops.maxplus(x.to(cuda), w.to(cuda))
        assert torch.equal(y, yd.cpu()) and torch.equal(am, ad.cpu())


def test_maxplus_host_rejects_device_tensors(cuda):
    from mk_iii_technologies_tsrn_b200 import ops
    with pytest.raises(ValueError):
        ops.maxplus_host(torch.zeros(4, 4, device=cuda), torch.zeros(4, 4))
