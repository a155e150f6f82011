"""Column-sharded max-plus GEMM with the all-gather fused into the epilogue.

On one GPU the multi-destination store is checked with two local buffers; the
two-rank test (peer stores over NVLink into symmetric memory) runs when the box
has at least two GPUs."""
import ctypes
import datetime
import os
import socket

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,Ns,col0,force_tma,stream_k", [
    (512, 1024, 192, 512, 256, True, 1),    # fused TMA epilogue (deferred argmax search)
    (512, 1024, 192, 512, 256, False, 1),   # below the TMA threshold: generic + copies
    (96, 300, 50, 100, 150, False, 1),      # generic + copies
    # 160 tiles: the stream-K schedule (forced) with the destination stores of
    # the split tiles' merges, as an 8-rank shard of a large GEMM takes it
    (2048, 2560, 256, 1280, 640, True, 2),
    (2048, 2560, 256, 1280, 640, True, 3)])   # the same, tiles cut into 4 k-aligned pieces
def test_sharded_entry_two_local_destinations(cuda, M, N, K, Ns, col0, force_tma, stream_k):
    from mk_iii_technologies_tsrn_b200 import _lib
    lib = _lib.load()
    old = lib.tp_set_argmax_tma_min_terms(0 if force_tma else 1 << 30)
    old_sk = lib.tp_set_stream_k(stream_k)
    try:
        _two_local_destinations(lib, cuda, M, N, K, Ns, col0)
    finally:
        lib.tp_set_stream_k(old_sk)
        lib.tp_set_argmax_tma_min_terms(old)


def _two_local_destinations(lib, cuda, M, N, K, Ns, col0):
    g = torch.Generator(device=cuda).manual_seed(0)
    x = torch.randn(M, K, device=cuda, generator=g)
    w = torch.randn(Ns, K, device=cuda, generator=g)
    b = torch.randn(Ns, device=cuda, generator=g)
    ys = [torch.full((M, N), float("nan"), device=cuda) for _ in range(2)]
    ams = [torch.full((M, N), -1, device=cuda, dtype=torch.int32) for _ in range(2)]
    yd = (ctypes.c_void_p * 2)(*[t.data_ptr() for t in ys])
    ad = (ctypes.c_void_p * 2)(*[t.data_ptr() for t in ams])
    st = lib.tp_maxplus_fwd_sharded(M, Ns, K, ctypes.c_void_p(x.data_ptr()), K,
                                    ctypes.c_void_p(w.data_ptr()), K,
                                    ctypes.c_void_p(b.data_ptr()), yd, ad, 2, N, col0,
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, lib.tp_status_string(st)
    torch.cuda.synchronize()
    ry, ri = oracle.maxplus_fwd(x.cpu().numpy(), w.cpu().numpy(), b.cpu().numpy())
    for y, am in zip(ys, ams):
        np.testing.assert_array_equal(y[:, col0:col0 + Ns].cpu().numpy(), ry)
        np.testing.assert_array_equal(am[:, col0:col0 + Ns].cpu().numpy(), ri)
        assert torch.all(torch.isnan(y[:, :col0])) and torch.all(torch.isnan(y[:, col0 + Ns:]))
        assert torch.all(am[:, :col0] == -1)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_rank_worker(rank, world, port, mode, force_tma, q):
    try:
        import sys
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        import torch.distributed as dist
        from mk_iii_technologies_tsrn_b200.dist import ShardedMaxPlus
        from mk_iii_technologies_tsrn_b200 import _lib
        if force_tma:      # this small case would otherwise take the generic kernel
            _lib.load().tp_set_argmax_tma_min_terms(0)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        M, N, K = 512, 1024, 320
        g = torch.Generator(device=dev).manual_seed(0)
        x = torch.randn(M, K, device=dev, generator=g)
        w = torch.randn(N, K, device=dev, generator=g)
        op = ShardedMaxPlus(M, N, K, mode=mode, device=dev)
        ok = True
        for rep in range(2):                   # two calls in a row
            y, am = op(x, w[op.col0:op.col0 + op.Ns].contiguous())
            torch.cuda.synchronize()
            ry, ri = oracle.maxplus_fwd(x.cpu().numpy(), w.cpu().numpy())
            ok &= bool(np.array_equal(y.cpu().numpy(), ry))
            ok &= bool(np.array_equal(am.cpu().numpy(), ri))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok))
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


@pytest.mark.parametrize("mode,force_tma", [("p2p", True), ("p2p", False), ("nccl", True)])
def test_two_rank_sharded_gemm(cuda, mode, force_tma):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, 2, port, mode, force_tma, q))
             for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert out == {0: True, 1: True}, out


def _two_rank_host_worker(rank, world, port, q):
    try:
        import sys
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        import torch.distributed as dist
        from mk_iii_technologies_tsrn_b200.dist import maxplus_host_sharded
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        M, N, K = 768, 1024, 288
        g = torch.Generator().manual_seed(0)
        x = torch.randn(M, K, generator=g)
        w = torch.randn(N, K, generator=g)
        w[torch.rand(N, K, generator=g) < 0.05] = float("-inf")
        Mr, Ns = M // world, N // world
        ok = True
        for rep in range(2):                   # two calls in a row
            y, am = maxplus_host_sharded(x[rank * Mr:(rank + 1) * Mr].pin_memory(),
                                         w[rank * Ns:(rank + 1) * Ns].pin_memory())
            torch.cuda.synchronize()
            ry, ri = oracle.maxplus_fwd(x.numpy(), w[rank * Ns:(rank + 1) * Ns].numpy())
            ok &= bool(np.array_equal(y.numpy(), ry)) and bool(np.array_equal(am.numpy(), ri))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok))
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


def test_two_rank_host_sharded_gemm(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_rank_host_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert out == {0: True, 1: True}, out
