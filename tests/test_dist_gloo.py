"""Host-side multi-rank logic on CPU (gloo, world size 2): shard bounds, the
rank-major -> row-major layout of the gathered shards, and a simulated
failure of one rank that the others observe as an error, not a hang."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _column_sharded_worker(rank, world, port, q):
    try:
        import sys
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        from mk_iii_technologies_tsrn_b200.dist import rank_major_to_rows, shard_bounds
        _init(rank, world, port)
        M, N, K = 12, 10, 9
        rng = np.random.default_rng(0)
        x = rng.standard_normal((M, K)).astype(np.float32)
        w = rng.standard_normal((N, K)).astype(np.float32)
        n0, n1 = shard_bounds(N, world, rank)
        y, idx = oracle.maxplus_fwd(x, w[n0:n1])              # this rank's columns
        ys = [torch.empty(M, n1 - n0) for _ in range(world)]
        dist.all_gather(ys, torch.tensor(y))
        full = rank_major_to_rows(torch.stack(ys)).numpy()
        ry, _ = oracle.maxplus_fwd(x, w)
        q.put((rank, bool(np.array_equal(full, ry))))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))


def _failing_worker(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            raise RuntimeError("simulated rank failure before the collective")
        t = torch.ones(4)
        dist.all_reduce(t)          # rank 1 never joins: must time out, not hang
        q.put((rank, "no error"))
    except Exception as e:
        q.put((rank, type(e).__name__))


def _run(fn, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, v = q.get(timeout=timeout)
        out[r] = v
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


def test_shard_bounds_cover_exactly():
    from mk_iii_technologies_tsrn_b200.dist import shard_bounds
    for n in (0, 1, 7, 8, 8192, 10):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(8, 2, 2)


def test_rank_major_to_rows():
    from mk_iii_technologies_tsrn_b200.dist import rank_major_to_rows
    full = torch.arange(3 * 8, dtype=torch.float32).reshape(3, 8)
    shards = torch.stack([full[:, 0:4], full[:, 4:8]])      # [P, M, Ns]
    assert torch.equal(rank_major_to_rows(shards), full)


def test_column_sharded_gather_two_ranks():
    out = _run(_column_sharded_worker)
    assert out == {0: True, 1: True}


def test_rank_failure_is_an_error_not_a_hang():
    out = _run(_failing_worker, timeout=90)
    assert out[1] == "RuntimeError"
    assert out[0] != "no error"          # the survivor's collective failed
