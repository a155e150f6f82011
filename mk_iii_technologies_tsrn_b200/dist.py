"""Multi-GPU execution of the tropical hot path (one process per GPU).

The reference is single-device; these are the B200 multi-GPU forms of its
hot path:

* ``ShardedMaxPlus`` -- the max-plus GEMM sharded by output columns: rank r
  owns W[r*N/P:(r+1)*N/P] and all of x and produces those columns of y and
  argmax.  Two exchange modes:

  - ``"p2p"`` (default on CUDA): every rank's full output lives in symmetric
    memory; the GEMM kernel stores each of its outputs into all ranks' copies
    over NVLink (peer stores from the epilogue, ``tp_maxplus_fwd_sharded``), so
    the all-gather costs no separate pass and overlaps the compute.
  - ``"nccl"``: the rank computes its shard into a local buffer, then
    ``all_gather_into_tensor`` (NCCL) gathers the rank-major shards, and a
    transpose copy restores the row-major [M, N] layout.

* ``shard_rows`` -- batch (row) sharding for the independent-row ops (tropical
  linear, scores, scan): no exchange at all.

Every rank must call the same methods in the same order (collectives).
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib
from .ops import _ptr, _require_cuda, _stream, maxplus_strided


BARRIER_TIMEOUT_MS = 20000   # device-side barrier wait limit (a missing peer ends it)


def shard_bounds(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous, even split of ``n`` items over ``world`` ranks (first ranks larger)."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_rows(t: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """This rank's block of rows (dim 0) of ``t`` (a view, no copy)."""
    a, b = shard_bounds(t.shape[0], world, rank)
    return t[a:b]


def rank_major_to_rows(gathered: torch.Tensor) -> torch.Tensor:
    """[P, M, Ns] (all-gather output) -> [M, P*Ns] row-major."""
    P, M, Ns = gathered.shape
    return gathered.permute(1, 0, 2).reshape(M, P * Ns)


class ShardedMaxPlus:
    """Column-sharded max-plus GEMM ``y = max_k(x + W)`` with int32 argmax over a group."""

    def __init__(self, M: int, N: int, K: int, *, group=None, mode: Optional[str] = None,
                 argmax: bool = True, device=None):
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if N % self.world:
            raise ValueError(f"N={N} must be divisible by the world size {self.world}")
        self.M, self.N, self.K = M, N, K
        self.Ns = N // self.world
        self.col0 = self.rank * self.Ns
        self.argmax = argmax
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.mode = mode or ("p2p" if self.world > 1 else "local")
        if self.mode == "p2p":
            self._setup_p2p()
        else:
            self.y_shard = torch.empty(M, self.Ns, device=self.device)
            self.am_shard = (torch.empty(M, self.Ns, device=self.device, dtype=torch.int32)
                             if argmax else None)
            if self.world > 1:
                self.y_all = torch.empty(self.world, M, self.Ns, device=self.device)
                self.am_all = (torch.empty(self.world, M, self.Ns, device=self.device,
                                           dtype=torch.int32) if argmax else None)

    # ------------------------------------------------------------------ p2p
    def _setup_p2p(self):
        # plain peer stores only: no NVLink multicast object is needed
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        import torch.distributed._symmetric_memory as symm_mem

        name = self.group.group_name
        self.y = symm_mem.empty(self.M, self.N, dtype=torch.float32, device=self.device)
        self.y_h = symm_mem.rendezvous(self.y, name)
        self.am = None
        if self.argmax:
            self.am = symm_mem.empty(self.M, self.N, dtype=torch.int32, device=self.device)
            self.am_h = symm_mem.rendezvous(self.am, name)
        order = [self.rank] + [r for r in range(self.world) if r != self.rank]
        yp = [self.y_h.buffer_ptrs[r] for r in order]
        self._ydst = (ctypes.c_void_p * len(order))(*yp)
        self._adst = None
        if self.argmax:
            ap = [self.am_h.buffer_ptrs[r] for r in order]
            self._adst = (ctypes.c_void_p * len(order))(*ap)

    def __call__(self, x: torch.Tensor, w_shard: torch.Tensor,
                 bias_shard: Optional[torch.Tensor] = None):
        """x [M,K] and this rank's w_shard [N/P,K] -> full (y [M,N], argmax [M,N] | None).

        In "p2p" mode the returned tensors are the rank's symmetric buffers:
        they are rewritten by the next call (on every rank)."""
        _require_cuda(x, w_shard, bias_shard)
        if self.mode == "p2p":
            return self._call_p2p(x, w_shard, bias_shard)
        y, am = maxplus_strided(x, w_shard, bias_shard, argmax=self.argmax,
                                out=self.y_shard, out_argmax=self.am_shard)
        if self.world == 1:
            return y, am
        dist.all_gather_into_tensor(self.y_all, y, group=self.group)
        if self.argmax:
            dist.all_gather_into_tensor(self.am_all, am, group=self.group)
        return (rank_major_to_rows(self.y_all),
                rank_major_to_rows(self.am_all) if self.argmax else None)

    def _call_p2p(self, x, w_shard, bias_shard):
        if x.dtype != torch.float32 or w_shard.dtype != torch.float32:
            raise TypeError("the fused sharded GEMM takes float32 operands")
        if x.shape != (self.M, self.K) or w_shard.shape != (self.Ns, self.K):
            raise ValueError("operand shapes do not match the layout this object was built for")
        # peers must be done reading the previous result before it is rewritten
        self.y_h.barrier(channel=0, timeout_ms=BARRIER_TIMEOUT_MS)
        with torch.cuda.device(self.device):
            st = _lib.load().tp_maxplus_fwd_sharded(
                self.M, self.Ns, self.K, _ptr(x), x.stride(0), _ptr(w_shard), w_shard.stride(0),
                _ptr(bias_shard), self._ydst, self._adst, self.world, self.N, self.col0,
                _stream(self.device))
        _lib.check(st, "tp_maxplus_fwd_sharded")
        # every rank's stores into my buffers are complete after this
        self.y_h.barrier(channel=1, timeout_ms=BARRIER_TIMEOUT_MS)
        return self.y, self.am


def maxplus_host_sharded(x_rows: torch.Tensor, w_shard: torch.Tensor, *, group=None,
                         argmax: bool = True, out: Optional[torch.Tensor] = None,
                         out_argmax: Optional[torch.Tensor] = None):
    """Column-sharded max-plus GEMM from host memory to host memory.

    Rank r holds, in (pinned) host memory, its block of rows of x
    (``x_rows`` [M/P, K], rows r*M/P ... of the full x) and its block of rows of
    W (``w_shard`` [N/P, K]).  Each rank uploads only those two over PCIe; the
    full x is assembled on every GPU by an in-place NCCL all-gather over NVLink
    while the rank's own row block is already being multiplied; the other row
    blocks follow once the gather lands.  Returns this rank's columns of y (and
    argmax) for ALL M rows in pinned host memory ([M, N/P]): the result is
    column-sharded across the ranks' hosts, the union being y = max_k(x + W).
    Every rank of ``group`` must call this with equal shapes.  Results equal
    :func:`~.ops.maxplus` of the full operands bit for bit."""
    if x_rows.is_cuda or w_shard.is_cuda:
        raise ValueError("maxplus_host_sharded takes host tensors")
    group = group or dist.group.WORLD
    P, r = dist.get_world_size(group), dist.get_rank(group)
    Mr, K = x_rows.shape
    Ns = w_shard.shape[0]
    if w_shard.shape[1] != K:
        raise ValueError("x and W shards differ in K")
    _lib.load()          # no CPU computation: fails loudly without the CUDA library
    dev = torch.device("cuda", torch.cuda.current_device())
    M = Mr * P
    y_host = out if out is not None else torch.empty(M, Ns, pin_memory=True)
    a_host = None
    if argmax:
        a_host = out_argmax if out_argmax is not None else torch.empty(
            M, Ns, dtype=torch.int32, pin_memory=True)
    main = torch.cuda.current_stream(dev)
    s_in, s_comm, s_out = (torch.cuda.Stream(dev) for _ in range(3))
    for s in (s_in, s_comm, s_out):
        s.wait_stream(main)
    x_full = torch.empty(M, K, device=dev)
    w_dev = torch.empty(Ns, K, device=dev)
    y = torch.empty(M, Ns, device=dev)
    am = torch.empty(M, Ns, device=dev, dtype=torch.int32) if argmax else None
    own = slice(r * Mr, (r + 1) * Mr)
    with torch.cuda.stream(s_in):
        x_full[own].copy_(x_rows, non_blocking=True)
        w_dev.copy_(w_shard, non_blocking=True)
    landed = torch.cuda.Event()
    landed.record(s_in)
    s_comm.wait_event(landed)
    with torch.cuda.stream(s_comm):
        # in place: rank r's input is its own slot of the output
        dist.all_gather_into_tensor(x_full, x_full[own], group=group)
    gathered = torch.cuda.Event()
    gathered.record(s_comm)

    def product(rows: slice):
        maxplus_strided(x_full[rows], w_dev, argmax=argmax, out=y[rows],
                        out_argmax=am[rows] if argmax else None)
        done = torch.cuda.Event()
        done.record(main)
        s_out.wait_event(done)
        with torch.cuda.stream(s_out):
            y_host[rows].copy_(y[rows], non_blocking=True)
            if argmax:
                a_host[rows].copy_(am[rows], non_blocking=True)

    main.wait_event(landed)
    product(own)
    main.wait_event(gathered)
    for rows in (slice(0, r * Mr), slice((r + 1) * Mr, M)):
        if rows.stop > rows.start:
            product(rows)
    for s in (s_in, s_comm, s_out):
        main.wait_stream(s)
    return y_host, a_host
