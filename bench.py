#!/usr/bin/env python
"""Benchmark of the tropical hot path on B200 (one process per GPU).

Default workload (``--workload gemm``): the fp32 max-plus GEMM with int32 argmax
at M = N = K = 8192 -- ``y[m,n] = max_k(x[m,k] + W[n,k])`` -- on synthetic
N(0,1) inputs with 5% of W set to -inf (seeded).  A step is one pass of the hot
path over the whole problem: at N GPUs each rank computes its output-column
shard W[r*N/P:(r+1)*N/P] and the shards of y and argmax are exchanged (peer
stores fused into the GEMM epilogue, or NCCL with ``--exchange nccl``; strong
scaling: the total problem is fixed).  The metric is max-plus Gop/s =
2*M*N*K / step time (one add and one max per term).  Every run checks the
result bit for bit against the oracle on sampled rows x the first and last 64
columns of every rank's range, on every rank, and exits non-zero on a
mismatch.  The end-to-end number runs the public host entry: ``ops.maxplus_host``
on one GPU, ``dist.maxplus_host_sharded`` on several (each rank's row block
of x and its W shard over PCIe, x gathered over NVLink).  The JSON line also
carries a ``secondary`` list: every workload below measured in the same run.

Batch workloads split the configuration's batch over the ranks
(``--scaling strong``, default; ``--scaling weak`` gives every rank all of it):

``--workload scan``: the tropical SSM scan at B=16, T=4096, C=1024: forward
(read b, x; write h: 12 B/elem) plus argmax-path backward recomputing the
winners (read g, h, b, x; write gu: 20 B/elem); metric GB/s of those
algorithmic bytes.  Few lanes per GPU (B=2 at 8 GPUs, or ``--scan-batch 2``
on one) run the chunk-parallel scan.

Workloads whose data fit in L2 (config 1, the DTN block, the scan at B <= 2
per GPU) overwrite a 256 MiB buffer before every timed step, outside that
step's CUDA events, and report the sum of the steps' device times; the other
workloads read inputs larger than L2 every step.

``--workload linear``: config 1, the tropical linear x [1024,256] (x) W [256,256]
forward with int32 argmax and the argmax backward; Gop/s of forward ops.

``--workload tsrn_attn``: the TSRN tropical top-k attention of config 5 (B=64, H=8,
T=1024, d_h=80, top_k=16, causal) through the fused kernel; tokens/s.

``--workload esn``: the echo-state reservoir recurrence of config 5's first
TSRN block (research/tsrn_dml.py:1073: GRU-gated, d_reservoir = d_model / 2 =
320; B=64, T=1024) in one fused launch from the input projections to the state
sequence H; ``--esn-mode leaky`` runs the leaky reservoir of tsrn_gpu.py
(d_reservoir = d_model = 640) instead.  Metric tokens/s.

``--workload tsrn_block``: config 5's hot path, the tropical branches of the first
TSRN block (research/tsrn_dml.py:1096-1106: fused top-k attention, GRU reservoir,
tropical SSM, with their LayerNorms and projections) on B=64 sequences of
T=1024 tokens, d=640; tokens/s and each branch's share of the step.

``--workload tsrn_train``: the same branches in training (forward + backward of
every parameter and the input under autograd: the attention's sparse backward,
the reservoir's one-launch backward through time, the scan's argmax-path
backward); tokens/s.

``--workload dtn``: config 2, the drop-in DTNAttention(256, 8) block
(tropical Q/K projections with the STE backward, tropical score, Maslov
softmax) forward + backward at B=128, L=64; metric tokens/s.

Every timed region lasts at least 0.6 s (short steps are repeated) so that the
clock sampler sees it; a kernel's timed-out device-side wait raises after each
timed region.

``--dtype bf16`` stores the GEMM operands in bf16 (widened exactly on the GPU;
the arithmetic stays fp32); with ``--arith bf16`` every sum is rounded to bf16
as the reference does on bf16 tensors (packed bf16x2 kernel).

``--impl reference`` times the reference's own CPU implementation (its PyTorch
expression, restated in ``oracle/torch_ref.py``) on the host cores for the same
metric, on a bounded sample of the workload; only rank 0 runs it.

Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402


# ----------------------------------------------------------------------------- helpers
def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload",
                   choices=["gemm", "scan", "dtn", "linear", "tsrn_attn", "esn", "tsrn_block",
                            "tsrn_train"],
                   default="gemm")
    p.add_argument("--size", type=int, default=8192, help="M = N = K of the GEMM workload")
    p.add_argument("--dtype", choices=["f32", "bf16"], default="f32",
                   help="GEMM operand storage")
    p.add_argument("--arith", choices=["f32", "bf16"], default="f32",
                   help="bf16 operands: fp32 arithmetic (exact widening) or bf16 arithmetic "
                        "(sums rounded to bf16, as the reference on bf16 tensors; packed "
                        "bf16x2 kernel)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-graph", action="store_true",
                   help="dtn workload: run the step eagerly instead of replaying a CUDA graph")
    p.add_argument("--att-batch", type=int, default=64,
                   help="sequences per rank of the tsrn_attn workload (64 = config 5)")
    p.add_argument("--esn-mode", choices=["gru", "leaky"], default="gru",
                   help="esn workload: GRU-gated reservoir of config 5 (research/tsrn_dml.py, "
                        "d_reservoir 320) or the leaky one of tsrn_gpu.py (d_reservoir 640)")
    p.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                   help="batch workloads (scan, dtn, linear, tsrn_attn, esn, tsrn_block): "
                        "'strong' splits the configuration's batch over the ranks, 'weak' "
                        "gives every rank the whole batch")
    p.add_argument("--scan-batch", type=int, default=16,
                   help="batch of the scan workload (config 3: 16; 2 = its per-GPU "
                        "share at 8 GPUs, where the chunk-parallel mode runs)")
    p.add_argument("--no-secondary", action="store_true",
                   help="default GEMM line only: skip the other workloads' sub-lines")
    p.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                   help="N>1 GEMM: fused peer-store epilogue (p2p) or NCCL all-gather")
    return p.parse_args()


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        torch.distributed.init_process_group(
            "nccl", timeout=datetime.timedelta(seconds=180),
            device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.proc = subprocess.Popen(
            [exe, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
             "-i", str(self.gpu), "-f", self.path],
            stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [s.strip() for s in line.split(",")]
                    if len(parts) < 9:
                        continue
                    try:
                        sm.append(float(parts[1]))
                        mx = float(parts[2])
                    except ValueError:
                        continue
                    for n, v in zip(names, parts[5:9]):
                        if v.lower().startswith("active"):
                            reasons.add(n)
        finally:
            os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


def profiled_traffic(key):
    """DRAM bytes per launch of a kernel from a committed ncu capture (profiles/traffic.txt)."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        for line in f:
            parts = line.split()
            if len(parts) >= 2 and parts[0] == key:
                return int(parts[1])
    return None


def local_batch(total: int, world: int, args) -> int:
    """Rows of a batch workload this rank runs: the whole batch (weak scaling) or
    its 1/world share (strong scaling: the configuration's batch split over the
    ranks, no exchange between them)."""
    if args.scaling == "weak" or world == 1:
        return total
    if total % world:
        raise SystemExit(f"batch {total} does not split over {world} ranks")
    return total // world


def parallelism(total: int, local: int, world: int, what: str = "batch") -> str:
    if world == 1:
        return "single GPU"
    if local == total:
        return f"{what} replicated x{world} (weak: {total} per rank)"
    return f"{what}-sharded x{world} (strong: {local} of {total} per rank, no exchange)"


TF32_PEAK_SOURCE = ("dense TF32 rate taken as half of MEASURED_PEAKS.json bf16_tflops "
                    "(cuBLAS bf16 burst; the tensor cores run TF32 at half the bf16 rate); "
                    "of measured")


def tf32_peak():
    """Dense TF32 tensor-core rate (TFLOP/s): half the measured bf16 GEMM burst rate
    (fallback 1590 TFLOP/s bf16 when the file is absent)."""
    return measured_peaks().get("bf16_tflops", 1590.0) / 2.0


def ffma_peak():
    """fp32 FMA rate (TFLOP/s) of the register-only probe: the better of scalar
    FFMA (form 7) and packed fma.f32x2 (form 9), measured in this run."""
    from mk_iii_technologies_tsrn_b200 import ops
    best = 0.0
    for form in (7, 9):
        ops.probe_addmax(form, 148 * 8, 50)
        pms, terms = ops.probe_addmax(form, 148 * 8, 400)
        best = max(best, 2.0 * terms / (pms / 1e3) / 1e12)
    return best


def steps_for(step, requested: int, world: int, min_s: float = 0.6, cap: int = 20000) -> int:
    """At least ``requested`` timed steps, and enough that the timed region lasts
    ``min_s`` seconds (so that the clock sampler sees it); the count is agreed
    over the ranks (max) so that every rank runs the same collectives."""
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(3):
        step()
    e1.record()
    torch.cuda.synchronize()
    per = max(e0.elapsed_time(e1) / 3.0, 1e-3)
    n = int(min(cap, max(requested, math.ceil(min_s * 1e3 / per))))
    if world > 1:
        t = torch.tensor([n], device="cuda", dtype=torch.int64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        n = int(t.item())
    return n


def time_steps(step, steps, world):
    """Device time of `steps` calls of step() between barrier+sync fences (max over ranks)."""
    stream = torch.cuda.current_stream()
    barrier(world)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        step()
    end.record(stream)
    torch.cuda.synchronize()
    # a bounded device-side wait that ran out means a kernel returned early:
    # the step's results (and its timing) are not valid -- raise
    from mk_iii_technologies_tsrn_b200 import ops
    ops.check_device_error()
    barrier(world)
    return max_over_ranks(start.elapsed_time(end), world)


L2_FLUSH_BYTES = 256 << 20      # written before each cold step: twice the 126 MB L2
_flush_buf = None


def time_steps_cold(step, steps, world):
    """Device time of `steps` calls of step(), each after an L2 flush (a 256 MiB
    buffer overwritten) that lies outside its own pair of CUDA events: the sum
    of the steps' times, max over ranks.  For workloads whose data fit in L2,
    so that no step reads what the previous one left in L2."""
    global _flush_buf
    if _flush_buf is None:
        _flush_buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    barrier(world)
    torch.cuda.synchronize()
    pairs = []
    for _ in range(steps):
        _flush_buf.fill_(1)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        step()
        e1.record(stream)
        pairs.append((e0, e1))
    torch.cuda.synchronize()
    from mk_iii_technologies_tsrn_b200 import ops
    ops.check_device_error()
    barrier(world)
    return max_over_ranks(sum(a.elapsed_time(b) for a, b in pairs), world)


# ----------------------------------------------------------------------------- CPU baseline
def cpu_gemm_rate(size: int, target_s: float = 12.0, bf16: bool = False):
    """Reference expression (oracle/torch_ref.py) on a row sample of the size^3 problem
    (on bf16 tensors when ``bf16``: the reference's own bf16 arithmetic)."""
    from oracle.torch_ref import maxplus_fwd_torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(1)
    w = torch.randn(size, size, generator=g)
    x = torch.randn(1024, size, generator=g)
    if bf16:
        w, x = w.bfloat16(), x.bfloat16()
    # warm up on 1 row, calibrate on 4, then size the sample for ~target_s seconds
    maxplus_fwd_torch(x[:1], w)
    t0 = time.perf_counter()
    maxplus_fwd_torch(x[:4], w)
    dt1 = (time.perf_counter() - t0) / 4
    rows = int(max(1, min(1024, target_s / max(dt1, 1e-6))))
    t0 = time.perf_counter()
    maxplus_fwd_torch(x[:rows], w)
    dt = time.perf_counter() - t0
    ops = 2.0 * rows * size * size
    return {"value": ops / dt / 1e9, "unit": "Gop/s", "cores": threads, "kind": "port",
            "sample": f"{rows} of {size} rows of x against all of W ({size}x{size}) "
                      f"through the reference expression W[None]+x[:,None] -> max(-1) "
                      f"(values + indices){' on bf16 tensors' if bf16 else ''}, {dt:.1f} s"}


def cpu_scan_rate(B, T, C, target_s: float = 12.0):
    from oracle.torch_ref import scan_closed_form_torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(1)
    b_rows = 1
    a = -torch.rand(C, generator=g)
    u = (0.1 * torch.randn(b_rows, T, C, generator=g)) + torch.randn(b_rows, T, C, generator=g)
    t0 = time.perf_counter()
    scan_closed_form_torch(u, a)
    dt = time.perf_counter() - t0
    reps = int(max(1, min(50, target_s / max(dt, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(reps):
        scan_closed_form_torch(u, a)
    dt = (time.perf_counter() - t0) / reps
    elems = b_rows * T * C
    # the reference closed form is forward-only; count its forward bytes (12 B/elem)
    return {"value": 12.0 * elems / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"closed-form forward (research/tsrn_dml.py:961-972) on 1 of {B} batch "
                      f"rows (T={T}, C={C}), {reps} reps, forward bytes only"}


# ----------------------------------------------------------------------------- workloads
def gemm_workload(args, world, rank):
    from mk_iii_technologies_tsrn_b200 import ops, _lib

    lib = _lib.load()
    lib.tp_set_pointer_checks(0)  # validated once below; keep per-call host cost out
    S = args.size
    if S % world:
        raise SystemExit(f"size {S} not divisible by {world} ranks")
    M, N, K = S, S, S
    Nr = N // world
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(M, K, device=dev, generator=gen)
    gw = torch.Generator(device=dev).manual_seed(1)
    W_full_rows = torch.randn(N, K, device=dev, generator=gw)
    gm = torch.Generator(device=dev).manual_seed(2)
    W_full_rows[torch.rand(N, K, device=dev, generator=gm) < 0.05] = float("-inf")
    W = W_full_rows[rank * Nr:(rank + 1) * Nr].contiguous()
    # columns the self-check compares: the first and last 64 of EVERY rank's
    # column range (at N>1 the other ranks' columns arrive over NVLink or NCCL)
    ce = min(64, Nr)
    chk_cols = torch.cat([torch.arange(r * Nr, r * Nr + ce) for r in range(world)] +
                         [torch.arange((r + 1) * Nr - ce, (r + 1) * Nr) for r in range(world)])
    W_chk = W_full_rows[chk_cols.to(dev)].cpu()
    del W_full_rows
    if args.dtype == "bf16":
        x, W = x.to(torch.bfloat16), W.to(torch.bfloat16)
    bf16_arith = args.dtype == "bf16" and args.arith == "bf16"
    if args.arith == "bf16" and args.dtype != "bf16":
        raise SystemExit("--arith bf16 needs --dtype bf16")
    if bf16_arith and world > 1:
        raise SystemExit("--arith bf16 is a single-GPU workload here")
    y = torch.empty(M, Nr, device=dev)
    am = torch.empty(M, Nr, device=dev, dtype=torch.int32)
    sharded = None
    if world > 1:
        from mk_iii_technologies_tsrn_b200.dist import ShardedMaxPlus
        sharded = ShardedMaxPlus(M, N, K, mode=args.exchange, device=dev)

    kernel_ms = []

    def step(record=False):
        if record:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
        if sharded is None:
            ops.maxplus_strided(x, W, out=y, out_argmax=am, arith=args.arith)
        elif args.dtype == "bf16":
            sharded(ops.widen_bf16(x), ops.widen_bf16(W))
        else:
            sharded(x, W)          # shard GEMM + exchange (fused or NCCL)
        if record:
            e1.record()
            kernel_ms.append((e0, e1))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # bit-exact self-check against the oracle (oracle.maxplus_fwd: the
    # reference expression tropformer.py:131,141) on sampled rows x the columns
    # above.  Every rank checks its own full result, so at N>1 the columns that
    # the other ranks wrote are compared too; the verdict is reduced over the
    # ranks (MIN) and any mismatch ends the run with a non-zero exit code.
    import oracle
    import numpy as np
    chk_rows = torch.tensor([0, 1, M // 2 + 3, M - 1])
    if sharded is None:
        yo, ao = y, am
    else:
        yo, ao = sharded(x.float(), W.float())   # every rank takes the same collective steps
    torch.cuda.synchronize()
    ref_fn = oracle.maxplus_fwd_bf16 if bf16_arith else oracle.maxplus_fwd
    wref = W_chk.to(x.dtype).float() if args.dtype == "bf16" else W_chk
    ry, ri = ref_fn(x[chk_rows.to(dev)].float().cpu().numpy(), wref.numpy())
    cc = chk_cols.to(dev)
    got_y = yo[chk_rows.to(dev)][:, cc].cpu().numpy()
    got_i = ao[chk_rows.to(dev)][:, cc].cpu().numpy()
    ok = bool(np.array_equal(got_y, ry) and np.array_equal(got_i, ri))
    flag = torch.tensor([1 if ok else 0], device=dev, dtype=torch.int32)
    if world > 1:
        torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MIN)
    if not ok:
        bad = np.argwhere((got_y != ry) | (got_i != ri))[:4]
        print(f"rank {rank}: max-plus self-check MISMATCH at (row, column) "
              f"{[(int(chk_rows[a]), int(chk_cols[b])) for a, b in bad]}", file=sys.stderr,
              flush=True)
    if int(flag.item()) != 1:
        raise SystemExit("max-plus self-check failed against the oracle")
    check_desc = (f"bit-exact vs oracle on {len(chk_rows)} rows x {len(chk_cols)} columns "
                  f"(first/last {ce} of each of the {world} rank column ranges), "
                  f"all ranks (MIN-reduced)")

    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    ms = time_steps(lambda: step(record=True), args.steps, world)
    clk = clocks.stop()
    torch.cuda.synchronize()
    kms = statistics.mean(a.elapsed_time(b) for a, b in kernel_ms)
    kms = max_over_ranks(kms, world)

    ops_per_step = 2.0 * M * N * K
    value = ops_per_step / (ms / args.steps / 1e3) / 1e9

    # ---- end to end through the public API: pinned host in, pinned host out
    hx = x.cpu().pin_memory()
    hW = W.cpu().pin_memory()
    hy = torch.empty(M, Nr).pin_memory()
    ham = torch.empty(M, Nr, dtype=torch.int32).pin_memory()
    dx = torch.empty_like(x)
    dW = torch.empty_like(W)
    host_sharded = sharded is not None and args.dtype == "f32"
    if host_sharded:
        # each rank's host holds its row block of x and its W shard
        hx = x[rank * (M // world):(rank + 1) * (M // world)].cpu().pin_memory()

    def e2e_step():
        if sharded is None and args.dtype == "f32":
            # the host-to-host entry point: x in row blocks, overlapped with the
            # computation and with the results' return
            ops.maxplus_host(hx, hW, out=hy, out_argmax=ham)
            return
        if host_sharded:
            # the rank's row block of x and its W shard over PCIe, x all-gathered
            # over NVLink while the own block computes, the rank's columns of y
            # and argmax back to its host
            from mk_iii_technologies_tsrn_b200.dist import maxplus_host_sharded
            maxplus_host_sharded(hx, hW, out=hy, out_argmax=ham)
            return
        dx.copy_(hx, non_blocking=True)
        dW.copy_(hW, non_blocking=True)
        if sharded is None:
            ys, ams = ops.maxplus_strided(dx, dW, out=y, out_argmax=am, arith=args.arith)
        else:
            if args.dtype == "bf16":
                yf, af = sharded(ops.widen_bf16(dx), ops.widen_bf16(dW))
            else:
                yf, af = sharded(dx, dW)
            ys, ams = yf[:, rank * Nr:(rank + 1) * Nr], af[:, rank * Nr:(rank + 1) * Nr]
        hy.copy_(ys, non_blocking=True)   # this rank's columns of the result
        ham.copy_(ams, non_blocking=True)

    for _ in range(2):
        e2e_step()
    e2e_steps = max(3, min(args.steps, 5))
    e2e_ms = time_steps(e2e_step, e2e_steps, world)
    e2e_value = ops_per_step / (e2e_ms / e2e_steps / 1e3) / 1e9
    h2d = hx.numel() * hx.element_size() + hW.numel() * hW.element_size()
    d2h = (hy.numel() + ham.numel()) * 4

    # ---- roofline.  Max-plus is CUDA-core work (one add and one max per term;
    # tensor cores do not apply).  The peak is the fastest rate any form of the
    # add+max instruction mix reaches in the register-only probe, measured in
    # this run (forms: scalar, packed add.f32x2, 3-input max, mixes).  For
    # context, the nominal issue limit of the packed form is 128 terms per
    # clock per SM; measured forms reach about half of it.
    probe = {}
    for form in range(7):
        ops.probe_addmax(form, 148 * 8, 50)                      # warm
        pms, terms = ops.probe_addmax(form, 148 * 8, 400)
        probe[form] = 2.0 * terms / (pms / 1e3) / 1e12           # Top/s (2 ops per term)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    mhz = (clk or {}).get("sm_mhz") or measured_peaks().get("sm_max_mhz", 1965.0)
    issue_limit = 256.0 * sms * mhz * 1e6 / 1e12
    # the peak of the arithmetic the kernel runs: fp32 forms 0-4, bf16x2 forms 5-6
    peak = max(probe[f] for f in ((5, 6) if bf16_arith else range(5)))
    per_gpu_ops = 2.0 * M * Nr * K
    achieved = per_gpu_ops / (kms / 1e3) / 1e12
    roofline = {"bound": "cuda-core", "achieved": achieved, "peak": peak, "unit": "Top/s",
                "frac": achieved / peak,
                "traffic": profiled_traffic(f"maxplus_tma_gemm{S}") if world == 1 else None,
                "peak_source": "in-repo register-only add+max probe (tp_probe_addmax), best "
                               "instruction form of the kernel's arithmetic (" +
                               ("bf16x2" if bf16_arith else "fp32") +
                               "), measured in this run; of measured",
                "probe_top_s": {"fadd_fmnmx": probe[0], "fadd2_fmnmx3": probe[1],
                                "fadd2_fmnmx3_nan": probe[2], "2fadd_fmnmx3_nan": probe[3],
                                "mixed": probe[4], "bf16x2_add_max": probe[5],
                                "bf16x2_add_max_nan": probe[6]},
                "nominal_issue_limit_top_s": issue_limit,
                "kernel_ms": kms}
    res = {
        "metric": "max-plus GEMM Gop/s (fp32, with int32 argmax)" if args.dtype == "f32" else
                  ("max-plus GEMM Gop/s (bf16 operands, bf16 arithmetic, with int32 argmax)"
                   if bf16_arith else
                   "max-plus GEMM Gop/s (bf16 operands, fp32 arithmetic, with int32 argmax)"),
        "value": value,
        "unit": "Gop/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None,
        "dtype": "bf16" if bf16_arith else "f32",
        "data": "synthetic: x, W ~ N(0,1) (seeded), 5% of W = -inf",
        "config": {"workload": f"maxplus_gemm M=N=K={S} {args.dtype} operands + int32 argmax"
                               + (", bf16 arithmetic" if bf16_arith else ""),
                   "operand_storage": args.dtype,
                   "arithmetic": "bf16" if bf16_arith else "f32",
                   "M": M, "N": N, "K": K,
                   "parallelism": (f"column-shard x{world}, " + (
                       "all-gather fused into the GEMM epilogue (peer stores into "
                       "symmetric memory over NVLink)" if args.exchange == "p2p" else
                       "NCCL all-gather of y/argmax")) if world > 1 else "single GPU",
                   "l2": "inputs (2 x 256 MiB) larger than L2",
                   "self_check": check_desc},
        "e2e": {"value": e2e_value, "unit": "Gop/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "path": ("ops.maxplus_host (x row blocks over PCIe overlapped with the "
                         "products and the results' return)") if sharded is None and
                        args.dtype == "f32" else
                        ("dist.maxplus_host_sharded: per rank its 1/P row block of x and its "
                         "W shard over PCIe, x all-gathered over NVLink (NCCL, in place) "
                         "while the own block computes, the rank's columns of y/argmax "
                         "back to its host (column-sharded result)") if host_sharded else
                        "device copies + the device entry"},
        # one max-plus kernel per step (+2 exact widening kernels for bf16 operands with
        # fp32 arithmetic; +2 barrier kernels at N>1)
        "gpu_launches": args.steps * (3 if (args.dtype == "bf16" and not bf16_arith) else 1),
        "roofline": roofline,
        "clocks": clk,
    }
    return res


def scan_workload(args, world, rank):
    from mk_iii_technologies_tsrn_b200 import ops, _lib

    _lib.load().tp_set_pointer_checks(0)
    B, T, C = local_batch(getattr(args, "scan_batch", 16), world, args), 4096, 1024
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(100 + rank)
    a = -torch.rand(C, device=dev, generator=gen)
    b = 0.1 * torch.randn(B, T, C, device=dev, generator=gen)
    x = torch.randn(B, T, C, device=dev, generator=gen)
    g = torch.randn(B, T, C, device=dev, generator=gen)
    ninf = float("-inf")
    fwd_ms, bwd_ms = [], []

    def step(record=False):
        e = [torch.cuda.Event(enable_timing=True) for _ in range(3)] if record else None
        if record:
            e[0].record()
        h, _ = ops.scan_forward(b, x, a, ninf)
        if record:
            e[1].record()
        ops.scan_backward(g, a, ninf, b=b, x=x, h=h, need_ga=True)
        if record:
            e[2].record()
            fwd_ms.append((e[0], e[1]))
            bwd_ms.append((e[1], e[2]))

    for _ in range(args.warmup):
        step()
    steps = steps_for(step, args.steps, world)
    # inputs that fit in L2 (b, x, g at B <= 2): every timed step starts cold
    cold = 3 * B * T * C * 4 < 2 * (126 << 20)
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    ms = (time_steps_cold if cold else time_steps)(lambda: step(True), steps, world)
    clk = clocks.stop()
    f_ms = max_over_ranks(statistics.mean(p.elapsed_time(q) for p, q in fwd_ms), world)
    b_ms = max_over_ranks(statistics.mean(p.elapsed_time(q) for p, q in bwd_ms), world)
    elems = B * T * C
    bytes_step = 32.0 * elems * world
    value = bytes_step / (ms / steps / 1e3) / 1e9
    peak = measured_peaks().get("hbm_gbs", 6650.0)
    ach_f = 12.0 * elems / (f_ms / 1e3) / 1e9
    ach_b = 20.0 * elems / (b_ms / 1e3) / 1e9

    hb, hx_, hg = b.cpu().pin_memory(), x.cpu().pin_memory(), g.cpu().pin_memory()
    hh = torch.empty(B, T, C).pin_memory()
    hgu = torch.empty(B, T, C).pin_memory()
    db, dx, dg = torch.empty_like(b), torch.empty_like(x), torch.empty_like(g)

    def e2e_step():
        db.copy_(hb, non_blocking=True)
        dx.copy_(hx_, non_blocking=True)
        dg.copy_(hg, non_blocking=True)
        h, _ = ops.scan_forward(db, dx, a, ninf)
        gu, _, _ = ops.scan_backward(dg, a, ninf, b=db, x=dx, h=h, need_ga=True)
        hh.copy_(h, non_blocking=True)
        hgu.copy_(gu, non_blocking=True)

    for _ in range(2):
        e2e_step()
    e2e_ms = time_steps(e2e_step, 3, world)
    e2e_value = bytes_step / (e2e_ms / 3 / 1e3) / 1e9
    return {
        "metric": "tropical scan GB/s (fwd 12 B/elem + argmax-path bwd 20 B/elem)",
        "value": value, "unit": "GB/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms / steps, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: a=-U(0,1), b~N(0,0.1), x~N(0,1), g~N(0,1), h0=-inf (seeded)",
        "config": {"workload": f"tropical_ssm_scan B={B * world} T={T} C={C}, fwd+bwd",
                   "parallelism": parallelism(getattr(args, "scan_batch", 16), B, world),
                   "mode": ops.scan_mode(B, T, C),
                   "l2": f"inputs (3 x {B * T * C * 4 >> 20} MiB)" + (
                       " fit L2: L2 flushed (256 MiB written) before every timed step, "
                       "outside its events" if cold else " larger than L2")},
        "e2e": {"value": e2e_value, "unit": "GB/s",
                "h2d_bytes_per_step": 3 * elems * 4, "d2h_bytes_per_step": 2 * elems * 4},
        "gpu_launches": 3 * steps,
        "roofline": {"bound": "hbm", "achieved": ach_b, "peak": peak, "unit": "GB/s",
                     "frac": ach_b / peak, "traffic": profiled_traffic("scan_bwd_tma_config3"),
                     "algorithmic_bytes": 20 * elems,
                     "kernel": "scan_bwd_tma (recompute path)",
                     "fwd": {"achieved": ach_f, "frac": ach_f / peak, "ms": f_ms},
                     "bwd_ms": b_ms,
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)"},
        "clocks": clk,
    }


def count_library_kernels(fn) -> int:
    """Number of this library's kernels (namespace tp::) one call of fn launches."""
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return sum(1 for e in prof.events()
               if e.device_type == torch.autograd.DeviceType.CUDA and "tp::" in e.name)


def dtn_workload(args, world, rank):
    """Config 2: DTNAttention(256, 8) forward + backward at B=128 (per rank), L=64."""
    from mk_iii_technologies_tsrn_b200 import ops, _lib
    from mk_iii_technologies_tsrn_b200.dtn import DTNAttention

    _lib.load().tp_set_pointer_checks(0)
    B, L, D, H = local_batch(128, world, args), 64, 256, 8
    dev = torch.device("cuda")
    torch.manual_seed(1 + rank)
    attn = DTNAttention(D, H, dropout=0.0).to(dev)
    with torch.no_grad():
        attn.q_proj.weight.normal_(0.0, 0.02)
        attn.k_proj.weight.normal_(0.0, 0.02)
        attn.maslov.log_temps.copy_(torch.log(torch.rand(H, device=dev) * 0.9 + 0.1))
    attn.train()
    gen = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(B, L, D, device=dev, generator=gen, requires_grad=True)
    g = torch.randn(B, L, D, device=dev, generator=gen)

    def eager_step():
        out, _ = attn(x)
        out.backward(g)

    step = eager_step
    graph = None
    if not args.no_graph:
        # the whole forward + backward captured once and replayed each step:
        # the same kernels without the per-launch host cost of the Python /
        # autograd loop (gradients are rewritten by every replay, as after a
        # zero_grad(set_to_none=True))
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                attn.zero_grad(set_to_none=True)
                x.grad = None
                eager_step()
        torch.cuda.current_stream().wait_stream(side)
        attn.zero_grad(set_to_none=True)
        x.grad = None
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            eager_step()
        step = graph.replay

    for _ in range(args.warmup):
        step()
    steps = steps_for(step, args.steps, world)
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    ms = time_steps_cold(step, steps, world)
    clk = clocks.stop()
    tokens = B * L * world
    value = tokens / (ms / steps / 1e3)
    # dominant kernels (about 40% of the step): the STE backward of a tropical
    # projection (M=B*64, N=K=256): its stats pass and the one-pass gx + gW
    # kernel each evaluate one exponential per (m, n, k) term -> 2*M*N*K per
    # call, against the SFU-bound probe of the same per-term instruction form
    xf = x.detach().reshape(-1, D)
    wq = attn.q_proj.weight.detach()
    y0, _ = ops.maxplus(xf, wq, argmax=False)
    gq = torch.randn(xf.shape[0], D, device=dev, generator=gen)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(3):
        ops.maxplus_backward_smooth("ste", 1.0, xf, wq, gq, ref_max=y0)
    s0.record()
    for _ in range(20):
        ops.maxplus_backward_smooth("ste", 1.0, xf, wq, gq, ref_max=y0)
    s1.record()
    torch.cuda.synchronize()
    kms = s0.elapsed_time(s1) / 20
    achieved = 2.0 * xf.shape[0] * D * D / (kms / 1e3) / 1e12
    ops.probe_addmax(8, 148 * 8, 50)
    pms, terms = ops.probe_addmax(8, 148 * 8, 400)
    peak = terms / (pms / 1e3) / 1e12
    # end to end: activations from pinned host, input gradient back
    hx = x.detach().cpu().pin_memory()
    hgx = torch.empty_like(hx).pin_memory()
    dx = torch.empty_like(x.detach())

    def e2e_step():
        dx.copy_(hx, non_blocking=True)
        xi = dx.requires_grad_(True)
        out, _ = attn(xi)
        out.backward(g)
        hgx.copy_(xi.grad, non_blocking=True)
        xi.grad = None
        dx.requires_grad_(False)

    if graph is not None:
        # the captured step reads the static input x and leaves x.grad: the
        # step's activations arrive in x, its input gradient leaves from x.grad
        def e2e_step():
            with torch.no_grad():
                x.copy_(hx, non_blocking=True)
            graph.replay()
            hgx.copy_(x.grad, non_blocking=True)

    for _ in range(2):
        e2e_step()
    e2e_ms = time_steps(e2e_step, 3, world)
    try:   # counted on an eager step: the graph replays the same kernels
        per_step = count_library_kernels(eager_step)
    except Exception:   # profiler unavailable: leave the count out rather than guess
        per_step = None
    return {
        "metric": "DTN tropical attention block tokens/s (fwd+bwd, train mode)",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms / steps, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: x ~ N(0,1), upstream grad ~ N(0,1), Q/K weights N(0,0.02), "
                "tau_h ~ U(0.1,1) (seeded)",
        "config": {"workload": f"DTNAttention d_model=256 heads=8 B={B * world} L=64 fwd+bwd "
                               "(STE)",
                   "parallelism": parallelism(128, B, world),
                   "launch": "CUDA graph of the whole step" if graph is not None else "eager",
                   "l2": "activations 8 MiB (fit L2): L2 flushed (256 MiB written) before "
                         "every timed step, outside its events"},
        "e2e": {"value": tokens / (e2e_ms / 3 / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": hx.numel() * 4, "d2h_bytes_per_step": hgx.numel() * 4},
        "gpu_launches": per_step * steps if per_step is not None else None,
        "roofline": {"bound": "sfu (ex2)", "achieved": achieved, "peak": peak,
                     "unit": "T exp/s", "frac": achieved / peak, "traffic": None,
                     "kernel": f"STE backward of the Q projection (M={B * L}, N=K=256): stats "
                               "pass + one-pass gx/gW kernel, 2*M*N*K exponentials per call",
                     "kernel_ms": kms,
                     "peak_source": "in-repo SFU probe of the same per-term form "
                                    "(tp_probe_addmax form 8), this run; of measured"},
        "clocks": clk,
    }


def linear_workload(args, world, rank):
    """Config 1: tropical linear x [1024,256] (x) W [256,256] forward with int32 argmax
    plus the argmax backward (upstream g ~ N(0,1)); per rank (weak scaling)."""
    from mk_iii_technologies_tsrn_b200 import ops, _lib

    _lib.load().tp_set_pointer_checks(0)
    M, K, N = local_batch(1024, world, args), 256, 256
    dev = torch.device("cuda")
    gen = torch.Generator().manual_seed(rank)
    hx = torch.randn(M, K, generator=gen).pin_memory()
    hw = torch.randn(N, K, generator=gen)
    hg = torch.randn(M, N, generator=gen).pin_memory()
    x = hx.to(dev).requires_grad_(True)
    w = hw.to(dev).requires_grad_(True)
    gy = hg.to(dev)

    def step(xi=x, gi=gy):
        y = ops.MaxPlusLinearFunction.apply(xi, w, None, "argmax", 1.0)
        gx, gw = torch.autograd.grad(y, (xi, w), gi)
        return y, gx, gw

    # parity on this workload before timing: values and the gradient scatter
    y, gx, gw = step()
    ry, ri, rgx, rgw = oracle_linear(hx, hw, hg)
    if not torch.equal(y.detach().cpu(), ry):
        raise RuntimeError("config-1 forward differs from the reference expression")
    if (gx.cpu() - rgx).abs().max() > 1e-4 or (gw.cpu() - rgw).abs().max() > 1e-3:
        raise RuntimeError("config-1 backward differs from the reference autograd")
    steps = max(args.steps, 50)
    timed = step
    graph = None
    if not args.no_graph:
        # forward + backward captured once and replayed: the step is a few
        # short kernels, so per-launch host cost would otherwise dominate (the
        # gradients land in xs.grad / ws.grad, rewritten by every replay).
        # Fresh leaves: autograd binds a leaf's gradient accumulation to the
        # stream of its first backward, which must not be the legacy stream.
        xs = x.detach().clone().requires_grad_(True)
        ws = w.detach().clone().requires_grad_(True)

        def graph_step():
            y = ops.MaxPlusLinearFunction.apply(xs, ws, None, "argmax", 1.0)
            y.backward(gy)
            return y

        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                xs.grad = ws.grad = None
                graph_step()
        torch.cuda.current_stream().wait_stream(side)
        xs.grad = ws.grad = None
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            static_y = graph_step()
        graph.replay()
        torch.cuda.synchronize()
        if not torch.equal(static_y.detach().cpu(), ry) or \
                (xs.grad.cpu() - rgx).abs().max() > 1e-4:
            raise RuntimeError("config-1 step replayed from the CUDA graph differs")
        timed = graph.replay
    for _ in range(max(args.warmup, 10)):
        timed()
    steps = steps_for(timed, steps, world)
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    ms = time_steps_cold(timed, steps, world)
    clk = clocks.stop()
    ops_step = 2.0 * M * N * K
    value = ops_step * world / (ms / steps / 1e3) / 1e9
    # dominant kernel: the forward with argmax, timed alone
    xd = x.detach()
    wd = w.detach()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ops.maxplus(xd, wd)
    e0.record()
    for _ in range(50):
        ops.maxplus(xd, wd)
    e1.record()
    torch.cuda.synchronize()
    kms = e0.elapsed_time(e1) / 50
    probe = []
    for form in range(5):
        ops.probe_addmax(form, 148 * 8, 50)
        pms, terms = ops.probe_addmax(form, 148 * 8, 400)
        probe.append(2.0 * terms / (pms / 1e3) / 1e12)
    peak = max(probe)
    achieved = ops_step / (kms / 1e3) / 1e12
    # end to end: x and g from pinned host, y and gx back
    dx = torch.empty_like(xd)
    dg = torch.empty_like(gy)
    hy = torch.empty(M, N).pin_memory()
    hgx = torch.empty(M, K).pin_memory()

    def e2e_step():
        dx.copy_(hx, non_blocking=True)
        dg.copy_(hg, non_blocking=True)
        xi = dx.requires_grad_(True)
        y, gx, _ = step(xi, dg)
        hy.copy_(y.detach(), non_blocking=True)
        hgx.copy_(gx, non_blocking=True)
        dx.requires_grad_(False)

    if graph is not None:
        def e2e_step():   # inputs into the captured step's static tensors
            with torch.no_grad():
                xs.copy_(hx, non_blocking=True)
            gy.copy_(hg, non_blocking=True)
            graph.replay()
            hy.copy_(static_y.detach(), non_blocking=True)
            hgx.copy_(xs.grad, non_blocking=True)

    for _ in range(5):
        e2e_step()
    e2e_ms = time_steps(e2e_step, steps, world)
    try:
        per_step = count_library_kernels(step)
    except Exception:   # profiler unavailable: leave the count out rather than guess
        per_step = None
    return {
        "metric": "tropical linear fwd+argmax+bwd Gop/s (2*M*N*K forward ops per step)",
        "value": value, "unit": "Gop/s", "n_gpus": world, "steps": steps,
        "warmup": max(args.warmup, 10), "ms_per_step": ms / steps, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: x, W, g ~ N(0,1) (seeded)",
        "config": {"workload": f"tropical linear M={M * world} K=256 N=256 fwd + int32 argmax "
                               "+ argmax backward (eval mode), no bias",
                   "parallelism": parallelism(1024, M, world, "rows"),
                   "launch": "CUDA graph of the whole step" if graph is not None else "eager",
                   "l2": "inputs 2 MiB (smaller than L2): L2 flushed (256 MiB written) before "
                         "every timed step, outside its events"},
        "e2e": {"value": ops_step * world / (e2e_ms / steps / 1e3) / 1e9, "unit": "Gop/s",
                "h2d_bytes_per_step": (hx.numel() + hg.numel()) * 4,
                "d2h_bytes_per_step": (hy.numel() + hgx.numel()) * 4},
        "gpu_launches": per_step * steps if per_step is not None else None,
        "roofline": {"bound": "cuda-core", "achieved": achieved, "peak": peak, "unit": "Top/s",
                     "frac": achieved / peak, "traffic": None,
                     "kernel": f"max-plus forward with argmax (M={M}, N=K=256): too few "
                               "tiles to fill 148 SMs",
                     "kernel_ms": kms,
                     "peak_source": "in-repo add+max probe, best form, this run; of measured"},
        "clocks": clk,
    }


TSRN_ATT = dict(B=64, H=8, T=1024, dh=80, top_k=16)   # TSRN block at scale 1 (config 5)


def tsrn_attn_workload(args, world, rank):
    """The TSRN tropical top-k attention of config 5 at scale 1 (B=64 per rank, H=8,
    T=1024, d_h=80, top_k=16, causal): the fused kernel from Q/K/V (after QK-norm and
    RoPE) to the attention context."""
    from mk_iii_technologies_tsrn_b200 import ops, _lib

    _lib.load().tp_set_pointer_checks(0)
    B, H, T, dh, k = (TSRN_ATT[n] for n in ("B", "H", "T", "dh", "top_k"))
    B = local_batch(args.att_batch, world, args)
    dev = torch.device("cuda")
    gen = torch.Generator().manual_seed(10 + rank)
    # LayerNorm'd, rotated Q and K have unit-variance entries; V as projected
    hQ = torch.randn(B, H, T, dh, generator=gen).pin_memory()
    hK = torch.randn(B, H, T, dh, generator=gen).pin_memory()
    hV = torch.randn(B, H, T, dh, generator=gen).pin_memory()
    Q, K, V = hQ.to(dev), hK.to(dev), hV.to(dev)
    slopes = (2.0 ** (-8.0 / H * (torch.arange(H, dtype=torch.float32) + 1))).to(dev)
    # parity on a slice of this workload before timing (oracle on CPU, fp64)
    if rank == 0:
        import numpy as np
        import oracle
        out = ops.tsrn_attention(Q[:1, :2, :256].contiguous(), K[:1, :2, :256].contiguous(),
                                 V[:1, :2, :256].contiguous(), slopes[:2], k, True)
        ref, S = oracle.tsrn_attention_fwd(hQ[:1, :2, :256].numpy(), hK[:1, :2, :256].numpy(),
                                           hV[:1, :2, :256].numpy(), slopes[:2].cpu().numpy(),
                                           k, True)
        srt = -np.sort(-S, axis=-1)
        with np.errstate(invalid="ignore"):          # -inf - -inf in fully masked rows
            gap = np.abs(srt[..., k - 1] - srt[..., k])
        ok = ~(np.isfinite(gap) & (gap < 1e-4))     # rows whose top-k cut is not a near-tie
        if not np.allclose(out.cpu().numpy()[ok], ref[ok], rtol=1e-4, atol=2e-5):
            raise RuntimeError("fused TSRN attention differs from the oracle")

    def step():
        return ops.tsrn_attention(Q, K, V, slopes, k, True)

    for _ in range(args.warmup):
        step()
    steps = steps_for(step, args.steps, world)
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    ms = time_steps(step, steps, world)
    clk = clocks.stop()
    tokens = B * T * world
    value = tokens / (ms / steps / 1e3)
    # roofline: the score contraction on the tensor cores (causal: sum over rows of
    # (i+1) keys; three TF32 products of dh multiply-adds each, the 3xTF32 split)
    # against the dense TF32 rate (half the measured bf16 GEMM rate)
    tf32_flops = 3 * 2.0 * B * H * dh * T * (T + 1) / 2
    peak = tf32_peak()
    achieved = tf32_flops / (ms / steps / 1e3) / 1e12
    hout = torch.empty(B, H, T, dh).pin_memory()

    def e2e_step():   # the host entry: sequence groups' copies overlap the computation
        ops.tsrn_attention_host(hQ, hK, hV, slopes, k, True, out=hout)

    for _ in range(2):
        e2e_step()
    e2e_steps = max(3, min(args.steps, 5))
    e2e_ms = time_steps(e2e_step, e2e_steps, world)
    try:
        per_step = count_library_kernels(step)
    except Exception:   # profiler unavailable: leave the count out rather than guess
        per_step = None
    return {
        "metric": "TSRN tropical top-k attention tokens/s (fused fwd, inference)",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms / steps, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: Q, K, V ~ N(0,1) (seeded; the statistics of LayerNorm'd, rotated "
                "Q/K), ALiBi slopes 2^(-8(h+1)/H)",
        "config": {"workload": f"TSRN TropicalAttention B={B * world} H={H} T={T} d_h={dh} "
                               f"top_k={k} causal (config 5, scale 1)",
                   "parallelism": parallelism(args.att_batch, B, world),
                   "l2": f"Q/K/V 3 x {B * H * T * dh * 4 >> 20} MiB"},
        "e2e": {"value": tokens / (e2e_ms / e2e_steps / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": 3 * hQ.numel() * 4, "d2h_bytes_per_step": hout.numel() * 4},
        "gpu_launches": per_step * steps if per_step is not None else None,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s", "frac": achieved / peak,
                     "traffic": (profiled_traffic("att_tc_kernel_b64") * B // 64
                                 if profiled_traffic("att_tc_kernel_b64") else None),
                     "kernel": "att_tc_kernel (tcgen05 kind::tf32 score contraction, 3xTF32, "
                               "causal) incl. its two-pass top-k selection and V gather",
                     "limiter": "the per-score selection epilogue, not the tensor pipe "
                                "(ncu at B=8: issue active 39%, tensor pipe 9.6%)",
                     "peak_source": TF32_PEAK_SOURCE},
        "clocks": clk,
    }


# config 5 reservoir: research/tsrn_dml.py:1073, d_reservoir = d_model // 2 (GRU);
# tsrn_gpu.py:615 builds the leaky one with d_reservoir = d_model
ESN = dict(B=64, T=1024, dr_leaky=640, dr_gru=320)


def esn_inputs(mode, B, T, gen):
    """Reservoir inputs with the reference modules' statistics: U = W_in(LayerNorm(x))
    (default nn.Linear init: entries of variance 1/3), W_res sparse N(0,1) at 10% density
    scaled to spectral radius sigmoid(0) * 1.5 = 0.75, leak sigmoid(0.3); GRU gates from
    zero-initialised weights plus N(0, 0.1^2) (a trained-from-init state) and the
    reference's biases 0.85 / 2.0."""
    dr = ESN["dr_leaky"] if mode == "leaky" else ESN["dr_gru"]
    U = torch.randn(B, T, dr, generator=gen) / math.sqrt(3.0)
    W = torch.randn(dr, dr, generator=gen) * (torch.rand(dr, dr, generator=gen) > 0.9).float()
    Ws = W * (0.75 / torch.linalg.eigvals(W).abs().max().real)
    if mode == "leaky":
        return dr, (U, Ws, torch.sigmoid(torch.tensor(0.3)))
    Wz_u, Wr_u, Wzh, Wrh = (0.1 * torch.randn(dr, dr, generator=gen) / math.sqrt(dr)
                            for _ in range(4))
    Uz = U @ Wz_u.T + 0.85
    Ur = U @ Wr_u.T + 2.0
    return dr, (U, Uz, Ur, Wzh, Wrh, Ws)


def esn_workload(args, world, rank):
    """The reservoir recurrence of config 5's first block (GRU, d_reservoir 320; or the
    leaky tsrn_gpu.py one), B=64 sequences per rank of T=1024 steps, fused (one launch
    per call) from the input projections to H."""
    from mk_iii_technologies_tsrn_b200 import ops, _lib

    _lib.load().tp_set_pointer_checks(0)
    mode, B, T = args.esn_mode, local_batch(ESN["B"], world, args), ESN["T"]
    dev = torch.device("cuda")
    gen = torch.Generator().manual_seed(20 + rank)
    dr, host = esn_inputs(mode, B, T, gen)
    hU = host[0].pin_memory()
    dev_in = [t.to(dev) for t in host]
    fn = ops.esn_leaky_fwd if mode == "leaky" else ops.esn_gru_fwd
    # parity on a slice of this workload before timing (oracle on CPU, fp64)
    if rank == 0:
        import numpy as np
        import oracle
        Bs, Ts = 2, 64
        sl = [t[:Bs, :Ts].contiguous() if t.dim() == 3 else t for t in dev_in]
        out = fn(*sl).cpu().numpy()
        hs = [t.cpu().numpy() for t in sl]
        ref = oracle.esn_leaky_fwd(*hs) if mode == "leaky" else oracle.esn_gru_fwd(*hs)
        if not np.allclose(out, ref, rtol=0, atol=2e-5):
            raise RuntimeError("fused reservoir recurrence differs from the oracle")

    def step():
        return fn(*dev_in)

    for _ in range(args.warmup):
        step()
    steps = steps_for(step, args.steps, world)
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    ms = time_steps(step, steps, world)
    clk = clocks.stop()
    tokens = B * T * world
    value = tokens / (ms / steps / 1e3)
    gates = 1 if mode == "leaky" else 3
    peak = ffma_peak()
    achieved = 2.0 * gates * B * T * dr * dr / (ms / steps / 1e3) / 1e12
    hH = torch.empty(B, T, dr).pin_memory()

    def e2e_step():   # the host entry: time windows' copies overlap the recurrence
        if mode == "leaky":
            ops.esn_fwd_host(hU, dev_in[1], lk=dev_in[2].reshape(1).to(dev), out=hH)
        else:   # Uz, Ur derive from U on the device in the module: read in place
            ops.esn_fwd_host(hU, dev_in[5], Uz=dev_in[1], Ur=dev_in[2], Wzh=dev_in[3],
                             Wrh=dev_in[4], out=hH)

    for _ in range(2):
        e2e_step()
    e2e_steps = max(3, min(args.steps, 5))
    e2e_ms = time_steps(e2e_step, e2e_steps, world)
    try:
        per_step = count_library_kernels(step)
    except Exception:   # profiler unavailable: leave the count out rather than guess
        per_step = None
    name = ("leaky EchoStateReservoir (tsrn_gpu.py)" if mode == "leaky"
            else "GRU-gated EchoStateReservoir (research/tsrn_dml.py)")
    return {
        "metric": f"echo-state reservoir tokens/s ({mode}, fused recurrence, inference)",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms / steps, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded): U with the statistics of W_in(LayerNorm(x)), sparse "
                "W_res scaled to spectral radius 0.75" + ("" if mode == "leaky" else
                                                          ", GRU gate inputs"),
        "config": {"workload": f"{name} d_reservoir={dr} B={B * world} T={T}" +
                               (" (config 5 first-block reservoir)" if mode == "gru" else ""),
                   "parallelism": parallelism(ESN["B"], B, world),
                   "l2": f"U and H {B * T * dr * 4 / 2**20:.0f} MiB each"},
        "e2e": {"value": tokens / (e2e_ms / e2e_steps / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": hU.numel() * 4, "d2h_bytes_per_step": hH.numel() * 4},
        "gpu_launches": per_step * steps if per_step is not None else None,
        "roofline": {"bound": "cuda-core fp32 FMA (recurrent mat-vec products); the "
                              "recurrence is latency-bound per step",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": None,
                     "kernel": "esn_kernel",
                     "peak_source": "in-repo register-only FMA probe (tp_probe_addmax: best "
                                    "of scalar FFMA form 7 and packed f32x2 form 9), this "
                                    "run; of measured"},
        "clocks": clk,
    }


TSRN_BLOCK = dict(B=64, T=1024, d=640, H=8, top_k=16)   # config 5, scale-1 block 0


def _tsrn_block_module(dev, seed):
    """TSRNTropicalPath at config 5's block-0 shape, reference initialisation, with
    the zero-initialised output projections (reservoir readout, SSM C_proj and
    gates) drawn small so that every branch changes the residual stream."""
    from mk_iii_technologies_tsrn_b200.tsrn_block import TSRNTropicalPath
    torch.manual_seed(seed)
    d, H, k = TSRN_BLOCK["d"], TSRN_BLOCK["H"], TSRN_BLOCK["top_k"]
    m = TSRNTropicalPath(d, k, H)
    with torch.no_grad():
        m.reservoir.readout.weight.normal_(0.0, 0.02)
        m.reservoir.W_z.weight.normal_(0.0, 0.02)
        m.reservoir.W_r.weight.normal_(0.0, 0.02)
        m.tropical_ssm.C_proj.weight.normal_(0.0, 0.02)
        m.tropical_ssm.gate_B.weight.normal_(0.0, 0.02)
        m.tropical_ssm.gate_out.weight.normal_(0.0, 0.02)
        m.reservoir._cached_v.normal_()    # the power iteration's start, seeded here
    return m.to(dev).eval()


def tsrn_block_workload(args, world, rank):
    """Config 5's hot path: the tropical branches of the first TSRN block
    (research/tsrn_dml.py:1096-1106, scale 1: d=640, 8 heads, top_k=16) -- fused
    top-k attention, GRU echo-state reservoir (d_r=320), tropical SSM scan
    (h_init=0) with their LayerNorms and projections -- inference on B=64 sequences
    of T=1024 tokens (split over the ranks)."""
    from mk_iii_technologies_tsrn_b200 import ops, _lib

    _lib.load().tp_set_pointer_checks(0)
    B = local_batch(TSRN_BLOCK["B"], world, args)
    T, d, H, k = TSRN_BLOCK["T"], TSRN_BLOCK["d"], TSRN_BLOCK["H"], TSRN_BLOCK["top_k"]
    dev = torch.device("cuda")
    m = _tsrn_block_module(dev, 30)
    gen = torch.Generator().manual_seed(40 + rank)
    hx = torch.randn(B, T, d, generator=gen).pin_memory()
    x = hx.to(dev)
    names = ("attn", "reservoir", "tropical_ssm")
    branch_ms = {n: [] for n in names}

    def step(record=False):
        ev = None
        if record:
            ev = {n: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for n in names}
        with torch.no_grad():
            y = m(x, events=ev)
        if record:
            for n in names:
                branch_ms[n].append(ev[n])
        return y

    # parity on a slice before timing: the CPU port of the reference block
    if rank == 0:
        from oracle.torch_ref import tsrn_block_torch
        sd = {kk: v.detach().cpu() for kk, v in m.state_dict().items()}
        xs = hx[:1, :128].clone()
        with torch.no_grad():
            got = m(xs.to(dev)).cpu()
        ref = tsrn_block_torch(xs, sd, H, k)
        err = (got - ref).abs().max().item()
        if not err < 2e-3:
            raise RuntimeError(f"TSRN block tropical path differs from the reference port ({err})")
    for _ in range(args.warmup):
        step()
    steps = steps_for(step, args.steps, world)
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    ms = time_steps(lambda: step(True), steps, world)
    clk = clocks.stop()
    tokens = B * T * world
    value = tokens / (ms / steps / 1e3)
    share = {n: max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in branch_ms[n]),
                               world) for n in names}
    step_ms = ms / steps
    # the two recurrent / selection kernels timed alone on this step's inputs
    with torch.no_grad():
        xa = m.ln_attn(x)
        Q, K, V = m.attn.project(xa)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ops.tsrn_attention(Q, K, V, m.attn.alibi_slopes, k, True)
        e0.record()
        for _ in range(3):
            ops.tsrn_attention(Q, K, V, m.attn.alibi_slopes, k, True)
        e1.record()
        torch.cuda.synchronize()
        att_ms = e0.elapsed_time(e1) / 3
        esn_in = m.reservoir.recurrence_inputs(m.ln_res(x))
        ops.esn_gru_fwd(*esn_in)
        e0.record()
        for _ in range(3):
            ops.esn_gru_fwd(*esn_in)
        e1.record()
        torch.cuda.synchronize()
        esn_ms = e0.elapsed_time(e1) / 3
        del Q, K, V, esn_in, xa
    dr = d // 2
    att_flops = 3 * 2.0 * B * H * (d // H) * T * (T + 1) / 2
    esn_flops = 2.0 * 3 * B * T * dr * dr
    if att_ms >= esn_ms:
        dom = {"kernel": "att_tc_kernel (tcgen05 3xTF32 score contraction, causal, with its "
                         "top-k selection)", "bound": "tensor", "peak": tf32_peak(),
               "peak_source": TF32_PEAK_SOURCE,
               "achieved": att_flops / (att_ms / 1e3) / 1e12, "kernel_ms": att_ms}
    else:
        dom = {"kernel": "esn_kernel (GRU reservoir recurrence; latency-bound per step)",
               "bound": "cuda-core fp32 FMA", "peak": ffma_peak(),
               "peak_source": "in-repo register-only FMA probe (tp_probe_addmax: best of "
                              "scalar FFMA form 7 and packed f32x2 form 9), this run; of "
                              "measured",
               "achieved": esn_flops / (esn_ms / 1e3) / 1e12, "kernel_ms": esn_ms}
    hy = torch.empty(B, T, d).pin_memory()
    dx = torch.empty_like(x)

    def e2e_step():
        dx.copy_(hx, non_blocking=True)
        with torch.no_grad():
            y = m(dx)
        hy.copy_(y, non_blocking=True)

    for _ in range(2):
        e2e_step()
    e2e_steps = max(3, min(args.steps, 5))
    e2e_ms = time_steps(e2e_step, e2e_steps, world)
    try:
        per_step = count_library_kernels(step)
    except Exception:   # profiler unavailable: leave the count out rather than guess
        per_step = None
    return {
        "metric": "TSRN block tropical path tokens/s (attention + reservoir + SSM, inference)",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: x ~ N(0,1) residual stream (seeded), reference initialisation "
                "(zero-initialised output projections drawn N(0,0.02))",
        "config": {"workload": f"TSRN block-0 tropical branches B={B * world} T={T} d={d} "
                               f"H={H} top_k={k} d_reservoir={dr} (config 5, scale 1)",
                   "parallelism": parallelism(TSRN_BLOCK["B"], B, world),
                   "branch_ms": share,
                   "branch_share": {n: share[n] / step_ms for n in names},
                   "hot_kernel_ms": {"tsrn_attention": att_ms, "esn_gru": esn_ms},
                   "not_included": "sheaf diffusion, Clifford FFN, p-adic memory and the "
                                   "embedding / head of the 50.19M-parameter model "
                                   "(non-tropical)",
                   "l2": f"residual stream {B * T * d * 4 >> 20} MiB"},
        "e2e": {"value": tokens / (e2e_ms / e2e_steps / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": hx.numel() * 4, "d2h_bytes_per_step": hy.numel() * 4},
        "gpu_launches": per_step * steps if per_step is not None else None,
        "roofline": {"bound": dom["bound"] + " (dominant kernel)", "achieved": dom["achieved"],
                     "peak": dom["peak"], "unit": "TFLOP/s", "frac": dom["achieved"] / dom["peak"],
                     "traffic": None, "kernel": dom["kernel"], "kernel_ms": dom["kernel_ms"],
                     "peak_source": dom["peak_source"]},
        "clocks": clk,
    }


def tsrn_train_workload(args, world, rank):
    """Config 5's tropical branches in training: the first TSRN block's attention
    (tensor-core forward saving each row's kept keys, sparse backward), GRU
    reservoir (one-launch forward and backward through time) and tropical SSM
    (scan forward, argmax-path backward) with their LayerNorms and fp32
    projections under autograd -- forward + backward of B=64 sequences of
    T=1024 tokens (split over the ranks), gradients for every parameter and the
    input."""
    from mk_iii_technologies_tsrn_b200 import ops, _lib

    _lib.load().tp_set_pointer_checks(0)
    B = local_batch(TSRN_BLOCK["B"], world, args)
    T, d, H, k = TSRN_BLOCK["T"], TSRN_BLOCK["d"], TSRN_BLOCK["H"], TSRN_BLOCK["top_k"]
    dev = torch.device("cuda")
    m = _tsrn_block_module(dev, 30).train()
    gen = torch.Generator().manual_seed(50 + rank)
    hx = torch.randn(B, T, d, generator=gen).pin_memory()
    hg = torch.randn(B, T, d, generator=gen).pin_memory()
    x = hx.to(dev).requires_grad_(True)
    gy = hg.to(dev)

    def step():
        m.zero_grad(set_to_none=True)
        x.grad = None
        y = m(x)
        y.backward(gy)
        return y

    # before timing: the training forward agrees with the inference forward on a
    # slice (fp32 against 3xTF32 projections, the PyTorch prologue against the
    # fused one: rounding, and near-ties at the top-k cut), and every gradient is
    # finite
    if rank == 0:
        xs = x[:1, :256].detach().clone().requires_grad_(True)
        ys = m(xs)
        with torch.no_grad():
            ye = m(xs.detach())
        ys.sum().backward()
        err = ((ys.detach() - ye).abs().max() / ye.abs().max()).item()
        bad = [n for n, prm in m.named_parameters()
               if prm.grad is None or not torch.isfinite(prm.grad).all()]
        if not err < 2e-3 or bad or not torch.isfinite(xs.grad).all():
            raise RuntimeError(f"TSRN training step check failed ({err}, {bad[:3]})")
        m.zero_grad(set_to_none=True)
    for _ in range(args.warmup):
        step()
    steps = steps_for(step, args.steps, world)
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    ms = time_steps(step, steps, world)
    clk = clocks.stop()
    tokens = B * T * world
    value = tokens / (ms / steps / 1e3)
    # the dominant kernel, timed alone on this step's inputs: the reservoir's
    # backward through time (three dr x dr products per step, as the forward)
    dr = d // 2
    with torch.no_grad():
        U, Uz, Ur, Wzh, Wrh, Ws = m.reservoir.recurrence_inputs(m.ln_res(x.detach()))
        Hs = ops.esn_gru_fwd(U, Uz, Ur, Wzh, Wrh, Ws)
        fac = [torch.rand_like(Hs) * 0.25 for _ in range(5)]
        dH = torch.randn_like(Hs)
        ops.esn_gru_bwd(dH, *fac, Wzh, Wrh, Ws)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(3):
            ops.esn_gru_bwd(dH, *fac, Wzh, Wrh, Ws)
        e1.record()
        torch.cuda.synchronize()
        bptt_ms = e0.elapsed_time(e1) / 3
        del U, Uz, Ur, Hs, fac, dH
    peak = ffma_peak()
    achieved = 2.0 * 3 * B * T * dr * dr / (bptt_ms / 1e3) / 1e12
    hdx = torch.empty(B, T, d).pin_memory()

    def e2e_step():   # inputs and the upstream gradient from host, dL/dx back to host
        with torch.no_grad():
            x.copy_(hx, non_blocking=True)
            gy.copy_(hg, non_blocking=True)
        step()
        hdx.copy_(x.grad, non_blocking=True)

    for _ in range(2):
        e2e_step()
    e2e_steps = max(3, min(args.steps, 5))
    e2e_ms = time_steps(e2e_step, e2e_steps, world)
    try:
        per_step = count_library_kernels(step)
    except Exception:   # profiler unavailable: leave the count out rather than guess
        per_step = None
    return {
        "metric": "TSRN block tropical path training tokens/s (attention + reservoir + SSM, "
                  "fwd + bwd)",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms / steps, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: x and the upstream gradient ~ N(0,1) (seeded), reference "
                "initialisation (zero-initialised output projections drawn N(0,0.02))",
        "config": {"workload": f"TSRN block-0 tropical branches, training step, B={B * world} "
                               f"T={T} d={d} H={H} top_k={k} d_reservoir={dr} (config 5)",
                   "parallelism": parallelism(TSRN_BLOCK["B"], B, world),
                   "bptt_kernel_ms": bptt_ms,
                   "l2": f"residual stream {B * T * d * 4 >> 20} MiB"},
        "e2e": {"value": tokens / (e2e_ms / e2e_steps / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": 2 * hx.numel() * 4, "d2h_bytes_per_step": hdx.numel() * 4},
        "gpu_launches": per_step * steps if per_step is not None else None,
        "roofline": {"bound": "cuda-core fp32 FMA (dominant kernel)", "achieved": achieved,
                     "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                     "traffic": (profiled_traffic("esn_bwd_kernel_b64") * B // 64
                                 if profiled_traffic("esn_bwd_kernel_b64") else None),
                     "kernel": "esn_bwd_kernel (GRU reservoir backward through time; "
                               "latency-bound per step)", "kernel_ms": bptt_ms,
                     "peak_source": "in-repo register-only FMA probe (tp_probe_addmax: best "
                                    "of scalar FFMA form 7 and packed f32x2 form 9), this "
                                    "run; of measured"},
        "clocks": clk,
    }


def cpu_tsrn_train_rate(target_s: float = 10.0):
    """The reference block's tropical branches on CPU torch (oracle/torch_ref.py) with
    autograd: forward + backward of one sequence of T=1024 tokens."""
    from oracle.torch_ref import tsrn_block_torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    m = _tsrn_block_module(torch.device("cpu"), 30)
    params = {n for n, _ in m.named_parameters()}
    T, d, H, k = TSRN_BLOCK["T"], TSRN_BLOCK["d"], TSRN_BLOCK["H"], TSRN_BLOCK["top_k"]
    gen = torch.Generator().manual_seed(50)
    x = torch.randn(1, T, d, generator=gen)
    gy = torch.randn(1, T, d, generator=gen)

    def one():
        sd = {n: v.detach().clone().requires_grad_(n in params)
              for n, v in m.state_dict().items()}
        xx = x.clone().requires_grad_(True)
        tsrn_block_torch(xx, sd, H, k).backward(gy)

    t0 = time.perf_counter()
    one()
    dt = time.perf_counter() - t0
    reps = int(max(1, min(10, target_s / max(dt, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(reps):
        one()
    dt = (time.perf_counter() - t0) / reps
    return {"value": T / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"1 of {TSRN_BLOCK['B']} sequences (T={T}) through the reference "
                      f"block's tropical branches on CPU torch, forward + autograd backward, "
                      f"{reps} reps, {dt:.2f} s each"}


def cpu_tsrn_block_rate(target_s: float = 10.0):
    """The reference block's tropical branches on CPU torch (oracle/torch_ref.py, pinned
    to the reference module) on one sequence of T=1024 tokens."""
    from oracle.torch_ref import tsrn_block_torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    m = _tsrn_block_module(torch.device("cpu"), 30)
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    T, d, H, k = TSRN_BLOCK["T"], TSRN_BLOCK["d"], TSRN_BLOCK["H"], TSRN_BLOCK["top_k"]
    x = torch.randn(1, T, d, generator=torch.Generator().manual_seed(40))
    with torch.no_grad():
        t0 = time.perf_counter()
        tsrn_block_torch(x, sd, H, k)
        dt = time.perf_counter() - t0
        reps = int(max(1, min(10, target_s / max(dt, 1e-6))))
        t0 = time.perf_counter()
        for _ in range(reps):
            tsrn_block_torch(x, sd, H, k)
        dt = (time.perf_counter() - t0) / reps
    return {"value": T / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"1 of {TSRN_BLOCK['B']} sequences (T={T}) through the reference "
                      f"block's tropical branches on CPU torch, {reps} reps, {dt:.2f} s each"}


def cpu_esn_rate(mode, target_s: float = 10.0):
    from oracle.torch_ref import esn_gru_torch, esn_leaky_torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    B, T = ESN["B"], ESN["T"]
    gen = torch.Generator().manual_seed(20)
    dr, host = esn_inputs(mode, B, T, gen)
    fn = esn_leaky_torch if mode == "leaky" else esn_gru_torch
    t0 = time.perf_counter()
    fn(*host)
    dt = time.perf_counter() - t0
    reps = int(max(1, min(20, target_s / max(dt, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(reps):
        fn(*host)
    dt = (time.perf_counter() - t0) / reps
    return {"value": B * T / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"B={B}, T={T}: one step of the workload (d_reservoir={dr}) through the "
                      f"reference {mode} loop (oracle/torch_ref.py), {reps} reps, {dt:.2f} s each"}


def cpu_tsrn_attn_rate(target_s: float = 10.0):
    from oracle.torch_ref import tsrn_attention_torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    H, T, dh, k = TSRN_ATT["H"], TSRN_ATT["T"], TSRN_ATT["dh"], TSRN_ATT["top_k"]
    gen = torch.Generator().manual_seed(10)
    Q, K, V = (torch.randn(1, H, T, dh, generator=gen) for _ in range(3))
    slopes = 2.0 ** (-8.0 / H * (torch.arange(H, dtype=torch.float32) + 1))
    t0 = time.perf_counter()
    tsrn_attention_torch(Q, K, V, slopes, k)
    dt = time.perf_counter() - t0
    reps = int(max(1, min(5, target_s / max(dt, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(reps):
        tsrn_attention_torch(Q, K, V, slopes, k)
    dt = (time.perf_counter() - t0) / reps
    return {"value": T / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"one sequence (B=1 of 64, H={H}, T={T}, d_h={dh}) through the reference "
                      f"attention expressions (oracle/torch_ref.py), {reps} reps, {dt:.2f} s each"}


def oracle_linear(hx, hw, hg):
    from oracle.torch_ref import tropical_linear_fwd_bwd_torch

    y, idx, gx, gw = tropical_linear_fwd_bwd_torch(hx, hw, hg)
    return y, idx, gx, gw


def cpu_linear_rate(target_s: float = 10.0):
    from oracle.torch_ref import tropical_linear_fwd_bwd_torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(1024, 256, generator=gen)
    w = torch.randn(256, 256, generator=gen)
    g = torch.randn(1024, 256, generator=gen)
    t0 = time.perf_counter()
    tropical_linear_fwd_bwd_torch(x, w, g)
    dt = time.perf_counter() - t0
    reps = int(max(1, min(50, target_s / max(dt, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(reps):
        tropical_linear_fwd_bwd_torch(x, w, g)
    dt = (time.perf_counter() - t0) / reps
    return {"value": 2.0 * 1024 * 256 * 256 / dt / 1e9, "unit": "Gop/s", "cores": threads,
            "kind": "port",
            "sample": f"the whole config-1 step (reference eval TropicalLinear expression "
                      f"fwd + autograd bwd, oracle/torch_ref.py), {reps} reps, "
                      f"{dt * 1e3:.1f} ms each"}


def cpu_dtn_rate(target_s: float = 10.0):
    from oracle.torch_ref import DTNAttentionRef

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    torch.manual_seed(1)
    ref = DTNAttentionRef(256, 8)
    B = 2
    x = torch.randn(B, 64, 256, requires_grad=True)
    t0 = time.perf_counter()
    out, _ = ref(x)
    out.sum().backward()
    dt = time.perf_counter() - t0
    reps = int(max(1, min(20, target_s / max(dt, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(reps):
        out, _ = ref(x)
        out.sum().backward()
    dt = (time.perf_counter() - t0) / reps
    return {"value": B * 64 / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"reference DTNAttention expressions (oracle/torch_ref.py) fwd+bwd at "
                      f"B={B} of 128, L=64, d=256, H=8; {reps} reps"}


def reference_arm(args, world, rank):
    if rank != 0:
        return None
    if args.workload == "esn":
        cb = cpu_esn_rate(args.esn_mode, target_s=max(3.0, 2.0 * args.steps))
        metric = f"echo-state reservoir tokens/s ({args.esn_mode}, fused recurrence, inference)"
        dr = ESN["dr_leaky"] if args.esn_mode == "leaky" else ESN["dr_gru"]
        cfg = {"workload": f"{args.esn_mode} EchoStateReservoir d_reservoir={dr} "
                           f"B={ESN['B']} T={ESN['T']} (torch CPU)"}
    elif args.workload == "tsrn_block":
        cb = cpu_tsrn_block_rate(target_s=max(3.0, 2.0 * args.steps))
        metric = "TSRN block tropical path tokens/s (attention + reservoir + SSM, inference)"
        cfg = {"workload": "TSRN block-0 tropical branches d=640 H=8 top_k=16 d_reservoir=320 "
                           "T=1024 (torch CPU)"}
    elif args.workload == "tsrn_train":
        cb = cpu_tsrn_train_rate(target_s=max(3.0, 2.0 * args.steps))
        metric = ("TSRN block tropical path training tokens/s (attention + reservoir + SSM, "
                  "fwd + bwd)")
        cfg = {"workload": "TSRN block-0 tropical branches, training step, d=640 H=8 top_k=16 "
                           "d_reservoir=320 T=1024 (torch CPU, autograd)"}
    elif args.workload == "tsrn_attn":
        cb = cpu_tsrn_attn_rate(target_s=max(3.0, 2.0 * args.steps))
        metric = "TSRN tropical top-k attention tokens/s (fused fwd, inference)"
        cfg = {"workload": "TSRN TropicalAttention H=8 T=1024 d_h=80 top_k=16 causal "
                           "(torch CPU)"}
    elif args.workload == "linear":
        cb = cpu_linear_rate(target_s=max(3.0, 2.0 * args.steps))
        metric = "tropical linear fwd+argmax+bwd Gop/s (2*M*N*K forward ops per step)"
        cfg = {"workload": "tropical linear M=1024 K=256 N=256 fwd + argmax + argmax backward "
                           "(torch CPU)"}
    elif args.workload == "dtn":
        cb = cpu_dtn_rate(target_s=max(3.0, 2.0 * args.steps))
        metric = "DTN tropical attention block tokens/s (fwd+bwd, train mode)"
        cfg = {"workload": "DTNAttention d_model=256 heads=8 L=64 fwd+bwd (torch CPU)"}
    elif args.workload == "gemm" and args.dtype == "bf16" and args.arith == "bf16":
        cb = cpu_gemm_rate(args.size, target_s=max(3.0, 2.0 * args.steps), bf16=True)
        metric = "max-plus GEMM Gop/s (bf16 operands, bf16 arithmetic, with int32 argmax)"
        cfg = {"workload": f"maxplus_gemm M=N=K={args.size} bf16 tensors + int64 argmax "
                           f"(torch CPU)", "M": args.size, "N": args.size, "K": args.size}
    elif args.workload == "gemm":
        cb = cpu_gemm_rate(args.size, target_s=max(3.0, 2.0 * args.steps))
        metric = "max-plus GEMM Gop/s (fp32, with int32 argmax)"
        cfg = {"workload": f"maxplus_gemm M=N=K={args.size} fp32 + int64 argmax (torch CPU)",
               "M": args.size, "N": args.size, "K": args.size}
    else:
        cb = cpu_scan_rate(16, 4096, 1024, target_s=max(3.0, 2.0 * args.steps))
        metric = "tropical scan GB/s (fwd 12 B/elem + argmax-path bwd 20 B/elem)"
        cfg = {"workload": "tropical_ssm_scan B=16 T=4096 C=1024 (closed form, torch CPU)"}
    return {"metric": metric, "value": cb["value"], "unit": cb["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded)", "config": cfg, "impl": "reference",
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


SECONDARY_KEYS = ("metric", "value", "unit", "ms_per_step", "steps", "warmup", "scaling",
                  "config", "e2e", "roofline", "clocks", "gpu_launches", "cpu_baseline")


def secondary_workloads(args, world, rank):
    """The other configurations of the hot path, measured in the same run as the
    GEMM headline: each workload with its own warm-up, device-timed steps (max
    over ranks), clocks, roofline, end-to-end and (one GPU) CPU baseline on a
    shorter sample.  Batch workloads are split over the ranks (strong scaling)."""
    import copy
    out = []
    plan = [("scan", scan_workload, lambda: cpu_scan_rate(16, 4096, 1024, target_s=5.0)),
            ("dtn", dtn_workload, lambda: cpu_dtn_rate(target_s=5.0)),
            ("tsrn_attn", tsrn_attn_workload, lambda: cpu_tsrn_attn_rate(target_s=5.0)),
            ("esn", esn_workload, lambda: cpu_esn_rate("gru", target_s=5.0)),
            ("tsrn_block", tsrn_block_workload, lambda: cpu_tsrn_block_rate(target_s=5.0)),
            ("tsrn_train", tsrn_train_workload, lambda: cpu_tsrn_train_rate(target_s=5.0)),
            ("linear", linear_workload, lambda: cpu_linear_rate(target_s=3.0))]
    for name, fn, cpu in plan:
        sub = copy.copy(args)
        sub.workload = name
        sub.steps = max(3, min(args.steps, 10))
        sub.warmup = max(3, min(args.warmup, 5))
        sub.scaling = "strong"
        sub.esn_mode = "gru"
        torch.cuda.empty_cache()
        r = fn(sub, world, rank)
        torch.cuda.synchronize()
        if rank == 0 and r is not None:
            if world == 1 and not args.no_cpu_baseline:
                r["cpu_baseline"] = cpu()
            entry = {"workload": name}
            entry.update({k: r[k] for k in SECONDARY_KEYS if k in r})
            out.append(entry)
    torch.cuda.empty_cache()
    return out


def main():
    args = parse_args()
    world, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            res = reference_arm(args, world, rank)
        elif args.workload == "gemm":
            res = gemm_workload(args, world, rank)
        elif args.workload == "dtn":
            res = dtn_workload(args, world, rank)
        elif args.workload == "linear":
            res = linear_workload(args, world, rank)
        elif args.workload == "tsrn_attn":
            res = tsrn_attn_workload(args, world, rank)
        elif args.workload == "esn":
            res = esn_workload(args, world, rank)
        elif args.workload == "tsrn_block":
            res = tsrn_block_workload(args, world, rank)
        elif args.workload == "tsrn_train":
            res = tsrn_train_workload(args, world, rank)
        else:
            res = scan_workload(args, world, rank)
        if res is not None and args.impl == "ours" and rank == 0 and world == 1 \
                and not args.no_cpu_baseline:
            if args.workload == "gemm":
                res["cpu_baseline"] = cpu_gemm_rate(
                    args.size, bf16=(args.dtype == "bf16" and args.arith == "bf16"))
            elif args.workload == "dtn":
                res["cpu_baseline"] = cpu_dtn_rate()
            elif args.workload == "linear":
                res["cpu_baseline"] = cpu_linear_rate()
            elif args.workload == "tsrn_attn":
                res["cpu_baseline"] = cpu_tsrn_attn_rate()
            elif args.workload == "esn":
                res["cpu_baseline"] = cpu_esn_rate(args.esn_mode)
            elif args.workload == "tsrn_block":
                res["cpu_baseline"] = cpu_tsrn_block_rate()
            elif args.workload == "tsrn_train":
                res["cpu_baseline"] = cpu_tsrn_train_rate()
            else:
                res["cpu_baseline"] = cpu_scan_rate(16, 4096, 1024)
        if args.impl == "ours" and args.workload == "gemm" and not args.no_secondary \
                and args.dtype == "f32" and args.size == 8192:
            sec = secondary_workloads(args, world, rank)
            if res is not None:
                res["secondary"] = sec
        if rank == 0 and res is not None:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1 and torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
