"""Tensor-level tropical ops over the C ABI, plus their autograd functions.

Every op here runs the sm_100a kernels of ``_tropical_b200.so`` on the
tensors' CUDA device and the current stream.  CPU tensors are rejected with a
RuntimeError: there is deliberately no CPU fallback (the reference binding's
silent fallback, ``cuda/maxplus_binding.py:137-148``, hid the fact that its
GPU path never ran correctly).

Reference expressions each op replaces (Mediocr3Mik3/MK_III_Technologies_TSRN):

* :func:`maxplus` -- ``scores = W[None] + x[:, None]; scores.max(-1)`` plus bias
  (``tropformer.py:127-145``); values and int32 argmax bit-exact.
* :func:`tropical_scores` -- ``_tropical_max(Q.unsqueeze(3) + K.unsqueeze(2), -1) * scale``
  (``deep_tropical_net.py:148-150``, ``tropformer.py:378-381``).
* :func:`lse_scores` -- ``logsumexp_c(Q[..., :, None, c] + K[..., None, :, c])``, the TSRN
  tropical attention score (``research/tsrn_dml.py:438-460``).
* :func:`tropical_scan` -- the ``TropicalSSM`` max-plus recurrence
  (``research/tsrn_dml.py:961-972``), evaluated as the exact sequential recurrence.
"""
from __future__ import annotations

import contextlib
import ctypes
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import TP_BWD_LSE, TP_BWD_STE, TP_DTYPE_BF16, TP_DTYPE_BF16_ARITH, TP_DTYPE_F32

MODES = ("argmax", "ste", "lse")


# --------------------------------------------------------------------------- helpers
def _require_cuda(*tensors: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "tropical ops run only on CUDA tensors (sm_100a kernels); got a "
                f"{t.device} tensor -- there is no CPU fallback"
            )
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise RuntimeError("no tensor arguments")
    return dev


class DeviceWaitTimeout(RuntimeError):
    """A bounded wait inside a kernel ran out of its budget: that kernel returned
    early and its outputs (and those of later kernels that read them) are
    incomplete."""

    def __init__(self, code: int, device):
        what = {_lib.TP_DEVERR_BARRIER_TIMEOUT: "an mbarrier wait (TMA pipeline or cluster "
                                                "exchange)",
                _lib.TP_DEVERR_FLAG_TIMEOUT: "a flag wait (stream-K partials)"}.get(
                    code, f"device error code {code}")
        super().__init__(f"{what} on {device} ran out of its wait budget; the kernel "
                         "returned early and its results are incomplete")
        self.code = code


def check_device_error(device=None, reset: bool = True) -> None:
    """Raise :class:`DeviceWaitTimeout` if a kernel on ``device`` (default: the
    current CUDA device) recorded a timed-out wait since the last reset.

    Synchronises with the device.  The library's kernels never hang: a wait that
    cannot complete ends after the budget (:func:`set_wait_budget`) and leaves a
    code here, which this call turns into an exception (and clears, unless
    ``reset`` is False)."""
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None \
        else torch.device(device)
    with torch.cuda.device(dev):
        code = lib.tp_device_error(1 if reset else 0)
    if code < 0:
        raise _lib.TropicalLibraryError("tp_device_error", -code, f"CUDA error {-code}")
    if code:
        raise DeviceWaitTimeout(code, dev)


def set_wait_budget(seconds: float, device=None) -> float:
    """Set the budget of every bounded device-side wait on ``device`` (default
    2 s) and return the previous one, in seconds.  Synchronous; not during
    stream capture."""
    lib = _lib.load()
    prev = ctypes.c_int64(0)
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None \
        else torch.device(device)
    with torch.cuda.device(dev):
        st = lib.tp_set_wait_budget_ns(int(round(seconds * 1e9)), ctypes.byref(prev))
    _lib.check(st, "tp_set_wait_budget_ns")
    return prev.value / 1e9


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(dev: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return TP_DTYPE_F32
    if t.dtype == torch.bfloat16:
        return TP_DTYPE_BF16
    raise TypeError(f"tropical ops take float32 or bfloat16 operands, got {t.dtype}")


def _f32(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    if t is None:
        return None
    if t.dtype != torch.float32:
        raise TypeError(f"expected a float32 tensor, got {t.dtype}")
    return t


def _batch2(t: torch.Tensor) -> Tuple[int, int, int, int]:
    """(B1, B2, s_b1, s_b2) for a tensor with 0, 1 or 2 leading batch dims."""
    lead = t.dim() - 2
    if lead == 0:
        return 1, 1, 0, 0
    if lead == 1:
        return t.shape[0], 1, t.stride(0), 0
    if lead == 2:
        return t.shape[0], t.shape[1], t.stride(0), t.stride(1)
    raise ValueError("at most two leading batch dimensions are supported")


def widen_bf16(t: torch.Tensor) -> torch.Tensor:
    """Exact bf16 -> fp32 copy of a tensor by the library's kernel."""
    dev = _require_cuda(t)
    t = t.contiguous()
    out = torch.empty(t.shape, device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        st = _lib.load().tp_convert_bf16_to_f32(t.numel(), _ptr(t), _ptr(out), _stream(dev))
    _lib.check(st, "tp_convert_bf16_to_f32")
    return out


def _widen_pays(x: torch.Tensor, w: torch.Tensor) -> bool:
    # 2-D operands big enough for the TMA kernel: widening costs < 1% there
    return (x.dim() == 2 and w.dim() == 2 and x.shape[0] >= 128 and w.shape[0] >= 128
            and x.shape[1] >= 64 and x.shape[0] * w.shape[0] >= 16 * 128 * 128)


# --------------------------------------------------------------------------- forward ops
def maxplus_strided(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None,
                    *, argmax: bool = True, scale: float = 1.0,
                    out: Optional[torch.Tensor] = None,
                    out_argmax: Optional[torch.Tensor] = None, arith: str = "f32"):
    """Batched max-plus product on strided views.

    ``x``: [..., M, K], ``w``: [..., N, K] (same 0-2 leading batch dims, any
    strides); returns ``y`` [..., M, N] fp32 and ``argmax`` [..., M, N] int32
    (or None).  ``y = (max_k(x + w) [+ bias]) * scale``.

    ``arith``: "f32" adds in fp32 (bf16 operands are widened exactly);
    "bf16" (bf16 operands only) rounds every sum to bf16 as torch does on bf16
    tensors -- the reference expression evaluated in bf16 -- and runs the
    packed bf16x2 kernel on large problems.
    """
    dev = _require_cuda(x, w, bias)
    if x.dtype != w.dtype:
        raise TypeError(f"x and w must share a dtype, got {x.dtype} and {w.dtype}")
    if arith not in ("f32", "bf16"):
        raise ValueError(f"arith must be 'f32' or 'bf16', got {arith!r}")
    code = _dtype_code(x)
    if arith == "bf16":
        if code != TP_DTYPE_BF16:
            raise TypeError("arith='bf16' needs bf16 operands")
        code = TP_DTYPE_BF16_ARITH
    elif code == TP_DTYPE_BF16 and _widen_pays(x, w):
        # large bf16 problems: widen exactly to fp32 scratch, run the fp32 TMA kernel
        x, w = widen_bf16(x), widen_bf16(w)
        code = TP_DTYPE_F32
    if x.dim() != w.dim() or x.shape[:-2] != w.shape[:-2]:
        raise ValueError(f"batch dims differ: {tuple(x.shape)} vs {tuple(w.shape)}")
    if x.shape[-1] != w.shape[-1]:
        raise ValueError(f"inner dims differ: {x.shape[-1]} vs {w.shape[-1]}")
    M, K = x.shape[-2], x.shape[-1]
    N = w.shape[-2]
    lead = tuple(x.shape[:-2])
    if bias is not None:
        bias = _f32(bias)
        if bias.shape != (N,) or not bias.is_contiguous():
            raise ValueError("bias must be a contiguous [N] float32 tensor")
    y = out if out is not None else torch.empty(lead + (M, N), device=dev, dtype=torch.float32)
    am = None
    if argmax:
        am = out_argmax if out_argmax is not None else torch.empty(
            lead + (M, N), device=dev, dtype=torch.int32)
    B1, B2, sx1, sx2 = _batch2(x)
    _, _, sw1, sw2 = _batch2(w)
    _, _, sy1, sy2 = _batch2(y)
    if am is not None:
        _, _, sa1, sa2 = _batch2(am)
        sam, san = am.stride(-2), am.stride(-1)
    else:
        sa1 = sa2 = sam = san = 0
    with torch.cuda.device(dev):
        st = _lib.load().tp_maxplus_fwd_strided(
            code, B1, B2, M, N, K,
            _ptr(x), sx1, sx2, x.stride(-2), x.stride(-1),
            _ptr(w), sw1, sw2, w.stride(-2), w.stride(-1),
            _ptr(bias),
            _ptr(y), sy1, sy2, y.stride(-2), y.stride(-1),
            _ptr(am), sa1, sa2, sam, san,
            float(scale), _stream(dev))
    _lib.check(st, "tp_maxplus_fwd_strided")
    return y, am


def maxplus(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None,
            *, argmax: bool = True, arith: str = "f32"):
    """``y[m,n] = max_k(x[m,k] + w[n,k]) (+ bias[n])`` and the lowest argmax k (int32)."""
    if x.dim() != 2 or w.dim() != 2:
        raise ValueError("maxplus takes x [M,K] and w [N,K]")
    return maxplus_strided(x, w, bias, argmax=argmax, arith=arith)


def maxplus_matmul(A: torch.Tensor, B: torch.Tensor, *, argmax: bool = False):
    """Max-plus matrix product ``C[i,j] = max_k(A[i,k] + B[k,j])`` with B stored
    [K, N] -- the layout of ``_tropical_matmul`` (benchmarks/synthetic_scheduling.py:35-38)
    and of ``maxplus_matmul_kernel`` (cuda/maxplus_gemm.cu:269-290).

    Returns C [M, N] fp32 (and the lowest maximising k as int32 when ``argmax``).
    Large products copy B once into the [N, K] layout (N*K elements against
    M*N*K terms) and run the TMA kernel; small ones read B in place through the
    strided kernel.  Values are identical either way."""
    if A.dim() != 2 or B.dim() != 2 or A.shape[1] != B.shape[0]:
        raise ValueError(f"maxplus_matmul takes A [M,K] and B [K,N], got {tuple(A.shape)} "
                         f"and {tuple(B.shape)}")
    Bt = B.t()                                     # [N, K] view, k stride N
    if _widen_pays(A, Bt) and A.dtype == torch.float32:
        Bt = Bt.contiguous()
        A = A.contiguous()
    y, am = maxplus_strided(A, Bt, argmax=argmax)
    return (y, am) if argmax else y


def maxplus_host(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None,
                 *, argmax: bool = True, out: Optional[torch.Tensor] = None,
                 out_argmax: Optional[torch.Tensor] = None, blocks: int = 4):
    """``maxplus`` on host-resident operands, results back in host memory, with the
    PCIe transfers overlapped with the computation.

    ``x`` [M,K], ``w`` [N,K] (and ``bias`` [N]) are CPU fp32 tensors, best pinned.
    Copies to the current CUDA device run on one stream, computation on the
    caller's current stream, results return on a second stream:

    * W travels in ``blocks`` row blocks (output columns), the first of them
      ahead of the first row block of x, so the first row block computes as one
      product per W block, each starting as soon as its block has landed;
    * x travels in ``blocks`` row blocks (the last one halved, so that less is
      left to return after the last product); each later block computes
      against all of W once it has landed;
    * each row block's y (and argmax) returns as soon as it is complete.

    Returns pinned host tensors (or fills ``out`` / ``out_argmax``); like any
    non-blocking copy they are complete once the current stream has been
    synchronised.  The results equal ``maxplus`` on device copies of the
    operands bit for bit."""
    if x.is_cuda or w.is_cuda or (bias is not None and bias.is_cuda):
        raise ValueError("maxplus_host takes host tensors; use maxplus for device tensors")
    if x.dim() != 2 or w.dim() != 2 or x.shape[1] != w.shape[1]:
        raise ValueError("maxplus_host takes x [M,K] and w [N,K]")
    _lib.load()  # no CPU computation: fails loudly without the CUDA library
    dev = torch.device("cuda", torch.cuda.current_device())
    M, K = x.shape
    N = w.shape[0]
    blocks = max(1, int(blocks))
    y = out if out is not None else torch.empty(M, N, pin_memory=True)
    am = None
    if argmax:
        am = out_argmax if out_argmax is not None else torch.empty(M, N, dtype=torch.int32,
                                                                   pin_memory=True)
    main = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    # device buffers belong to the caller's stream, which waits for both copy
    # streams before returning: the caching allocator reuses them only afterwards
    dx = torch.empty(M, K, device=dev)
    dw = torch.empty(N, K, device=dev)
    dy = torch.empty(M, N, device=dev)
    da = torch.empty(M, N, device=dev, dtype=torch.int32) if argmax else None
    db = torch.empty(N, device=dev) if bias is not None else None
    s_in.wait_stream(main)
    s_out.wait_stream(main)

    def spans(n, parts):
        step = max(128, -(-(-(-n // parts)) // 128) * 128)
        return [(a, min(n, a + step)) for a in range(0, n, step)]

    rows = spans(M, blocks)
    last_a, last_b = rows[-1]
    if last_b - last_a >= 256:               # halve the last row block
        mid = last_a + (((last_b - last_a) // 2 + 127) // 128) * 128
        rows[-1:] = [(last_a, mid), (mid, last_b)]
    cols = spans(N, blocks)

    ev_w, ev_x = [], []
    with torch.cuda.stream(s_in):
        for j, (c0, c1) in enumerate(cols):
            dw[c0:c1].copy_(_f32(w[c0:c1]), non_blocking=True)
            if db is not None:
                db[c0:c1].copy_(_f32(bias[c0:c1]), non_blocking=True)
            e = torch.cuda.Event()
            e.record(s_in)
            ev_w.append(e)
            if j == 0:
                a, b = rows[0]
                dx[a:b].copy_(_f32(x[a:b]), non_blocking=True)
                e = torch.cuda.Event()
                e.record(s_in)
                ev_x.append(e)
        for a, b in rows[1:]:
            dx[a:b].copy_(_f32(x[a:b]), non_blocking=True)
            e = torch.cuda.Event()
            e.record(s_in)
            ev_x.append(e)

    for i, ((a, b), e) in enumerate(zip(rows, ev_x)):
        main.wait_event(e)
        if i == 0 and len(cols) > 1:
            for (c0, c1), ew in zip(cols, ev_w):
                main.wait_event(ew)
                maxplus_strided(dx[a:b], dw[c0:c1], db[c0:c1] if db is not None else None,
                                argmax=argmax, out=dy[a:b, c0:c1],
                                out_argmax=da[a:b, c0:c1] if argmax else None)
        else:
            main.wait_event(ev_w[-1])   # all of W (in stream order before this x block)
            maxplus_strided(dx[a:b], dw, db, argmax=argmax, out=dy[a:b],
                            out_argmax=da[a:b] if argmax else None)
        done = torch.cuda.Event()
        done.record(main)
        s_out.wait_event(done)
        with torch.cuda.stream(s_out):
            y[a:b].copy_(dy[a:b], non_blocking=True)
            if argmax:
                am[a:b].copy_(da[a:b], non_blocking=True)
    main.wait_stream(s_out)
    main.wait_stream(s_in)
    return y, am


LF_MODES = {"primal": 0, "dual": 1, "blend": 2}


def maxplus_lfdual(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor],
                   mode: str, slopes: torch.Tensor, piece_bias: torch.Tensor,
                   x_grid: torch.Tensor, gate: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``lf_act(max_k(x + w) + bias)`` in one kernel (inference): the tropical
    up-projection and LFDualActivation of TropicalHybridFFN (tropformer.py:447).

    ``gate`` = sigmoid(blend_gate) [N] for mode "blend"."""
    dev = _require_cuda(x, w, bias, slopes, piece_bias, x_grid, gate)
    if x.dim() != 2 or w.dim() != 2 or x.shape[1] != w.shape[1]:
        raise ValueError("maxplus_lfdual takes x [M,K] and w [N,K]")
    if mode not in LF_MODES:
        raise ValueError(f"mode must be one of {tuple(LF_MODES)}")
    x, w = _f32(x).contiguous(), _f32(w).contiguous()
    M, K = x.shape
    N = w.shape[0]
    sl, pb, xg = (_f32(t).contiguous() for t in (slopes, piece_bias, x_grid))
    if not (sl.numel() == pb.numel() == xg.numel()):
        raise ValueError("slopes, biases and x_grid must have the same length")
    if bias is not None:
        bias = _f32(bias).contiguous()
    if mode == "blend":
        if gate is None or gate.numel() != N:
            raise ValueError("blend mode needs gate [N]")
        gate = _f32(gate).contiguous()
    y = torch.empty((M, N), device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        st = _lib.load().tp_maxplus_fwd_lfdual(
            TP_DTYPE_F32, M, N, K, _ptr(x), x.stride(0), _ptr(w), w.stride(0), _ptr(bias),
            _ptr(y), N, LF_MODES[mode], sl.numel(), _ptr(sl), _ptr(pb), _ptr(xg),
            _ptr(gate if mode == "blend" else None), _stream(dev))
    _lib.check(st, "tp_maxplus_fwd_lfdual")
    return y


def tropical_scores(Q: torch.Tensor, K: torch.Tensor, scale: float = 1.0, *, argmax: bool = True):
    """``S[..., i, j] = max_f(Q[..., i, f] + K[..., j, f]) * scale`` (+ int32 argmax f)."""
    return maxplus_strided(Q, K, None, argmax=argmax, scale=scale)


def lse_scores(Q: torch.Tensor, K: torch.Tensor, tau: float = 1.0, scale: float = 1.0,
               bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``S[..., i, j] = tau * logsumexp_f((Q[..., i, f] + K[..., j, f]) / tau) * scale``."""
    dev = _require_cuda(Q, K, bias)
    if Q.dtype != K.dtype:
        raise TypeError("Q and K must share a dtype")
    code = _dtype_code(Q)
    if Q.dim() != K.dim() or Q.shape[:-2] != K.shape[:-2] or Q.shape[-1] != K.shape[-1]:
        raise ValueError(f"shape mismatch {tuple(Q.shape)} vs {tuple(K.shape)}")
    M, Kd = Q.shape[-2], Q.shape[-1]
    N = K.shape[-2]
    lead = tuple(Q.shape[:-2])
    y = torch.empty(lead + (M, N), device=dev, dtype=torch.float32)
    B1, B2, sx1, sx2 = _batch2(Q)
    _, _, sw1, sw2 = _batch2(K)
    _, _, sy1, sy2 = _batch2(y)
    with torch.cuda.device(dev):
        st = _lib.load().tp_maxplus_lse_fwd_strided(
            code, float(tau), B1, B2, M, N, Kd,
            _ptr(Q), sx1, sx2, Q.stride(-2), Q.stride(-1),
            _ptr(K), sw1, sw2, K.stride(-2), K.stride(-1),
            _ptr(bias),
            _ptr(y), sy1, sy2, y.stride(-2), y.stride(-1),
            float(scale), _stream(dev))
    _lib.check(st, "tp_maxplus_lse_fwd_strided")
    return y


# --------------------------------------------------------------------------- backward ops
def maxplus_backward_argmax(am: torch.Tensor, gy: torch.Tensor, K: int, *,
                            need_gw: bool = True, need_gbias: bool = False,
                            scale: float = 1.0):
    """Scatter ``gy * scale`` to the argmax index: returns (gx [..,M,K], gw [..,N,K] | None,
    gbias [N] | None).  Autograd of ``scores.max(-1).values`` (tropformer.py:141)."""
    dev = _require_cuda(am, gy)
    gy = _f32(gy)
    if am.dtype != torch.int32 or am.shape != gy.shape:
        raise ValueError("argmax must be int32 with gy's shape")
    M, N = am.shape[-2], am.shape[-1]
    lead = tuple(am.shape[:-2])
    gx = torch.empty(lead + (M, K), device=dev, dtype=torch.float32)
    gw = torch.empty(lead + (N, K), device=dev, dtype=torch.float32) if need_gw else None
    gb = torch.empty((N,), device=dev, dtype=torch.float32) if need_gbias else None
    B1, B2, sa1, sa2 = _batch2(am)
    _, _, sg1, sg2 = _batch2(gy)
    _, _, sx1, sx2 = _batch2(gx)
    if gw is not None:
        _, _, sw1, sw2 = _batch2(gw)
        swn, swk = gw.stride(-2), gw.stride(-1)
    else:
        sw1 = sw2 = swn = swk = 0
    with torch.cuda.device(dev):
        st = _lib.load().tp_maxplus_bwd_argmax_strided(
            B1, B2, M, N, K,
            _ptr(am), sa1, sa2, am.stride(-2), am.stride(-1),
            _ptr(gy), sg1, sg2, gy.stride(-2), gy.stride(-1),
            _ptr(gx), sx1, sx2, gx.stride(-2), gx.stride(-1),
            _ptr(gw), sw1, sw2, swn, swk,
            _ptr(gb), float(scale), _stream(dev))
    _lib.check(st, "tp_maxplus_bwd_argmax_strided")
    return gx, gw, gb


def maxplus_backward_smooth(mode: str, tau: float, x: torch.Tensor, w: torch.Tensor,
                            gy: torch.Tensor, *, need_gw: bool = True,
                            need_gbias: bool = False, ref_max: Optional[torch.Tensor] = None):
    """STE (``tropformer.py:133-139``) or LSE/Maslov (``tropformer.py:95-97``) backward.

    ``x`` [B?, M, K], ``w`` [B?, N, K], ``gy`` [B?, M, N] (contiguous copies are made
    if needed).  Returns (gx, gw | None, gbias | None)."""
    if mode not in ("ste", "lse"):
        raise ValueError(f"smooth backward mode must be 'ste' or 'lse', got {mode!r}")
    dev = _require_cuda(x, w, gy)
    code = _dtype_code(x)
    if w.dtype != x.dtype:
        raise TypeError("x and w must share a dtype")
    gy = _f32(gy)
    squeeze = x.dim() == 2
    if squeeze:
        x, w, gy = x.unsqueeze(0), w.unsqueeze(0), gy.unsqueeze(0)
    x, w, gy = x.contiguous(), w.contiguous(), gy.contiguous()
    B, M, K = x.shape
    N = w.shape[1]
    if w.shape != (B, N, K) or gy.shape != (B, M, N):
        raise ValueError("shape mismatch in smooth backward")
    if ref_max is not None:
        ref_max = _f32(ref_max).contiguous()
        if ref_max.numel() != B * M * N:
            raise ValueError("ref_max must hold the [.., M, N] forward maxima")
    lib = _lib.load()
    ws_bytes = int(lib.tp_maxplus_bwd_smooth_workspace_bytes(B, M, N, K))
    ws = torch.empty(max(ws_bytes // 4, 4), device=dev, dtype=torch.float32)
    gx = torch.empty((B, M, K), device=dev, dtype=torch.float32)
    gw = torch.empty((B, N, K), device=dev, dtype=torch.float32) if need_gw else None
    gb = torch.empty((N,), device=dev, dtype=torch.float32) if need_gbias else None
    with torch.cuda.device(dev):
        st = lib.tp_maxplus_bwd_smooth_ref(
            TP_BWD_STE if mode == "ste" else TP_BWD_LSE, float(tau), code, B, M, N, K,
            _ptr(x), _ptr(w), _ptr(gy), _ptr(ref_max), _ptr(gx), _ptr(gw), _ptr(gb),
            _ptr(ws), ws.numel() * 4, _stream(dev))
    _lib.check(st, "tp_maxplus_bwd_smooth_ref")
    if squeeze:
        gx = gx[0]
        gw = gw[0] if gw is not None else None
    return gx, gw, gb


# --------------------------------------------------------------------------- scan
SCAN_MODES = ("auto", "sequential", "chunked")


def scan_mode(B: int, T: int, C: int, mode: str = "auto") -> str:
    """The scan evaluation for a shape: "sequential" (one warp per 32 channels
    of a batch row walks all of T) or "chunked" (time cut into chunks that run
    in parallel; same forward bits, see tp_scan_fwd_chunked).  "auto" chunks
    when the batch-row lanes give at most half a warp per SM and T is long
    (measured at T = 4096, C = 1024: chunked faster at B = 1 and 2, sequential
    at B >= 4)."""
    if mode not in SCAN_MODES:
        raise ValueError(f"scan mode must be one of {SCAN_MODES}, got {mode!r}")
    if mode != "auto":
        return mode
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    return "chunked" if (2 * B * -(-C // 32) <= sms and T >= 1024) else "sequential"


def _scan_workspace(B: int, T: int, C: int, dev, chunk: int = 0) -> torch.Tensor:
    n = _lib.load().tp_scan_chunked_workspace_bytes(B, T, C, chunk)
    if n < 0:
        raise ValueError(f"bad scan chunk length {chunk}")
    return torch.empty(max(n, 256), device=dev, dtype=torch.uint8)


def scan_forward(b: torch.Tensor, x: Optional[torch.Tensor], a: torch.Tensor,
                 h_init: float = float("-inf"), h0: Optional[torch.Tensor] = None,
                 *, need_mask: bool = False, mode: str = "auto", chunk: int = 0):
    """``h[:, t] = max(a + h[:, t-1], b[:, t] (+ x[:, t]))`` over [B, T, C] contiguous fp32.

    Returns (h, win_mask | None); win_mask is [B, ceil(T/32), C] int32 bit words.
    ``mode`` picks the evaluation (:func:`scan_mode`); both give the same bits.
    ``chunk`` (chunked mode): steps per chunk, a multiple of 32 (0: the
    library's choice)."""
    dev = _require_cuda(b, x, a, h0)
    b = _f32(b).contiguous()
    x = _f32(x).contiguous() if x is not None else None
    a = _f32(a).contiguous()
    h0 = _f32(h0).contiguous() if h0 is not None else None
    if b.dim() != 3:
        raise ValueError("scan input must be [B, T, C]")
    B, T, C = b.shape
    if x is not None and x.shape != b.shape:
        raise ValueError("b and x must have the same shape")
    if a.shape != (C,):
        raise ValueError("a must be [C]")
    if h0 is not None and h0.shape != (B, C):
        raise ValueError("h0 must be [B, C]")
    h = torch.empty_like(b)
    mask = (torch.empty((B, (T + 31) // 32, C), device=dev, dtype=torch.int32)
            if need_mask else None)
    with torch.cuda.device(dev):
        if scan_mode(B, T, C, mode) == "chunked":
            ws = _scan_workspace(B, T, C, dev, chunk)
            st = _lib.load().tp_scan_fwd_chunked(
                B, T, C, _ptr(b), _ptr(x), _ptr(a), float(h_init), _ptr(h0), _ptr(h),
                _ptr(mask), int(chunk), _ptr(ws), ws.numel(), _stream(dev))
            _lib.check(st, "tp_scan_fwd_chunked")
            return h, mask
        st = _lib.load().tp_scan_fwd(B, T, C, _ptr(b), _ptr(x), _ptr(a), float(h_init),
                                     _ptr(h0), _ptr(h), _ptr(mask), _stream(dev))
    _lib.check(st, "tp_scan_fwd")
    return h, mask


def scan_backward(gh: torch.Tensor, a: torch.Tensor, h_init: float = float("-inf"),
                  h0: Optional[torch.Tensor] = None, *, mask: Optional[torch.Tensor] = None,
                  b: Optional[torch.Tensor] = None, x: Optional[torch.Tensor] = None,
                  h: Optional[torch.Tensor] = None, need_ga: bool = True,
                  need_gh0: bool = False, mode: str = "auto", chunk: int = 0):
    """Argmax-path backward of :func:`scan_forward`: returns (gu, ga | None, gh0 | None).

    Winners come from ``mask`` when given, else are recomputed from (b, x, h).
    ``mode``/``chunk`` as in :func:`scan_forward`; in chunked mode gu and gh0
    are the same bits and ga agrees to rounding (its sum runs per chunk)."""
    dev = _require_cuda(gh, a, h0, mask, b, x, h)
    gh = _f32(gh).contiguous()
    B, T, C = gh.shape
    if mask is None and (b is None or h is None):
        raise ValueError("scan_backward needs the win mask or (b, h)")
    a = _f32(a).contiguous()
    gu = torch.empty_like(gh)
    ga = torch.empty((C,), device=dev, dtype=torch.float32) if need_ga else None
    gh0 = torch.empty((B, C), device=dev, dtype=torch.float32) if need_gh0 else None
    if scan_mode(B, T, C, mode) == "chunked":
        ws = _scan_workspace(B, T, C, dev, chunk)
        with torch.cuda.device(dev):
            st = _lib.load().tp_scan_bwd_chunked(
                B, T, C, _ptr(gh),
                _ptr(b.contiguous() if b is not None else None),
                _ptr(x.contiguous() if x is not None else None),
                _ptr(a), float(h_init), _ptr(h0.contiguous() if h0 is not None else None),
                _ptr(h.contiguous() if h is not None else None),
                _ptr(mask), _ptr(gu), _ptr(ga), _ptr(gh0), int(chunk), _ptr(ws), ws.numel(),
                _stream(dev))
        _lib.check(st, "tp_scan_bwd_chunked")
        return gu, ga, gh0
    ws = torch.empty((B, C), device=dev, dtype=torch.float32) if need_ga else None
    with torch.cuda.device(dev):
        st = _lib.load().tp_scan_bwd(
            B, T, C, _ptr(gh),
            _ptr(b.contiguous() if b is not None else None),
            _ptr(x.contiguous() if x is not None else None),
            _ptr(a), float(h_init), _ptr(h0.contiguous() if h0 is not None else None),
            _ptr(h.contiguous() if h is not None else None),
            _ptr(mask), _ptr(gu), _ptr(ga), _ptr(gh0), _ptr(ws), _stream(dev))
    _lib.check(st, "tp_scan_bwd")
    return gu, ga, gh0


# --------------------------------------------------------------------------- autograd
class MaxPlusLinearFunction(torch.autograd.Function):
    """y = max_k(x + W) + bias with a selectable backward.

    mode "argmax": eval-mode TropicalLinear (gradient to the argmax only);
    mode "ste":    train-mode TropicalLinear STE (tropformer.py:133-139);
    mode "lse":    softmax(s/tau) gradient (cuda/maxplus_gemm.cu:181-259 intent)."""

    @staticmethod
    def forward(ctx, x, weight, bias, mode: str, tau: float):
        if mode not in MODES:
            raise ValueError(f"mode must be one of {MODES}")
        ctx.mode, ctx.tau, ctx.K = mode, float(tau), x.shape[1]
        ctx.has_bias = bias is not None
        if mode == "argmax":
            y, am = maxplus(x, weight, bias, argmax=True)
            ctx.save_for_backward(am)
            return y
        # smooth modes: keep the hard max (before bias): the backward's stats
        # pass starts from it instead of sweeping K for it again
        y0, _ = maxplus(x, weight, None, argmax=False)
        ctx.save_for_backward(x, weight, y0)
        return y0 + bias if bias is not None else y0.clone()

    @staticmethod
    def backward(ctx, gy):
        need_x, need_w, need_b = ctx.needs_input_grad[0], ctx.needs_input_grad[1], ctx.has_bias
        gy = gy.contiguous()
        if ctx.mode == "argmax":
            (am,) = ctx.saved_tensors
            gx, gw, gb = maxplus_backward_argmax(am, gy, ctx.K, need_gw=need_w,
                                                 need_gbias=need_b and ctx.needs_input_grad[2])
        else:
            x, w, y0 = ctx.saved_tensors
            gx, gw, gb = maxplus_backward_smooth(ctx.mode, ctx.tau, x, w, gy, need_gw=need_w,
                                                 need_gbias=need_b and ctx.needs_input_grad[2],
                                                 ref_max=y0)
        return (gx if need_x else None), gw, gb, None, None


class TropicalScoreFunction(torch.autograd.Function):
    """Hard tropical score ``max_f(Q + K) * scale`` over [B, H, L, d] views.

    Backward routes through the argmax (``_tropical_max`` hard branch,
    tropformer.py:93-94) or, with ``smooth_tau``, through softmax(s/tau) (the
    ``_USE_SMOOTH_MAX`` STE branch, tropformer.py:95-97)."""

    @staticmethod
    def forward(ctx, Q, K, scale: float, smooth_tau: Optional[float]):
        S, am = tropical_scores(Q, K, scale, argmax=smooth_tau is None)
        ctx.scale, ctx.smooth_tau, ctx.d = float(scale), smooth_tau, Q.shape[-1]
        if smooth_tau is None:
            ctx.save_for_backward(am)
        else:
            ctx.save_for_backward(Q, K)
        return S

    @staticmethod
    def backward(ctx, gS):
        gS = gS.contiguous()
        if ctx.smooth_tau is None:
            (am,) = ctx.saved_tensors
            gQ, gK, _ = maxplus_backward_argmax(am, gS, ctx.d, need_gw=ctx.needs_input_grad[1],
                                                scale=ctx.scale)
            return gQ, gK, None, None
        Q, K = ctx.saved_tensors
        lead = Q.shape[:-2]
        Qc = Q.reshape(-1, Q.shape[-2], Q.shape[-1])
        Kc = K.reshape(-1, K.shape[-2], K.shape[-1])
        g = (gS * ctx.scale).reshape(-1, gS.shape[-2], gS.shape[-1])
        gQ, gK, _ = maxplus_backward_smooth("lse", ctx.smooth_tau, Qc, Kc, g,
                                            need_gw=ctx.needs_input_grad[1])
        gQ = gQ.reshape(*lead, Q.shape[-2], Q.shape[-1])
        gK = gK.reshape(*lead, K.shape[-2], K.shape[-1]) if gK is not None else None
        return gQ, gK, None, None


class LSEScoreFunction(torch.autograd.Function):
    """Smooth tropical score ``logsumexp_f(Q + K)`` (TSRN, research/tsrn_dml.py:438-460).

    The gradient of logsumexp is softmax over f, i.e. the LSE backward with tau = 1."""

    @staticmethod
    def forward(ctx, Q, K, tau: float):
        ctx.tau = float(tau)
        ctx.save_for_backward(Q, K)
        return lse_scores(Q, K, tau)

    @staticmethod
    def backward(ctx, gS):
        Q, K = ctx.saved_tensors
        lead = Q.shape[:-2]
        Qc = Q.reshape(-1, Q.shape[-2], Q.shape[-1])
        Kc = K.reshape(-1, K.shape[-2], K.shape[-1])
        g = gS.contiguous().reshape(-1, gS.shape[-2], gS.shape[-1])
        gQ, gK, _ = maxplus_backward_smooth("lse", ctx.tau, Qc, Kc, g,
                                            need_gw=ctx.needs_input_grad[1])
        gQ = gQ.reshape(*lead, Q.shape[-2], Q.shape[-1])
        gK = gK.reshape(*lead, K.shape[-2], K.shape[-1]) if gK is not None else None
        return gQ, gK, None


class TropicalScanFunction(torch.autograd.Function):
    """``h_t = max(a + h_{t-1}, b_t (+ x_t))``; gradients of b and x are equal."""

    @staticmethod
    def forward(ctx, b, x, a, h_init: float, h0):
        h, mask = scan_forward(b, x, a, h_init, h0, need_mask=True)
        ctx.h_init = float(h_init)
        ctx.has_x = x is not None
        ctx.save_for_backward(a, h0, mask)
        return h

    @staticmethod
    def backward(ctx, gh):
        a, h0, mask = ctx.saved_tensors
        need_ga = ctx.needs_input_grad[2]
        need_gh0 = h0 is not None and ctx.needs_input_grad[4]
        gu, ga, gh0 = scan_backward(gh, a, ctx.h_init, h0, mask=mask, need_ga=need_ga,
                                    need_gh0=need_gh0)
        gb = gu if ctx.needs_input_grad[0] else None
        gx = gu if (ctx.has_x and ctx.needs_input_grad[1]) else None
        return gb, gx, ga, None, gh0


def tropical_scan(b, x, a, h_init: float = float("-inf"), h0=None):
    """Differentiable max-plus scan (see :class:`TropicalScanFunction`)."""
    return TropicalScanFunction.apply(b, x, a, h_init, h0)


def maxplus_linear(x, weight, bias=None, mode: str = "argmax", tau: float = 1.0):
    """Differentiable tropical linear on x [..., K] (leading dims flattened)."""
    lead = x.shape[:-1]
    y = MaxPlusLinearFunction.apply(x.reshape(-1, x.shape[-1]), weight, bias, mode, tau)
    return y.reshape(*lead, weight.shape[0])


# --------------------------------------------------------------------------- probe
def probe_addmax(form: int, blocks: int, iters: int, device=None) -> Tuple[float, int]:
    """Run the register-only add+max probe once; returns (ms, terms)."""
    dev = torch.device(device) if device is not None else torch.device("cuda")
    sink = torch.empty(blocks * 256, device=dev, dtype=torch.float32)
    lib = _lib.load()
    with torch.cuda.device(dev):
        s = torch.cuda.current_stream(dev)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(s)
        st = lib.tp_probe_addmax(form, blocks, 256, iters, _ptr(sink), _stream(dev))
        end.record(s)
        end.synchronize()
    _lib.check(st, "tp_probe_addmax")
    return start.elapsed_time(end), blocks * 256 * iters * 128


# --------------------------------------------------------------------------- TSRN attention
def _tsrn_attention_into(Q, K, V, slopes, top_k: int, causal: bool, Tc: int,
                         out: torch.Tensor, dev: torch.device) -> None:
    B, H, T, dh = Q.shape
    Tkv = K.shape[2]
    lib = _lib.load()
    ws_bytes = int(lib.tp_tsrn_attention_workspace_bytes(B, H, T, Tkv, dh))
    ws = torch.empty(max(ws_bytes // 4, 4), device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        st = lib.tp_tsrn_attention_fwd(B, H, T, Tkv, int(Tc), dh, _ptr(Q), _ptr(K), _ptr(V),
                                       _ptr(slopes), int(top_k), 1 if causal else 0, _ptr(out),
                                       _ptr(ws), ws.numel() * 4, _stream(dev))
    _lib.check(st, "tp_tsrn_attention_fwd")


def _attention_shapes(Q, K, V, slopes):
    if Q.dim() != 4 or K.shape != V.shape or K.shape[:2] != Q.shape[:2] or \
            K.shape[-1] != Q.shape[-1]:
        raise ValueError(f"shapes {tuple(Q.shape)}, {tuple(K.shape)}, {tuple(V.shape)}")
    if slopes.shape != (Q.shape[1],):
        raise ValueError("slopes must be [H]")


ATTENTION_PATHS = {"auto": 0, "cuda_cores": 1, "tensor_cores": 2}


def set_attention_path(path: str) -> str:
    """Kernel of the fused TSRN attention for this process: ``"auto"`` (the
    tcgen05 kernel -- dh <= 96, top_k <= 16, any Tkv -- when T >= 128 fills its
    128-query tiles, else the CUDA-core kernel within its limits -- dh <= 128,
    top_k <= 64, Tkv <= 6144), ``"cuda_cores"`` or ``"tensor_cores"``.
    Returns the previous choice."""
    if path not in ATTENTION_PATHS:
        raise ValueError(f"path must be one of {sorted(ATTENTION_PATHS)}, got {path!r}")
    prev = ctypes.c_int(0)
    _lib.check(_lib.load().tp_tsrn_attention_set_path(ATTENTION_PATHS[path], ctypes.byref(prev)),
               "tp_tsrn_attention_set_path")
    return {v: k for k, v in ATTENTION_PATHS.items()}[prev.value]


def tsrn_attention(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, slopes: torch.Tensor,
                   top_k: int, causal: bool = True, Tc: int = 0) -> torch.Tensor:
    """Fused TSRN tropical top-k attention forward (research/tsrn_dml.py:462-548 after RoPE):
    log-sum-exp scores, ALiBi, causal mask, top-k threshold, softmax and @V in one pass.

    ``Q`` [B,H,T,dh], ``K``/``V`` [B,H,Tkv,dh] fp32 (made contiguous), ``slopes`` [H];
    the first ``Tc`` keys are cross-window cached keys.  Forward only (inference)."""
    dev = _require_cuda(Q, K, V, slopes)
    _attention_shapes(Q, K, V, slopes)
    Q, K, V = (_f32(t).contiguous() for t in (Q, K, V))
    slopes = _f32(slopes).contiguous()
    out = torch.empty_like(Q)
    _tsrn_attention_into(Q, K, V, slopes, top_k, causal, Tc, out, dev)
    return out


def split_tf32(x: torch.Tensor):
    """(hi, lo) with x = hi + lo, hi exact in TF32 (the 13 low mantissa bits of x
    cleared), lo = x - hi exact in fp32 (0 where x is not finite); one kernel."""
    dev = _require_cuda(x)
    x = _f32(x).contiguous()
    hi, lo = torch.empty_like(x), torch.empty_like(x)
    with torch.cuda.device(dev):
        st = _lib.load().tp_split_tf32(_ptr(x), x.numel(), _ptr(hi), _ptr(lo), _stream(dev))
    _lib.check(st, "tp_split_tf32")
    return hi, lo


@contextlib.contextmanager
def _tf32_matmuls():
    """TF32 tensor-core matmuls inside the block, the caller's setting restored
    after (the legacy switch, the one this library's callers use)."""
    m = torch.backends.cuda.matmul
    prev = m.allow_tf32
    m.allow_tf32 = True
    try:
        yield
    finally:
        m.allow_tf32 = prev


# rows below which a projection stays a plain fp32 GEMM (the split passes and
# three launches do not pay off)
LINEAR_TF32X3_MIN_ROWS = 4096


def _mm3(ah, al, bh, bl):
    """ah @ bh + ah @ bl + al @ bh on the TF32 tensor cores (2-D operands, any
    strides; the parts from ``split_tf32``)."""
    with _tf32_matmuls():
        y = ah @ bh
        y.addmm_(ah, bl).addmm_(al, bh)
    return y


def matmul_tf32x3(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a @ b`` (2-D fp32 CUDA tensors) at fp32 accuracy on the TF32 tensor cores:
    both split into TF32 hi and lo parts, hi.hi + hi.lo + lo.hi.  With a's
    width a multiple of 4 the two corrections are one GEMM of depth 2K on
    [ah | al] and [bl; bh] (the output read and written once for both), else
    three GEMMs."""
    K = a.shape[1]
    bh, bl = split_tf32(b)
    if K % 4 == 0:
        A = split_tf32_cat(a, 2, 2)                         # [ah | al]
        with _tf32_matmuls():
            y = A[:, :K] @ bh
            y.addmm_(A, torch.cat((bl, bh), 0))
        return y
    ah, al = split_tf32(a)
    return _mm3(ah, al, bh, bl)


def matmul_tn_tf32x3(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a.T @ b`` for row-major a [R, M] and b [R, N] (a weight gradient over R
    rows) at fp32 accuracy on the TF32 tensor cores; a is split in its own
    layout and read transposed."""
    ah, al = split_tf32(a)
    bh, bl = split_tf32(b)
    return _mm3(ah.t(), al.t(), bh, bl)


def split_tf32_cat(x: torch.Tensor, nparts: int, lo_mask: int) -> torch.Tensor:
    """The parts of ``split_tf32`` row-concatenated: x [R, C] (C a multiple of 4)
    -> [R, nparts C], part p (columns p C .. (p+1) C) the lo part where bit p of
    ``lo_mask`` is set, else the hi part; one kernel."""
    dev = _require_cuda(x)
    x = _f32(x).contiguous()
    R, C = x.shape
    out = torch.empty(R, nparts * C, device=dev)
    with torch.cuda.device(dev):
        st = _lib.load().tp_split_tf32_cat(_ptr(x), R, C, _ptr(out), int(nparts), int(lo_mask),
                                           _stream(dev))
    _lib.check(st, "tp_split_tf32_cat")
    return out


def _linear3(xh, xl, wh, wl, b):
    """hi.hi + hi.lo + lo.hi (+ b) as three cuBLAS TF32 GEMMs on split parts."""
    with _tf32_matmuls():
        y = torch.addmm(b, xh, wh.t()) if b is not None else xh @ wh.t()
        y.addmm_(xh, wl.t()).addmm_(xl, wh.t())
    return y


def _linear2cat(A, Bm, b):
    """A = [xh | xl], Bm = [wl | wh]: hi.hi (+ b) as one TF32 GEMM, then the two
    correction products as one GEMM of depth 2K accumulated onto it -- the
    output is read and written once for both (three GEMMs read and write it
    twice), and the small terms are summed apart from the large one."""
    K = A.shape[1] // 2
    xh, wh = A[:, :K], Bm[:, K:]
    with _tf32_matmuls():
        y = torch.addmm(b, xh, wh.t()) if b is not None else xh @ wh.t()
        y.addmm_(A, Bm.t())
    return y


def linear_tf32x3(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None):
    """``x @ w.T (+ b)`` at fp32 accuracy on the TF32 tensor cores: x and w are
    split into TF32 hi and lo parts (``split_tf32``) and cuBLAS TF32 GEMMs sum
    hi.hi + hi.lo + lo.hi (the lo.lo term is below 2^-22 of the product):
    ~2e-6 relative against ~1.5e-6 for fp32 SGEMM at K = 640, 3.3x faster on
    B200 at [65536 x 640] x [640 x 1920].  With K a multiple of 4 the parts
    are row-concatenated (``split_tf32_cat``) and the two correction products
    run as one GEMM of depth 2K; else three GEMMs.  (One GEMM of depth 3K for
    all three products measured ~1e-5 relative: the tensor cores' accumulation
    drops bits of the small terms beside the large one.)  A non-finite x or w
    entry gives NaN where fp32 may give +-inf.  No autograd
    (``LinearTF32x3Function`` adds it)."""
    K = x.shape[-1]
    if K % 4 == 0:
        y = _linear2cat(split_tf32_cat(x.reshape(-1, K), 2, 2), split_tf32_cat(w, 2, 1), b)
        return y.reshape(*x.shape[:-1], w.shape[0])
    xh, xl = split_tf32(x.reshape(-1, K))
    wh, wl = split_tf32(w)
    return _linear3(xh, xl, wh, wl, b).reshape(*x.shape[:-1], w.shape[0])


class LinearTF32x3Function(torch.autograd.Function):
    """``linear_tf32x3`` with its backward in the same form: dx = dy @ w and
    dw = dy^T @ x as 3xTF32 GEMMs, db = the column sums of dy.  The forward's
    split parts of x and w are kept for the backward.  With K and N multiples
    of 4 the parts are row-concatenated: the forward and dx each take a hi.hi
    GEMM and one GEMM of depth 2K / 2N for the two corrections (dw, a small
    output, three GEMMs on views of the parts)."""

    @staticmethod
    def forward(ctx, x, w, b):
        K, N = x.shape[-1], w.shape[0]
        ctx.x_shape = x.shape
        ctx.has_bias = b is not None
        ctx.cat = K % 4 == 0 and N % 4 == 0
        if ctx.cat:
            A = split_tf32_cat(x.reshape(-1, K), 2, 2)      # [xh | xl]
            Bm = split_tf32_cat(w, 2, 1)                    # [wl | wh]
            ctx.save_for_backward(A, Bm)
            return _linear2cat(A, Bm, b).reshape(*x.shape[:-1], N)
        xh, xl = split_tf32(x.reshape(-1, K))
        wh, wl = split_tf32(w)
        ctx.save_for_backward(xh, xl, wh, wl)
        return _linear3(xh, xl, wh, wl, b).reshape(*x.shape[:-1], N)

    @staticmethod
    def backward(ctx, dy):
        K = ctx.x_shape[-1]
        dx = dw = db = None
        if ctx.cat:
            A, Bm = ctx.saved_tensors
            N = Bm.shape[0]
            xh, xl, wl, wh = A[:, :K], A[:, K:], Bm[:, :K], Bm[:, K:]
            G = split_tf32_cat(dy.reshape(-1, N), 2, 2)     # [gh | gl]
            gh, gl = G[:, :N], G[:, N:]
            if ctx.needs_input_grad[0]:
                Bw = torch.cat((wl, wh), 0)                  # [wl; wh]: gh.wl + gl.wh
                with _tf32_matmuls():
                    dx = gh @ wh
                    dx.addmm_(G, Bw)
                dx = dx.reshape(ctx.x_shape)
            if ctx.needs_input_grad[1]:
                dw = _mm3(gh.t(), gl.t(), xh, xl)
        else:
            xh, xl, wh, wl = ctx.saved_tensors
            N = wh.shape[0]
            gh, gl = split_tf32(dy.reshape(-1, N))
            if ctx.needs_input_grad[0]:
                dx = _mm3(gh, gl, wh, wl).reshape(ctx.x_shape)
            if ctx.needs_input_grad[1]:
                dw = _mm3(gh.t(), gl.t(), xh, xl)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            db = dy.reshape(-1, N).sum(0)
        return dx, dw, db


def linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None):
    """``F.linear`` of the drop-in modules: fp32-accurate 3xTF32 tensor-core GEMMs
    (``linear_tf32x3``; with autograd ``LinearTF32x3Function``) for CUDA fp32
    inputs of at least LINEAR_TF32X3_MIN_ROWS rows, the plain fp32 GEMM
    otherwise."""
    rows = x.numel() // max(x.shape[-1], 1)
    if rows < LINEAR_TF32X3_MIN_ROWS or not x.is_cuda or x.dtype != torch.float32 or \
            w.dtype != torch.float32:
        return torch.nn.functional.linear(x, w, b)
    try:
        torch.backends.cuda.matmul.allow_tf32
    except RuntimeError:     # the caller set TF32 through the newer API: keep fp32 GEMMs
        return torch.nn.functional.linear(x, w, b)
    needs_grad = torch.is_grad_enabled() and (
        x.requires_grad or w.requires_grad or (b is not None and b.requires_grad))
    if needs_grad:
        return LinearTF32x3Function.apply(x, w, b)
    return linear_tf32x3(x, w.detach(), None if b is None else b.detach())


def tsrn_attention_supports_lists(dh: int, top_k: int, Tkv: int = 0) -> bool:
    """Whether ``tsrn_attention_train_fwd`` (the tensor-core kernel) and the sparse
    backward (whose grouping kernel holds 3 words per key in shared memory) take
    this shape."""
    return 1 <= dh <= 96 and 1 <= top_k <= 16 and Tkv <= 16384


def tsrn_attention_train_fwd(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor,
                             slopes: torch.Tensor, top_k: int, causal: bool = True, Tc: int = 0):
    """``tsrn_attention`` on the tensor-core kernel, also returning what the sparse
    backward needs: per query row its kept keys [B*H*T, 32] (int32, -1 past the
    row's entries), their softmax weights and log-sum-exp scores before ALiBi
    (both [B*H*T, 32]) and the count [B*H*T] (-1 when ties kept more keys than
    the lists hold).  Returns (out, keys, weights, lse, count).  dh <= 96,
    top_k <= 16."""
    dev = _require_cuda(Q, K, V, slopes)
    _attention_shapes(Q, K, V, slopes)
    Q, K, V = (_f32(t).contiguous() for t in (Q, K, V))
    slopes = _f32(slopes).contiguous()
    B, H, T, dh = Q.shape
    Tkv = K.shape[2]
    out = torch.empty_like(Q)
    rows = B * H * T
    kj = torch.empty(rows, _lib.TP_ATT_LIST, device=dev, dtype=torch.int32)
    kp = torch.empty(rows, _lib.TP_ATT_LIST, device=dev, dtype=torch.float32)
    kl = torch.empty(rows, _lib.TP_ATT_LIST, device=dev, dtype=torch.float32)
    kn = torch.empty(rows, device=dev, dtype=torch.int32)
    lib = _lib.load()
    ws_bytes = int(lib.tp_tsrn_attention_workspace_bytes(B, H, T, Tkv, dh))
    ws = torch.empty(max(ws_bytes // 4, 4), device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        st = lib.tp_tsrn_attention_fwd_lists(B, H, T, Tkv, int(Tc), dh, _ptr(Q), _ptr(K), _ptr(V),
                                             _ptr(slopes), int(top_k), 1 if causal else 0,
                                             _ptr(out), _ptr(kj), _ptr(kp), _ptr(kl), _ptr(kn),
                                             _ptr(ws), ws.numel() * 4, _stream(dev))
    _lib.check(st, "tp_tsrn_attention_fwd_lists")
    return out, kj, kp, kl, kn


def tsrn_attention_sparse_bwd(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor,
                              dO: torch.Tensor, kj: torch.Tensor, kp: torch.Tensor,
                              kl: torch.Tensor, kn: torch.Tensor):
    """Gradients (dQ, dK, dV) of the fused attention from the kept-key lists of
    ``tsrn_attention_train_fwd`` (every kn >= 0): the backward of
    research/tsrn_dml.py:438-460, :509-524 with the top-k threshold detached.
    Three kernels (rows: dQ; group: a stable counting sort of the entries by
    key; keys: dK, dV): every gradient is summed in a fixed order."""
    dev = _require_cuda(Q, K, V, dO, kj, kp, kl, kn)
    Q, K, V, dO = (_f32(t).contiguous() for t in (Q, K, V, dO))
    B, H, T, dh = Q.shape
    Tkv = K.shape[2]
    S, L = B * H, _lib.TP_ATT_LIST
    dQ = torch.empty_like(Q)
    dK = torch.empty_like(K)
    dV = torch.empty_like(V)
    eds = torch.empty(S * T, L, device=dev, dtype=torch.float32)
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = lib.tp_tsrn_attention_bwd_rows(S, T, Tkv, dh, _ptr(Q), _ptr(K), _ptr(V), _ptr(dO),
                                            _ptr(kj), _ptr(kp), _ptr(kl), _ptr(kn), _ptr(dQ),
                                            _ptr(eds), _stream(dev))
        _lib.check(st, "tp_tsrn_attention_bwd_rows")
        # entries grouped by key (slice * Tkv + j), rows ascending inside a key
        order = torch.empty(S * T * L, device=dev, dtype=torch.int32)
        key_begin = torch.empty(S * Tkv, device=dev, dtype=torch.int32)
        key_count = torch.empty(S * Tkv, device=dev, dtype=torch.int32)
        st = lib.tp_tsrn_attention_bwd_group(S, T, Tkv, _ptr(kj), _ptr(order), _ptr(key_begin),
                                             _ptr(key_count), _stream(dev))
        _lib.check(st, "tp_tsrn_attention_bwd_group")
        st = lib.tp_tsrn_attention_bwd_keys(S, T, Tkv, dh, _ptr(Q), _ptr(K), _ptr(dO), _ptr(kp),
                                            _ptr(kl), _ptr(eds), _ptr(order), _ptr(key_begin),
                                            _ptr(key_count), _ptr(dK), _ptr(dV), _stream(dev))
        _lib.check(st, "tp_tsrn_attention_bwd_keys")
    return dQ, dK, dV


def tsrn_attention_prologue(qkv: torch.Tensor, B: int, T: int, H: int, dh: int,
                            q_norm: torch.nn.LayerNorm, k_norm: torch.nn.LayerNorm,
                            cos: torch.Tensor, sin: torch.Tensor, pos0: int = 0):
    """Q, K, V [B, H, T, dh] from the stacked projections ``qkv`` [B*T, 3*H*dh]
    (Q | K | V columns): per-head LayerNorm (``q_norm`` / ``k_norm``) and the
    rotary embedding of positions pos0..pos0+T-1 (tables ``cos``/``sin``
    [positions, dh/2]) on Q and K, head-major layout for all three -- the
    prologue of research/tsrn_dml.py:472-477 in one kernel (inference)."""
    dev = _require_cuda(qkv, cos, sin)

    def affine(ln):
        if ln.weight is None:
            return torch.ones(dh, device=dev), torch.zeros(dh, device=dev)
        return _f32(ln.weight.detach()).contiguous(), _f32(ln.bias.detach()).contiguous()

    qg, qb = affine(q_norm)
    kg, kb = affine(k_norm)
    if q_norm.eps != k_norm.eps:
        raise ValueError("q_norm and k_norm must share eps")
    return tsrn_attention_prologue_raw(qkv, B, T, H, dh, qg, qb, kg, kb, float(q_norm.eps),
                                       cos, sin, pos0)


def _prologue_checks(qkv, B, T, H, dh, cos, sin):
    d = H * dh
    if qkv.dim() != 2 or qkv.shape[0] != B * T or qkv.shape[1] < 3 * d or qkv.stride(1) != 1:
        raise ValueError(f"qkv must be [B*T, >= 3*H*dh] with unit column stride, "
                         f"got {tuple(qkv.shape)}")
    if cos.shape != sin.shape or cos.dim() != 2 or cos.shape[1] * 2 != dh:
        raise ValueError("cos / sin tables must be [positions, dh/2]")


def tsrn_attention_prologue_raw(qkv: torch.Tensor, B: int, T: int, H: int, dh: int,
                                qg: torch.Tensor, qb: torch.Tensor, kg: torch.Tensor,
                                kb: torch.Tensor, eps: float, cos: torch.Tensor,
                                sin: torch.Tensor, pos0: int = 0):
    """``tsrn_attention_prologue`` with the LayerNorm parameters as tensors."""
    dev = _require_cuda(qkv, qg, qb, kg, kb, cos, sin)
    qkv = _f32(qkv)
    _prologue_checks(qkv, B, T, H, dh, cos, sin)
    d = H * dh
    qg, qb, kg, kb = (_f32(t.detach()).contiguous() for t in (qg, qb, kg, kb))
    cos, sin = _f32(cos).contiguous(), _f32(sin).contiguous()
    Q, K, V = (torch.empty(B, H, T, dh, device=dev) for _ in range(3))
    with torch.cuda.device(dev):
        st = _lib.load().tp_tsrn_attention_prologue(
            B, T, H, dh, _ptr(qkv), qkv.stride(0), d, 2 * d, _ptr(qg), _ptr(qb), _ptr(kg),
            _ptr(kb), float(eps), _ptr(cos), _ptr(sin), cos.shape[0], int(pos0),
            _ptr(Q), _ptr(K), _ptr(V), _stream(dev))
    _lib.check(st, "tp_tsrn_attention_prologue")
    return Q, K, V


def tsrn_attention_prologue_bwd(qkv: torch.Tensor, B: int, T: int, H: int, dh: int,
                                qg: torch.Tensor, kg: torch.Tensor, eps: float,
                                cos: torch.Tensor, sin: torch.Tensor, dQ: torch.Tensor,
                                dK: torch.Tensor, dV: torch.Tensor, pos0: int = 0):
    """Backward of ``tsrn_attention_prologue_raw``: (dqkv [B*T, 3*H*dh], dq_gamma,
    dq_beta, dk_gamma, dk_beta) from the gradients of Q, K, V; one kernel over the
    rows plus an ordered sum of the parameter gradients (deterministic)."""
    dev = _require_cuda(qkv, qg, kg, cos, sin, dQ, dK, dV)
    qkv = _f32(qkv)
    _prologue_checks(qkv, B, T, H, dh, cos, sin)
    d = H * dh
    qg, kg = (_f32(t.detach()).contiguous() for t in (qg, kg))
    cos, sin = _f32(cos).contiguous(), _f32(sin).contiguous()
    dQ, dK, dV = (_f32(t).contiguous() for t in (dQ, dK, dV))
    dqkv = torch.zeros(B * T, qkv.shape[1], device=dev) if qkv.shape[1] != 3 * d else \
        torch.empty(B * T, 3 * d, device=dev)
    dp = torch.empty(4, dh, device=dev)
    lib = _lib.load()
    ws_bytes = int(lib.tp_tsrn_attention_prologue_bwd_workspace_bytes(B, T, H, dh))
    ws = torch.empty(max(ws_bytes // 4, 4), device=dev)
    with torch.cuda.device(dev):
        st = lib.tp_tsrn_attention_prologue_bwd(
            B, T, H, dh, _ptr(qkv), qkv.stride(0), d, 2 * d, _ptr(qg), _ptr(kg), float(eps),
            _ptr(cos), _ptr(sin), cos.shape[0], int(pos0), _ptr(dQ), _ptr(dK), _ptr(dV),
            _ptr(dqkv), _ptr(dp), _ptr(ws), ws.numel() * 4, _stream(dev))
    _lib.check(st, "tp_tsrn_attention_prologue_bwd")
    return dqkv, dp[0], dp[1], dp[2], dp[3]


def layer_norm_supported(D: int) -> bool:
    """Whether :func:`layer_norm_bwd` takes rows of ``D`` channels (a multiple of
    128, at most 1024)."""
    return 128 <= D <= 1024 and D % 128 == 0


def layer_norm_bwd(x: torch.Tensor, dy: torch.Tensor, weight: Optional[torch.Tensor],
                   eps: float):
    """Backward of ``F.layer_norm(x, (D,), weight, bias, eps)`` over the last
    dimension: (dx, dweight, dbias), one pass over x and dy with the row
    statistics recomputed; the parameter gradients are summed per block and then
    over blocks in a fixed order (the same bits on every call).  The pre-norms of
    the TSRN block's branches (research/tsrn_dml.py:1096-1106) in training."""
    dev = _require_cuda(x, dy, weight)
    D = x.shape[-1]
    if not layer_norm_supported(D):
        raise ValueError(f"layer_norm_bwd takes D a multiple of 128 up to 1024, got {D}")
    x2 = _f32(x).reshape(-1, D).contiguous()
    dy2 = _f32(dy).reshape(-1, D).contiguous()
    rows = x2.shape[0]
    w = _f32(weight.detach()).contiguous() if weight is not None else None
    dx = torch.empty_like(x2)
    dw = torch.empty(D, device=dev)
    db = torch.empty(D, device=dev)
    lib = _lib.load()
    ws_bytes = int(lib.tp_layernorm_bwd_workspace_bytes(rows, D))
    ws = torch.empty(max(ws_bytes // 4, 4), device=dev)
    with torch.cuda.device(dev):
        st = lib.tp_layernorm_bwd(rows, D, _ptr(x2), _ptr(dy2), _ptr(w), float(eps), _ptr(dx),
                                  _ptr(dw), _ptr(db), _ptr(ws), ws.numel() * 4, _stream(dev))
    _lib.check(st, "tp_layernorm_bwd")
    return dx.reshape(x.shape), dw, db


class LayerNormFunction(torch.autograd.Function):
    """LayerNorm over the last dimension: PyTorch's forward kernel, the backward
    of :func:`layer_norm_bwd`."""

    @staticmethod
    def forward(ctx, x, weight, bias, eps: float):
        ctx.save_for_backward(x, weight)
        ctx.eps = eps
        ctx.has_bias = bias is not None
        return torch.nn.functional.layer_norm(x, (x.shape[-1],), weight, bias, eps)

    @staticmethod
    def backward(ctx, dy):
        x, weight = ctx.saved_tensors
        dx, dw, db = layer_norm_bwd(x, dy, weight, ctx.eps)
        return (dx, dw if weight is not None else None, db if ctx.has_bias else None, None)


def layer_norm(x: torch.Tensor, weight: Optional[torch.Tensor], bias: Optional[torch.Tensor],
               eps: float = 1e-5) -> torch.Tensor:
    """``F.layer_norm`` over the last dimension with the backward of
    :func:`layer_norm_bwd` when autograd records on a supported CUDA fp32 shape
    (else PyTorch's own)."""
    needs = torch.is_grad_enabled() and (x.requires_grad or (
        weight is not None and weight.requires_grad) or (bias is not None and bias.requires_grad))
    if (needs and x.is_cuda and x.dtype == torch.float32 and layer_norm_supported(x.shape[-1])
            and (weight is None or weight.dtype == torch.float32)):
        return LayerNormFunction.apply(x, weight, bias, float(eps))
    return torch.nn.functional.layer_norm(x, (x.shape[-1],), weight, bias, eps)


def tsrn_attention_host(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor,
                        slopes: torch.Tensor, top_k: int, causal: bool = True, Tc: int = 0, *,
                        out: Optional[torch.Tensor] = None, chunks: int = 16) -> torch.Tensor:
    """``tsrn_attention`` on host-resident Q, K, V (CPU fp32, best pinned), result
    in host memory, the PCIe transfers overlapped with the computation: the
    batch runs in ``chunks`` groups of sequences; group i+1's inputs travel on
    one copy stream while group i computes on the caller's current stream and
    group i-1's output returns on a second copy stream.

    Returns a pinned host tensor (or fills ``out``); like any non-blocking copy
    it is complete once the current stream has been synchronised.  Equals
    ``tsrn_attention`` on device copies of the inputs bit for bit."""
    if Q.is_cuda or K.is_cuda or V.is_cuda:
        raise ValueError("tsrn_attention_host takes host Q, K, V; use tsrn_attention on device")
    _attention_shapes(Q, K, V, slopes)
    _lib.load()  # no CPU computation: fails loudly without the CUDA library
    dev = torch.device("cuda", torch.cuda.current_device())
    B = Q.shape[0]
    host_out = out if out is not None else torch.empty(Q.shape, pin_memory=True)
    main = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    dQ, dK, dV = (torch.empty(t.shape, device=dev) for t in (Q, K, V))
    dO = torch.empty(Q.shape, device=dev)
    sl = _f32(slopes).to(dev).contiguous()
    s_in.wait_stream(main)
    s_out.wait_stream(main)
    step = max(1, -(-B // max(1, int(chunks))))
    groups = [(a, min(B, a + step)) for a in range(0, B, step)]
    landed = []
    with torch.cuda.stream(s_in):
        for a, b in groups:
            for d, h in ((dQ, Q), (dK, K), (dV, V)):
                d[a:b].copy_(_f32(h[a:b]), non_blocking=True)
            e = torch.cuda.Event()
            e.record(s_in)
            landed.append(e)
    for (a, b), e in zip(groups, landed):
        main.wait_event(e)
        _tsrn_attention_into(dQ[a:b], dK[a:b], dV[a:b], sl, top_k, causal, Tc, dO[a:b], dev)
        done = torch.cuda.Event()
        done.record(main)
        s_out.wait_event(done)
        with torch.cuda.stream(s_out):
            host_out[a:b].copy_(dO[a:b], non_blocking=True)
    main.wait_stream(s_out)
    main.wait_stream(s_in)
    return host_out


# --------------------------------------------------------------------------- reservoir
def _rows(w: torch.Tensor, dr: int) -> Tuple[torch.Tensor, int]:
    """fp32 [dr, dr] weight view with unit column stride; returns (tensor, row stride)."""
    w = _f32(w)
    if w.shape != (dr, dr):
        raise ValueError(f"reservoir weight of shape {tuple(w.shape)}, expected ({dr}, {dr})")
    if w.stride(1) != 1 or w.stride(0) < dr:
        w = w.contiguous()
    return w, w.stride(0)


def _h0(h0: Optional[torch.Tensor], B: int, dr: int):
    if h0 is None:
        return None, 0
    if h0.shape != (B, dr):
        raise ValueError(f"h0 must be [B, dr] = {(B, dr)}, got {tuple(h0.shape)}")
    h0 = _f32(h0)
    if h0.stride(1) != 1:
        h0 = h0.contiguous()
    return h0, h0.stride(0)


def _esn_call(gru: bool, U, Uz, Ur, W, lk, h0, H, T: int, t_stride: int, dev) -> None:
    """One segmented launch: T steps of the [B, t_stride, dr] tensors U (Uz, Ur)
    and H starting at their base pointers (views), from state h0."""
    B, dr = U.shape[0], U.shape[2]
    lib = _lib.load()
    h0, ldh = _h0(h0, B, dr)
    with torch.cuda.device(dev):
        if gru:
            (Wzh, lz), (Wrh, lr), (Ws, ls) = W
            st = lib.tp_esn_gru_fwd_seg(B, T, t_stride, dr, _ptr(U), _ptr(Uz), _ptr(Ur),
                                        _ptr(Wzh), lz, _ptr(Wrh), lr, _ptr(Ws), ls, _ptr(h0),
                                        ldh, _ptr(H), _stream(dev))
        else:
            (Ws, ls), = W
            st = lib.tp_esn_leaky_fwd_seg(B, T, t_stride, dr, _ptr(U), _ptr(Ws), ls, _ptr(lk),
                                          _ptr(h0), ldh, _ptr(H), _stream(dev))
    _lib.check(st, "tp_esn_gru_fwd_seg" if gru else "tp_esn_leaky_fwd_seg")


def esn_gru_fwd(U: torch.Tensor, Uz: torch.Tensor, Ur: torch.Tensor, Wzh: torch.Tensor,
                Wrh: torch.Tensor, Ws: torch.Tensor,
                h0: Optional[torch.Tensor] = None) -> torch.Tensor:
    """GRU-gated echo-state recurrence over all T steps in one launch
    (research/tsrn_dml.py:834-840); returns H [B, T, dr].  Forward only.
    Wzh / Wrh may be the column slices ``W_z.weight[:, :dr]`` in place.
    ``h0`` [B, dr] continues a sequence from that state (default zeros, as the
    reference module starts)."""
    dev = _require_cuda(U, Uz, Ur, Wzh, Wrh, Ws, h0)
    U, Uz, Ur = (_f32(t).contiguous() for t in (U, Uz, Ur))
    B, T, dr = U.shape
    if Uz.shape != U.shape or Ur.shape != U.shape:
        raise ValueError("esn_gru_fwd: U, Uz and Ur must have the same shape")
    W = [_rows(w, dr) for w in (Wzh, Wrh, Ws)]
    H = torch.empty_like(U)
    _esn_call(True, U, Uz, Ur, W, None, h0, H, T, T, dev)
    return H


def esn_leaky_fwd(U: torch.Tensor, Ws: torch.Tensor, lk: torch.Tensor,
                  h0: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Leaky echo-state recurrence h = (1 - lk) h + lk tanh(h Ws^T + U_t) over
    all T steps in one launch (tsrn_gpu.py:480-484); ``lk`` is the device
    scalar sigmoid(leak).  Returns H [B, T, dr].  Forward only.  ``h0`` [B, dr]
    continues a sequence from that state (default zeros)."""
    dev = _require_cuda(U, Ws, lk, h0)
    U = _f32(U).contiguous()
    B, T, dr = U.shape
    lk = _f32(lk).reshape(1).contiguous()
    H = torch.empty_like(U)
    _esn_call(False, U, None, None, [_rows(Ws, dr)], lk, h0, H, T, T, dev)
    return H


def esn_gru_bwd(dH: torch.Tensor, fa: torch.Tensor, fz: torch.Tensor, fr: torch.Tensor,
                keep: torch.Tensor, r: torch.Tensor, Wzh: torch.Tensor, Wrh: torch.Tensor,
                Ws: torch.Tensor):
    """Backward through time of the GRU-gated recurrence in one launch: the
    reverse-time loop of the reference's autograd over research/tsrn_dml.py:834-840.
    dH and the per-step factors fa, fz, fr, keep, r are [B, T, dr] (see
    ``reservoir.GRUReservoirFunction``); returns (dAh, dAz, dAr), the gradients
    of the candidate's and both gates' pre-activations at every step."""
    dev = _require_cuda(dH, fa, fz, fr, keep, r, Wzh, Wrh, Ws)
    dH, fa, fz, fr, keep, r = (_f32(t).contiguous() for t in (dH, fa, fz, fr, keep, r))
    B, T, dr = dH.shape
    for t in (fa, fz, fr, keep, r):
        if t.shape != dH.shape:
            raise ValueError("esn_gru_bwd: every factor must have dH's shape [B, T, dr]")
    WT = [_rows(w.t().contiguous(), dr) for w in (Wzh, Wrh, Ws)]
    out = [torch.empty_like(dH) for _ in range(3)]
    with torch.cuda.device(dev):
        st = _lib.load().tp_esn_gru_bwd(B, T, dr, _ptr(dH), _ptr(fa), _ptr(fz), _ptr(fr),
                                         _ptr(keep), _ptr(r), _ptr(WT[0][0]), WT[0][1],
                                         _ptr(WT[1][0]), WT[1][1], _ptr(WT[2][0]), WT[2][1],
                                         _ptr(out[0]), _ptr(out[1]), _ptr(out[2]), _stream(dev))
    _lib.check(st, "tp_esn_gru_bwd")
    return tuple(out)


def esn_leaky_bwd(dH: torch.Tensor, fa: torch.Tensor, Ws: torch.Tensor, lk: torch.Tensor):
    """Backward through time of the leaky recurrence in one launch (the reverse
    loop of autograd over tsrn_gpu.py:480-484): dH and fa = lk (1 - s^2) are
    [B, T, dr], ``lk`` the device scalar.  Returns (dA, dHs): the gradient of
    each step's pre-activation and of each step's state h_t."""
    dev = _require_cuda(dH, fa, Ws, lk)
    dH, fa = (_f32(t).contiguous() for t in (dH, fa))
    B, T, dr = dH.shape
    if fa.shape != dH.shape:
        raise ValueError("esn_leaky_bwd: fa must have dH's shape [B, T, dr]")
    lk = _f32(lk).reshape(1).contiguous()
    WsT, ld = _rows(Ws.t().contiguous(), dr)
    dA, dHs = torch.empty_like(dH), torch.empty_like(dH)
    with torch.cuda.device(dev):
        st = _lib.load().tp_esn_leaky_bwd(B, T, dr, _ptr(dH), _ptr(fa), _ptr(WsT), ld, _ptr(lk),
                                           _ptr(dA), _ptr(dHs), _stream(dev))
    _lib.check(st, "tp_esn_leaky_bwd")
    return dA, dHs


def _copy_rows(dst: torch.Tensor, src: torch.Tensor, stream) -> None:
    """dst[b] <- src[b] for every row b of two [B, ...] views whose rows are
    contiguous runs (time windows of [B, T, dr] tensors): one 2-D copy."""
    B = src.shape[0]
    width = src[0].numel() * src.element_size()
    st = _lib.load().tp_memcpy2d_async(_ptr(dst), dst.stride(0) * dst.element_size(), _ptr(src),
                                       src.stride(0) * src.element_size(), width, B,
                                       ctypes.c_void_p(stream.cuda_stream))
    _lib.check(st, "tp_memcpy2d_async")


def esn_fwd_host(U: torch.Tensor, Ws: torch.Tensor, *, Uz: Optional[torch.Tensor] = None,
                 Ur: Optional[torch.Tensor] = None, Wzh: Optional[torch.Tensor] = None,
                 Wrh: Optional[torch.Tensor] = None, lk: Optional[torch.Tensor] = None,
                 out: Optional[torch.Tensor] = None, segments: int = 4) -> torch.Tensor:
    """Reservoir recurrence on host-resident inputs (CPU fp32 [B, T, dr], best
    pinned), H returned in host memory, PCIe transfers overlapped with the
    recurrence: the sequence runs in ``segments`` time windows, each continuing
    from the previous window's last state on the device; window i+1's inputs
    travel on one copy stream while window i runs on the caller's current
    stream and window i-1's states return on a second copy stream.  GRU-gated
    (tsrn_dml.py) when ``Uz``, ``Ur``, ``Wzh``, ``Wrh`` are given, else leaky
    (tsrn_gpu.py) with the device scalar ``lk``.  Weights are device tensors;
    ``Uz`` / ``Ur`` may be device tensors too (computed on the device from U,
    as the module does), which are then read in place.

    Returns a pinned host tensor (or fills ``out``); complete once the current
    stream has been synchronised.  Equals ``esn_gru_fwd`` / ``esn_leaky_fwd``
    on device copies bit for bit."""
    gru = Uz is not None
    if U.is_cuda:
        raise ValueError("esn_fwd_host takes host U; use esn_*_fwd on device")
    if gru and (Ur is None or Wzh is None or Wrh is None):
        raise ValueError("the GRU recurrence needs Uz, Ur, Wzh and Wrh")
    if not gru and lk is None:
        raise ValueError("the leaky recurrence needs lk")
    dev = _require_cuda(Ws, Wzh, Wrh, lk)
    ins = [U] + ([Uz, Ur] if gru else [])
    B, T, dr = U.shape
    for t in ins:
        if t.shape != (B, T, dr) or t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("U (Uz, Ur) must be contiguous fp32 [B, T, dr] tensors")
        if t.is_cuda and t.device != dev:
            raise RuntimeError(f"{t.device} input with weights on {dev}")
    W = [_rows(w, dr) for w in ((Wzh, Wrh, Ws) if gru else (Ws,))]
    lkd = _f32(lk).reshape(1).contiguous() if lk is not None else None
    host_H = out if out is not None else torch.empty((B, T, dr), pin_memory=True)
    main = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    dev_in = [t if t.is_cuda else torch.empty((B, T, dr), device=dev) for t in ins]
    dH = torch.empty((B, T, dr), device=dev)
    s_in.wait_stream(main)
    s_out.wait_stream(main)
    step = max(1, -(-T // max(1, int(segments))))
    wins = [(a, min(T, a + step)) for a in range(0, T, step)]
    landed = []
    for a, b in wins:
        for d, h in zip(dev_in, ins):
            if not h.is_cuda:
                _copy_rows(d[:, a:b], h[:, a:b], s_in)
        e = torch.cuda.Event()
        e.record(s_in)
        landed.append(e)
    for (a, b), e in zip(wins, landed):
        main.wait_event(e)
        h0 = dH[:, a - 1] if a > 0 else None
        _esn_call(gru, dev_in[0][:, a:], dev_in[1][:, a:] if gru else None,
                  dev_in[2][:, a:] if gru else None, W, lkd, h0, dH[:, a:], b - a, T, dev)
        done = torch.cuda.Event()
        done.record(main)
        s_out.wait_event(done)
        _copy_rows(host_H[:, a:b], dH[:, a:b], s_out)
    main.wait_stream(s_out)
    main.wait_stream(s_in)
    return host_H


def _maslov_inputs(T, C, g, tau, mask):
    """Contiguous fp32 scores, gate [B, Lq, H] and temperatures [H]; the mask
    as bytes (True where the module's ``mask == 0``) broadcast to [B, H, Lq, Lk]."""
    dev = _require_cuda(T, C, g, tau)
    if T.dim() != 4:
        raise ValueError("scores must be [B, H, Lq, Lk]")
    B, H, Lq, Lk = T.shape
    T = _f32(T).contiguous()
    if (C is None) != (g is None):
        raise ValueError("the classical scores and the gate come together")
    if C is not None:
        if C.shape != T.shape:
            raise ValueError(f"classical scores {tuple(C.shape)} != {tuple(T.shape)}")
        if g.shape != (B, Lq, H):
            raise ValueError(f"gate must be [B, Lq, H] = {(B, Lq, H)}, got {tuple(g.shape)}")
        C, g = _f32(C).contiguous(), _f32(g).contiguous()
    if tau.shape != (H,):
        raise ValueError(f"tau must be [H] = ({H},), got {tuple(tau.shape)}")
    tau = _f32(tau).detach().contiguous()
    m, ms = None, (0, 0, 0, 0)
    if mask is not None:
        if mask.device != dev:
            raise RuntimeError(f"mask on {mask.device}, scores on {dev}")
        m = torch.broadcast_to(mask == 0, (B, H, Lq, Lk))
        ms = tuple(m.stride())
    return dev, (B, H, Lq, Lk), T, C, g, tau, m, ms


def _gate_strides(g):
    return (0, 0, 0) if g is None else tuple(g.stride())


def maslov_softmax_fwd(T, C, g, tau, mask=None) -> torch.Tensor:
    """softmax((g*T + (1-g)*C masked to -1e9 where mask == 0) / tau_h) over the
    last dim (without C and g: softmax(T / tau_h)) -- DTNAttention's score blend
    and MaslovTemperature (deep_tropical_net.py:152-160, tropformer.py:206-212)."""
    dev, (B, H, Lq, Lk), T, C, g, tau, m, ms = _maslov_inputs(T, C, g, tau, mask)
    P = torch.empty_like(T)
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = lib.tp_maslov_softmax_fwd(B, H, Lq, Lk, _ptr(T), _ptr(C), _ptr(g), *_gate_strides(g),
                                       _ptr(m), *ms, _ptr(tau), _ptr(P), _stream(dev))
    _lib.check(st, "tp_maslov_softmax_fwd")
    return P


class MaslovSoftmaxFunction(torch.autograd.Function):
    """Autograd of the (gated) Maslov softmax: gradients for the tropical and
    classical scores, the gate and the temperatures, as PyTorch's autograd of
    the module expression forms them (deep_tropical_net.py:152-160)."""

    @staticmethod
    def forward(ctx, T, C, g, tau, mask):
        dev, shape, Tc, Cc, gc, tc, m, ms = _maslov_inputs(T, C, g, tau, mask)
        P = torch.empty_like(Tc)
        lib = _lib.load()
        with torch.cuda.device(dev):
            st = lib.tp_maslov_softmax_fwd(*shape, _ptr(Tc), _ptr(Cc), _ptr(gc),
                                           *_gate_strides(gc), _ptr(m), *ms, _ptr(tc), _ptr(P),
                                           _stream(dev))
        _lib.check(st, "tp_maslov_softmax_fwd")
        ctx.save_for_backward(Tc, Cc, gc, tc, P)
        ctx.mask = (m, ms)
        ctx.shape = shape
        return P

    @staticmethod
    def backward(ctx, dP):
        T, C, g, tau, P = ctx.saved_tensors
        m, ms = ctx.mask
        B, H, Lq, Lk = ctx.shape
        need_T, need_C, need_g, need_tau = ctx.needs_input_grad[:4]
        dev = T.device
        dP = _f32(dP).contiguous()
        dT = torch.empty_like(T) if need_T else None
        dC = torch.empty_like(T) if (need_C and C is not None) else None
        dg = torch.empty_like(g) if (need_g and g is not None) else None
        rows = torch.empty(B * H * Lq, device=dev) if need_tau else None
        lib = _lib.load()
        with torch.cuda.device(dev):
            st = lib.tp_maslov_softmax_bwd(B, H, Lq, Lk, _ptr(T), _ptr(C), _ptr(g),
                                           *_gate_strides(g), _ptr(m), *ms, _ptr(tau), _ptr(P),
                                           _ptr(dP), _ptr(dT), _ptr(dC), _ptr(dg), _ptr(rows),
                                           _stream(dev))
        _lib.check(st, "tp_maslov_softmax_bwd")
        dtau = None
        if need_tau:
            dtau = -rows.view(B, H, Lq).sum(dim=(0, 2)) / (tau * tau)
        return dT, dC, dg, dtau, None


def maslov_softmax(scores: torch.Tensor, tau: torch.Tensor, *,
                   classical: Optional[torch.Tensor] = None, gate: Optional[torch.Tensor] = None,
                   mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Differentiable ``softmax(s / tau_h)`` with ``s = gate*scores +
    (1-gate)*classical`` (or ``scores``), set to -1e9 where ``mask == 0``;
    ``scores``/``classical`` [B, H, Lq, Lk], ``gate`` [B, Lq, H], ``tau`` [H]."""
    return MaslovSoftmaxFunction.apply(scores, classical, gate, tau, mask)
