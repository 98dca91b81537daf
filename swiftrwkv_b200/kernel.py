"""Host mirror of SwiftRWKV's RWKVKernel module over the C ABI.

Same function names, argument order and meaning as Sources/RWKVKernel/*.swift;
arrays are torch CUDA tensors (torch supplies device memory and the stream --
all arithmetic runs in librwkvcuda).  Where the reference traps on a
`precondition`, these raise ValueError; a failed CUDA call raises RWKVError.

Layouts: r, w, k, v, a, b, out: [B, T, H, N]; states [B, H, N, N] fp32 with
rows = value index and columns = key index.  Inputs keep their dtype when all
six are fp32, bf16 or fp16 alike (the kernels compute in fp32 either way);
mixed inputs are promoted to fp32, as the reference does (WKV7.swift:254).
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import BF16, F16, F32, call

WKV7_HEAD_SIZE = 64  # WKV7.swift:7
WKV7_CHUNK = 16      # WKV7.swift:8

# Launch counters, as the reference keeps them for tests (WKV7.swift:181,
# WKV7Train.swift:358, X070Backbone.swift:435).
counters = {"wkv7SequenceLaunches": 0, "wkv7ChunkedLaunches": 0, "wkv7TrainForwardLaunches": 0,
            "wkv7BackwardLaunches": 0, "stepKernelCalls": 0, "tailKernelCalls": 0}

_DT = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}


def _stream():
    return ctypes_ptr(torch.cuda.current_stream().cuda_stream)


def ctypes_ptr(x):
    import ctypes
    return ctypes.c_void_p(x)


def _ptr(t):
    return None if t is None else _lib.P(t.data_ptr())


def _common_dtype(ts):
    dts = {t.dtype for t in ts}
    if len(dts) == 1 and next(iter(dts)) in _DT:
        return next(iter(dts))
    return torch.float32


def _prep(ts, dtype):
    return [t.to(dtype).contiguous() for t in ts]


def _state(h, shape):
    if h is None:
        return None
    if tuple(h.shape) != tuple(shape):
        raise ValueError(f"hIn {tuple(h.shape)} must be [B,H,D,D] = {list(shape)}")
    return h.to(torch.float32).contiguous()


def _check_seq(r, name):
    if r.dim() != 4:
        raise ValueError(f"{name}: inputs must be [B,T,H,D], got {tuple(r.shape)}")
    B, T, H, D = r.shape
    if T < 1:
        raise ValueError(f"{name}: T ({T}) must be >= 1")
    if D != WKV7_HEAD_SIZE:
        raise ValueError(f"{name}: D ({D}) must equal HEAD_SIZE {WKV7_HEAD_SIZE}")
    return B, T, H, D


def wkv7SequenceForward(r, w, k, v, a, b, hIn=None):
    """Frozen forward over the whole sequence in one launch (WKV7.swift:242-264).
    Returns (out [B,T,H,D], hOut [B,H,D,D] fp32)."""
    B, T, H, D = _check_seq(r, "wkv7SequenceForward")
    dt = _common_dtype((r, w, k, v, a, b))
    r, w, k, v, a, b = _prep((r, w, k, v, a, b), dt)
    h = _state(hIn, (B, H, D, D))
    out = torch.empty_like(r)
    h_out = torch.empty((B, H, D, D), device=r.device, dtype=torch.float32)
    call("rwkv_wkv7_forward", _DT[dt], *map(_ptr, (r, w, k, v, a, b, h, out, h_out)),
         B, T, H, D, _stream())
    counters["wkv7SequenceLaunches"] += 1
    return out, h_out


def wkv7ForwardWithState(r, w, k, v, a, b, hIn=None):
    """WKV7.swift:96-103: same result as wkv7SequenceForward."""
    return wkv7SequenceForward(r, w, k, v, a, b, hIn)


def wkv7ForwardChunked(r, w, k, v, a, b, hIn=None):
    """WKV7.swift:107-140: chunked by 16 in the reference; one launch here,
    bit-identical to wkv7SequenceForward as the reference requires."""
    return wkv7SequenceForward(r, w, k, v, a, b, hIn)


def wkv7PrefillChunked(r, w, k, v, a, b, hIn=None):
    """Prefill form of wkv7SequenceForward: 16-token chunks in the normalised
    DPLR form (rwkv_wkv7_forward_chunked); equal to it to fp32 rounding, not
    bitwise.  Returns (out [B,T,H,D], hOut [B,H,D,D] fp32)."""
    B, T, H, D = _check_seq(r, "wkv7PrefillChunked")
    dt = _common_dtype((r, w, k, v, a, b))
    r, w, k, v, a, b = _prep((r, w, k, v, a, b), dt)
    h = _state(hIn, (B, H, D, D))
    out = torch.empty_like(r)
    h_out = torch.empty((B, H, D, D), device=r.device, dtype=torch.float32)
    ws_bytes = int(_lib.lib().rwkv_wkv7_forward_chunked_workspace_size(B, T, H, D))
    ws = torch.empty(max(ws_bytes, 16), device=r.device, dtype=torch.uint8)
    call("rwkv_wkv7_forward_chunked", _DT[dt], *map(_ptr, (r, w, k, v, a, b, h, out, h_out)), None,
         B, T, H, D, _ptr(ws), ws_bytes, _stream())
    counters["wkv7ChunkedLaunches"] += 1
    return out, h_out


def wkv7Forward(r, w, k, v, a, b):
    """Zero initial state, final state dropped (WKV7.swift:143-148)."""
    return wkv7SequenceForward(r, w, k, v, a, b, None)[0]


def wkv7ChunkForward(r, w, k, v, a, b, hIn):
    """One chunk of exactly 16 steps (WKV7.swift:64-82): (out, hOut, saOut)."""
    B, T, H, D = _check_seq(r, "wkv7ChunkForward")
    if T != WKV7_CHUNK:
        raise ValueError(f"T ({T}) must equal CHUNK {WKV7_CHUNK}")
    out, h_out, sa, _ = _train_forward(r, w, k, v, a, b, hIn)
    return out, h_out, sa


def _train_forward(r, w, k, v, a, b, hIn):
    B, T, H, D = r.shape
    dt = _common_dtype((r, w, k, v, a, b))
    r, w, k, v, a, b = _prep((r, w, k, v, a, b), dt)
    h = _state(hIn, (B, H, D, D))
    out = torch.empty_like(r)
    h_out = torch.empty((B, H, D, D), device=r.device, dtype=torch.float32)
    sa = torch.empty(r.shape, device=r.device, dtype=torch.float32)
    ck = torch.empty((B, H, T // WKV7_CHUNK, D, D), device=r.device, dtype=torch.float32)
    call("rwkv_wkv7_train_forward", _DT[dt], *map(_ptr, (r, w, k, v, a, b, h, out, h_out, sa, ck)),
         B, T, H, D, _stream())
    counters["wkv7TrainForwardLaunches"] += 1
    return out, h_out, sa, ck


def wkv7Backward(r, w, k, v, a, b, hIn, hCkpt, dOut, dHOut=None):
    """The VJP kernel of wkv7TrainWithState (WKV7Train.swift:410-420):
    returns (dr, dw, dk, dv, da, db, dhIn)."""
    B, T, H, D = _check_seq(r, "wkv7Backward")
    if T % WKV7_CHUNK:
        raise ValueError(f"T ({T}) must be divisible by CHUNK {WKV7_CHUNK}")
    dt = _common_dtype((r, w, k, v, a, b, dOut))
    r, w, k, v, a, b, dOut = _prep((r, w, k, v, a, b, dOut), dt)
    h = _state(hIn, (B, H, D, D))
    dh = _state(dHOut, (B, H, D, D))
    grads = [torch.empty_like(r) for _ in range(6)]
    dh_in = torch.empty((B, H, D, D), device=r.device, dtype=torch.float32)
    ws_bytes = _lib.lib().rwkv_wkv7_backward_workspace_size(B, T, H, D)
    ws = torch.empty(max(int(ws_bytes), 16), device=r.device, dtype=torch.uint8)
    call("rwkv_wkv7_backward", _DT[dt], *map(_ptr, (r, w, k, v, a, b, h, hCkpt.contiguous(), dOut, dh)),
         *map(_ptr, grads), _ptr(dh_in), B, T, H, D, _ptr(ws), ws_bytes, _stream())
    counters["wkv7BackwardLaunches"] += 1
    return (*grads, dh_in)


def wkv7TrainForwardChunked(r, w, k, v, a, b, hIn=None):
    """Chunked form of the training forward (rwkv_wkv7_train_forward_chunked):
    returns (out, hOut, sa, hCkpt) like the sequential one, to fp32 rounding."""
    B, T, H, D = _check_seq(r, "wkv7TrainForwardChunked")
    if T % WKV7_CHUNK:
        raise ValueError(f"T ({T}) must be divisible by CHUNK {WKV7_CHUNK}")
    dt = _common_dtype((r, w, k, v, a, b))
    r, w, k, v, a, b = _prep((r, w, k, v, a, b), dt)
    h = _state(hIn, (B, H, D, D))
    out = torch.empty_like(r)
    h_out = torch.empty((B, H, D, D), device=r.device, dtype=torch.float32)
    sa = torch.empty(r.shape, device=r.device, dtype=torch.float32)
    ck = torch.empty((B, H, T // WKV7_CHUNK, D, D), device=r.device, dtype=torch.float32)
    ws_bytes = int(_lib.lib().rwkv_wkv7_forward_chunked_workspace_size(B, T, H, D))
    ws = torch.empty(max(ws_bytes, 16), device=r.device, dtype=torch.uint8)
    call("rwkv_wkv7_train_forward_chunked", _DT[dt], *map(_ptr, (r, w, k, v, a, b, h, out, h_out, sa, ck)),
         B, T, H, D, _ptr(ws), ws_bytes, _stream())
    counters["wkv7TrainForwardLaunches"] += 1
    return out, h_out, sa, ck


def wkv7BackwardChunked(r, w, k, v, a, b, hIn, hCkpt, dOut, dHOut=None):
    """Chunked (DPLR) form of wkv7Backward (rwkv_wkv7_backward_chunked): the
    same gradients (dr, dw, dk, dv, da, db, dhIn) to fp32 rounding."""
    B, T, H, D = _check_seq(r, "wkv7BackwardChunked")
    if T % WKV7_CHUNK:
        raise ValueError(f"T ({T}) must be divisible by CHUNK {WKV7_CHUNK}")
    dt = _common_dtype((r, w, k, v, a, b, dOut))
    r, w, k, v, a, b, dOut = _prep((r, w, k, v, a, b, dOut), dt)
    h = _state(hIn, (B, H, D, D))
    dh = _state(dHOut, (B, H, D, D))
    grads = [torch.empty_like(r) for _ in range(6)]
    dh_in = torch.empty((B, H, D, D), device=r.device, dtype=torch.float32)
    ws_bytes = int(_lib.lib().rwkv_wkv7_backward_chunked_workspace_size(B, T, H, D))
    ws = torch.empty(max(ws_bytes, 16), device=r.device, dtype=torch.uint8)
    call("rwkv_wkv7_backward_chunked", _DT[dt],
         *map(_ptr, (r, w, k, v, a, b, h, hCkpt.contiguous(), dOut, dh)), *map(_ptr, grads), _ptr(dh_in),
         B, T, H, D, _ptr(ws), ws_bytes, _stream())
    counters["wkv7BackwardLaunches"] += 1
    return (*grads, dh_in)


# The differentiable path's kernels: chunked (DPLR) forward and backward when
# True, the sequential ones (the reference's kernel structure) when False.
useChunkedTraining = True


class _WKV7Train(torch.autograd.Function):
    """Differentiable WKV-7 with explicit state: forward outputs are kept for
    the backward (wkv7KeepForwardOutputs = true, WKV7Train.swift:354)."""

    @staticmethod
    def forward(ctx, r, w, k, v, a, b, h0):
        ctx.chunked = useChunkedTraining
        fwd = wkv7TrainForwardChunked if ctx.chunked else _train_forward
        out, h_out, sa, ck = fwd(r, w, k, v, a, b, h0)
        ctx.save_for_backward(r, w, k, v, a, b, h0, ck)
        ctx.in_dtypes = [t.dtype for t in (r, w, k, v, a, b, h0)]
        return out, h_out

    @staticmethod
    def backward(ctx, d_out, d_h_out):
        r, w, k, v, a, b, h0, ck = ctx.saved_tensors
        if d_out is None:
            d_out = torch.zeros_like(r)
        bwd = wkv7BackwardChunked if ctx.chunked else wkv7Backward
        g = bwd(r, w, k, v, a, b, h0, ck, d_out, d_h_out)
        return tuple(gi.to(dt) for gi, dt in zip(g, ctx.in_dtypes))


def wkv7TrainWithState(r, w, k, v, a, b, hIn=None):
    """Differentiable forward with explicit boundary state (WKV7Train.swift:375-468):
    returns (out, hOut); gradients flow to all seven inputs, hIn included."""
    B, T, H, D = _check_seq(r, "wkv7TrainWithState")
    if T % WKV7_CHUNK:
        raise ValueError(f"T ({T}) must be divisible by CHUNK {WKV7_CHUNK}")
    h0 = hIn if hIn is not None else torch.zeros((B, H, D, D), device=r.device, dtype=torch.float32)
    if tuple(h0.shape) != (B, H, D, D):
        raise ValueError(f"hIn {tuple(h0.shape)} must be [B,H,D,D] = {[B, H, D, D]}")
    return _WKV7Train.apply(r, w, k, v, a, b, h0)


def wkv7Train(r, w, k, v, a, b):
    """Zero-state wrapper (WKV7Train.swift:472-475)."""
    return wkv7TrainWithState(r, w, k, v, a, b, None)[0]


def wkv7Steps(r, w, k, v, a, b, hIn=None):
    """Several differentiable steps (WKV7Step.swift:79-100): r..b [B, T, H, D]
    for any T >= 1, hIn [B, H, D, D] or None (zeros); returns (out [B, T, H, D]
    fp32, hOut [B, H, D, D]), differentiable w.r.t. all seven inputs.  The
    reference unrolls MLX ops; here T is padded to a multiple of CHUNK with
    identity steps (w = 1, r = k = v = a = b = 0: the state passes unchanged,
    the padded outputs are 0) and the WKV-7 training kernels run forward and
    backward, so the gradients are those of the unpadded steps."""
    if r.dim() != 4:
        raise ValueError(f"wkv7Steps expects [B,T,H,D], got {tuple(r.shape)}")
    B, T, H, D = _check_seq(r, "wkv7Steps")
    xs = [x.to(torch.float32) for x in (r, w, k, v, a, b)]
    for x in xs[1:]:
        if tuple(x.shape) != (B, T, H, D):
            raise ValueError(f"wkv7Steps: every input must be [B,T,H,D] = {[B, T, H, D]}")
    pad = (-T) % WKV7_CHUNK
    if pad:
        xs = [torch.cat([x, torch.full((B, pad, H, D), 1.0 if i == 1 else 0.0, device=x.device,
                                       dtype=torch.float32)], dim=1) for i, x in enumerate(xs)]
    out, h_out = wkv7TrainWithState(*xs, hIn)
    return out[:, :T], h_out


def wkv7Step(r, w, k, v, a, b, hIn=None):
    """One differentiable step (WKV7Step.swift:45-67): r..b [B, H, D] (out
    [B, H, D]) or [B, 1, H, D] (out [B, 1, H, D]); hIn [B, H, D, D] or None.
    Returns (out fp32, hOut [B, H, D, D])."""
    if r.dim() == 4:
        if r.shape[1] != 1:
            raise ValueError(f"wkv7Step takes exactly one token, for several use wkv7Steps (T={r.shape[1]})")
        return wkv7Steps(r, w, k, v, a, b, hIn)
    if r.dim() != 3:
        raise ValueError(f"wkv7Step expects [B,H,D] or [B,1,H,D], got {tuple(r.shape)}")
    out, h_out = wkv7Steps(*(x.unsqueeze(1) for x in (r, w, k, v, a, b)), hIn)
    return out[:, 0], h_out


def wkv7StepForward(r, w, k, v, a, b, h):
    """One token (WKV7DecodeKernels.swift:73-89): r..b [H, S] (or [rows, H, S]),
    h [H, S, S] (or [rows, H, S, S]).  Returns (out, h') fp32; h is not modified."""
    single = r.dim() == 2
    if single:
        r, w, k, v, a, b = (t.unsqueeze(0) for t in (r, w, k, v, a, b))
        h = h.unsqueeze(0)
    rows, H, S = r.shape
    if S != WKV7_HEAD_SIZE:
        raise ValueError(f"S ({S}) must equal HEAD_SIZE {WKV7_HEAD_SIZE}")
    if tuple(h.shape) != (rows, H, S, S):
        raise ValueError(f"state {tuple(h.shape)}, expected {[rows, H, S, S]}")
    r, w, k, v, a, b = _prep((r, w, k, v, a, b), torch.float32)
    h2 = h.to(torch.float32).contiguous().clone()
    out = torch.empty_like(r)
    call("rwkv_wkv7_step", F32, *map(_ptr, (r, w, k, v, a, b, h2, out)), rows, H, S, _stream())
    counters["stepKernelCalls"] += 1
    if single:
        return out[0], h2[0]
    return out, h2


def wkvTailApplies(headSize: int) -> bool:
    """WKV7DecodeKernels.swift:92."""
    return headSize % 32 == 0


def wkvTail(wkv, r, k, v, rK, lnWeight, lnBias, gate, nHead, headSize, rows=1, eps=64e-5):
    """Fused tmix tail (WKV7DecodeKernels.swift:106-178): returns [rows, D] fp32."""
    H, S = nHead, headSize
    if not wkvTailApplies(S):
        raise ValueError(f"tail: S={S} not a multiple of the warp width")
    D = H * S
    f = lambda t, n: t.reshape(n).to(torch.float32).contiguous()
    wkv, r, k, v, gate = (f(t, rows * D) for t in (wkv, r, k, v, gate))
    rK, lnWeight, lnBias = (f(t, D) for t in (rK, lnWeight, lnBias))
    out = torch.empty((rows, D), device=wkv.device, dtype=torch.float32)
    call("rwkv_wkv_tail", *map(_ptr, (wkv, r, k, v, rK, lnWeight, lnBias, gate, out)), rows, H, S,
         _lib.F(eps), _stream())
    counters["tailKernelCalls"] += 1
    return out


def wkv7StepTail(r, w, k, v, a, b, h, rK, lnWeight, lnBias, gate, eps=64e-5):
    """The step and the tail in one launch, updating h in place: r..b, gate
    [rows, H, S] fp32; h [rows, H, S, S]; returns the tail output [rows, H*S]."""
    rows, H, S = r.shape
    out = torch.empty((rows, H * S), device=r.device, dtype=torch.float32)
    call("rwkv_wkv7_step_tail", *map(_ptr, (r, w, k, v, a, b, h, rK, lnWeight, lnBias, gate, out)),
         rows, H, S, _lib.F(eps), _stream())
    return out
