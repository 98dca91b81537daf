"""CPU oracle for the WKV-7 and quantised-GEMV hot paths -- TEST INFRASTRUCTURE.

Thin numpy wrapper over ``oracle/_build/librwkv_oracle.so`` (built from
``rwkv_oracle.c`` by ``oracle/Makefile``).  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this
module; the product library never does.

Every function takes and returns numpy arrays in the reference's layouts:
r/w/k/v/a/b/y are ``[B,T,H,N]`` fp32, states ``[B,H,N,N]`` fp32 with rows = value
index dv and columns = key index dk (WKV7Step.swift:19-24).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "librwkv_oracle.so")
_lib = None

F32, BF16, F16 = 0, 1, 2
WKV_CHUNK = 16


def build() -> str:
    """Compile the oracle (make -C oracle); returns the library path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
    return _lib


def _p(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int) -> None:
    """OpenMP thread count used by the oracle's parallel loops."""
    os.environ["OMP_NUM_THREADS"] = str(n)
    try:
        gomp = ctypes.CDLL("libgomp.so.1")
        gomp.omp_set_num_threads(ctypes.c_int(n))
    except OSError:
        pass


# ----------------------------------------------------------------- fp16 / bf16

def f32_to_f16_bits(x):
    x = _f32(x)
    out = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_f16(_p(x), _p(out), ctypes.c_int64(x.size))
    return out


def f16_bits_to_f32(h):
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().orc_f16_to_f32(_p(h), _p(out), ctypes.c_int64(h.size))
    return out


def f32_to_bf16_bits(x):
    x = _f32(x)
    out = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_bf16(_p(x), _p(out), ctypes.c_int64(x.size))
    return out


def bf16_bits_to_f32(h):
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().orc_bf16_to_f32(_p(h), _p(out), ctypes.c_int64(h.size))
    return out


# ----------------------------------------------------------------------- WKV-7

def wkv7_forward(r, w, k, v, a, b, h_in=None, want_sa=False, ckpt_every=0):
    """Forward (WKV7.swift:193-226 order). Returns (y, h_out[, sa][, h_ckpt])."""
    r, w, k, v, a, b, h_in = (_f32(x) for x in (r, w, k, v, a, b, h_in))
    B, T, H, N = r.shape
    y = np.empty_like(r)
    h_out = np.empty((B, H, N, N), np.float32)
    sa = np.empty_like(r) if want_sa else None
    ck = np.empty((B, H, T // ckpt_every, N, N), np.float32) if ckpt_every else None
    lib().orc_wkv7_forward(_p(r), _p(w), _p(k), _p(v), _p(a), _p(b), _p(h_in), _p(y),
                           _p(h_out), _p(sa), _p(ck), ctypes.c_int(ckpt_every),
                           B, T, H, N)
    out = [y, h_out]
    if want_sa:
        out.append(sa)
    if ckpt_every:
        out.append(ck)
    return tuple(out)


def wkv7_backward_v2(r, w, k, v, a, b, h_ckpt, sa, dy, dh_out=None):
    """Reference v2 backward (WKV7Train.swift:247-330). Returns (dr,dw,dk,dv,da,db,dh_in)."""
    r, w, k, v, a, b, h_ckpt, sa, dy, dh_out = (
        _f32(x) for x in (r, w, k, v, a, b, h_ckpt, sa, dy, dh_out))
    B, T, H, N = r.shape
    assert T % WKV_CHUNK == 0
    grads = [np.empty_like(r) for _ in range(6)]
    dh_in = np.empty((B, H, N, N), np.float32)
    lib().orc_wkv7_backward_v2(_p(r), _p(w), _p(k), _p(v), _p(a), _p(b), _p(h_ckpt),
                               _p(sa), _p(dy), _p(dh_out), *(_p(g) for g in grads),
                               _p(dh_in), B, T, H, N)
    return (*grads, dh_in)


def wkv7_train(r, w, k, v, a, b, h_in=None, dy=None, dh_out=None):
    """Train forward (ckpt every 16) + v2 backward, the reference's train path."""
    y, h_out, sa, ck = wkv7_forward(r, w, k, v, a, b, h_in, want_sa=True,
                                    ckpt_every=WKV_CHUNK)
    if dy is None:
        return y, h_out
    return (y, h_out) + wkv7_backward_v2(r, w, k, v, a, b, ck, sa, dy, dh_out)


def wkv7_exact(r, w, k, v, a, b, h_in=None, dy=None, dh_out=None):
    """Double-precision forward (+ backward when dy is given), states kept for
    every step -- the autograd reference's semantics (WKV7Reference.swift:31-76).
    Returns (y, h_out) or (y, h_out, dr, dw, dk, dv, da, db, dh_in)."""
    r, w, k, v, a, b, h_in, dy, dh_out = (
        _f32(x) for x in (r, w, k, v, a, b, h_in, dy, dh_out))
    B, T, H, N = r.shape
    y = np.empty_like(r)
    h_out = np.empty((B, H, N, N), np.float32)
    if dy is None:
        lib().orc_wkv7_exact(_p(r), _p(w), _p(k), _p(v), _p(a), _p(b), _p(h_in), None,
                             None, _p(y), _p(h_out), None, None, None, None, None, None,
                             None, B, T, H, N)
        return y, h_out
    grads = [np.empty_like(r) for _ in range(6)]
    dh_in = np.empty((B, H, N, N), np.float32)
    lib().orc_wkv7_exact(_p(r), _p(w), _p(k), _p(v), _p(a), _p(b), _p(h_in), _p(dy),
                         _p(dh_out), _p(y), _p(h_out), *(_p(g) for g in grads), _p(dh_in),
                         B, T, H, N)
    return (y, h_out, *grads, dh_in)


def wkv7_step(r, w, k, v, a, b, h):
    """One token (WKV7DecodeKernels.swift:123-142): inputs [rows,H,N], state
    [rows,H,N,N].  Returns (y, h_new)."""
    r, w, k, v, a, b, h = (_f32(x) for x in (r, w, k, v, a, b, h))
    rows, H, N = r.shape
    y, h_new = wkv7_forward(*(x.reshape(rows, 1, H, N) for x in (r, w, k, v, a, b)), h)
    return y.reshape(rows, H, N), h_new


def wkv_tail(wkv, r, k, v, rk, lnw, lnb, g, H, S, eps=64e-5):
    """wkvTail (WKV7DecodeKernels.swift:190-262) on [rows, H*S] inputs."""
    wkv, r, k, v, rk, lnw, lnb, g = (_f32(x) for x in (wkv, r, k, v, rk, lnw, lnb, g))
    rows = wkv.size // (H * S)
    out = np.empty((rows, H * S), np.float32)
    lib().orc_wkv_tail(_p(wkv), _p(r), _p(k), _p(v), _p(rk), _p(lnw), _p(lnb), _p(g),
                       _p(out), rows, H, S, ctypes.c_float(eps))
    return out


# ------------------------------------------------------------ MLX affine (QLoRA)

def affine_quantize(W, group=64, bits=4):
    """Restated MLX affine quantiser (parity-unpinned). W [OUT, IN] fp32 values
    (fp16-exact). Returns (wq u32 [OUT, IN*bits/32], scales f16-bits, biases f16-bits)."""
    W = _f32(W)
    OUT, IN = W.shape
    wq = np.zeros((OUT, IN * bits // 32), np.uint32)
    sc = np.empty((OUT, IN // group), np.uint16)
    bi = np.empty((OUT, IN // group), np.uint16)
    lib().orc_affine_quantize(_p(W), OUT, IN, group, bits, _p(wq), _p(sc), _p(bi))
    return wq, sc, bi


def _sb_dtype(s):
    return F32 if s.dtype == np.float32 else F16


def affine_dequant(wq, scales, biases, group=64, bits=4):
    wq = np.ascontiguousarray(wq, np.uint32)
    OUT = wq.shape[0]
    IN = wq.shape[1] * 32 // bits
    out = np.empty((OUT, IN), np.float32)
    lib().orc_affine_dequant(_p(wq), _p(scales), _p(biases), _sb_dtype(scales), _p(out),
                             OUT, IN, group, bits)
    return out


def affine_gemv(x, wq, scales, biases, group=64, bits=4, exact=False):
    """y = x @ W.T with W the dequantised weight; x [rows, IN] fp32."""
    x = _f32(x)
    rows, IN = x.shape
    OUT = wq.shape[0]
    y = np.empty((rows, OUT), np.float32)
    fn = lib().orc_affine_gemv_exact if exact else lib().orc_affine_gemv
    fn(_p(x), _p(np.ascontiguousarray(wq, np.uint32)), _p(scales), _p(biases),
       _sb_dtype(scales), _p(y), rows, OUT, IN, group, bits)
    return y


def base_matmul_vjp(dy, W):
    """The bf16 backward of a frozen base projection y = x W^T, restated from
    X070Backbone.baseMatmul's VJP (Sources/RWKVGen/X070Backbone.swift:337-356):
    matmul(dy.asType(bf16), W.asType(bf16)), a bf16 result.  dy [rows, OUT],
    W [OUT, IN] (fp32 values; both rounded to bf16 here).  Returns
    (dx, exact): dx the bf16-rounded sum widened to fp32, exact the float64
    sum of the bf16 operands (a kernel's fp32 sum lies within fp32 rounding of
    it, so its bf16 rounding equals dx except at near-ties)."""
    dyb = bf16_bits_to_f32(f32_to_bf16_bits(dy)).astype(np.float64)
    Wb = bf16_bits_to_f32(f32_to_bf16_bits(W)).astype(np.float64)
    exact = dyb @ Wb
    return bf16_bits_to_f32(f32_to_bf16_bits(exact.astype(np.float32))), exact


# ------------------------------------------------------------------ .rwkvq sb6

def sb6_dequant(qblk, qsqm, ddm, OUT, IN, xbits):
    out = np.empty((OUT, IN), np.float32)
    lib().orc_sb6_dequant(_p(qblk), _p(qsqm), _p(ddm), _p(out), OUT, IN, xbits)
    return out


def sb6_gemv(x, qblk, qsqm, ddm, OUT, IN, xbits):
    x = _f32(x).reshape(IN)
    y = np.empty((OUT,), np.float32)
    lib().orc_sb6_gemv(_p(x), _p(qblk), _p(qsqm), _p(ddm), _p(y), OUT, IN, xbits)
    return y


def sb6_to_affine(qblk, qsqm, ddm, OUT, IN, xbits):
    bits = 4 + xbits
    wq = np.empty((OUT, IN // 32 * bits), np.uint32)
    sc = np.empty((OUT, IN // 32), np.float32)
    bi = np.empty((OUT, IN // 32), np.float32)
    ok = ctypes.c_int(0)
    lib().orc_sb6_to_affine(_p(qblk), _p(qsqm), _p(ddm), _p(wq), _p(sc), _p(bi), OUT, IN,
                            xbits, ctypes.byref(ok))
    return wq, sc, bi, bool(ok.value)


# ------------------------------------------------------------------ .rwkvq sym

def sym_dequant(qblk, qs, d, OUT, IN, bits, odtype=F32):
    out = np.empty((OUT, IN), np.float32 if odtype == F32 else np.uint16)
    lib().orc_sym_dequant(_p(qblk), _p(qs), _p(d), _p(out), odtype, OUT, IN, bits)
    return out


def sym_gemv(x, qblk, qs, d, OUT, IN, bits, out_per=None, nn=None):
    x = _f32(x)
    out_per = OUT if out_per is None else out_per
    nk = OUT // out_per
    nn = x.shape[0] // nk if nn is None else nn
    y = np.empty((nn, OUT), np.float32)
    lib().orc_sym_gemv(_p(x), _p(qblk), _p(qs), _p(d), _p(y), nn, OUT, IN, bits, out_per)
    return y


def sym_rows(ids, codes, qs, d, IN):
    ids = np.ascontiguousarray(ids, np.int32)
    out = np.empty((ids.size, IN), np.uint16)
    lib().orc_sym_rows(_p(ids), ids.size, _p(codes), _p(qs), _p(d), _p(out), IN)
    return out


# ------------------------------------------------------------------ state tuning

def state_layer_grad(r, w, k, v, a, b, dy, state):
    """Gradient of sum(y * dy) w.r.t. a layer's initial state [H,N,N] shared
    by the batch (StateTrainableSet, InitialState.swift:176-251): h_in[b] =
    state, the train forward + v2 backward, then dh_in summed over b in order."""
    B = r.shape[0]
    h_in = np.ascontiguousarray(np.broadcast_to(_f32(state), (B,) + state.shape))
    out = wkv7_train(r, w, k, v, a, b, h_in, dy)
    dh_in = out[-1]
    g = np.zeros(state.shape, np.float32)
    for i in range(B):
        g = (g + dh_in[i]).astype(np.float32)
    return g


def adamw_clip_step(param, m, v, grad, *, grad_scale, clip, lr, beta1, beta2, eps,
                    weight_decay, c1, c2):
    """One optimizer step of Trainer.run (Trainer.swift:141-161) with
    clipByGlobalNorm (:182-189), each elementwise operation rounded to fp32
    (numpy float32 arithmetic does not fuse).  The sum of squares is taken in
    double.  Returns (param, m, v, norm) as new arrays."""
    f = np.float32
    g = (_f32(grad) * f(grad_scale)).astype(f)
    norm = f(np.sqrt(f(np.sum((g * g).astype(np.float64)))))
    if clip > 0:
        s = min(f(1), f(f(clip) / f(norm + f(1e-6))))
        g = (g * f(s)).astype(f)
    m = (f(beta1) * _f32(m) + (f(1) - f(beta1)) * g).astype(f)
    v = (f(beta2) * _f32(v) + (f(1) - f(beta2)) * (g * g)).astype(f)
    mhat = (m / f(c1)).astype(f)
    vhat = (v / f(c2)).astype(f)
    upd = (mhat / (np.sqrt(vhat) + f(eps))).astype(f)
    p = _f32(param)
    if weight_decay > 0:
        upd = (upd + f(weight_decay) * p).astype(f)
    return (p - f(lr) * upd).astype(f), m, v, norm
