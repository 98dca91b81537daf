"""Host mirror of the quantised-base entry points the reference uses.

* MLX affine container (the QLoRA base): `quantized`, `dequantized`,
  `quantizedMM` with MLX's argument names (called at Sources/RWKVGen/
  LoRA.swift:68 and X070Backbone.swift:678-681, 759-766), plus `QuantBase`;
  `baseMatmulVJP`, the bf16 backward of a frozen base projection.
* .rwkvq sb6 / sym (Sources/RWKVQuant): `rwkvqDequantDense`, `rwkvqSb6GEMV`,
  `rwkvqDequantSym`, `rwkvqSymGEMV`, `symGEMVFused`, `RwkvqSymRowTable`,
  `nativeAffine`, with the reference's `...Applies` predicates.  GEMV entry
  points return None where the reference returns nil (shape not taken).

Arrays are torch CUDA tensors; packed buffers are uint8 / int32-viewed-uint32
tensors as the reference keeps them.  All arithmetic runs in librwkvcuda.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from ._lib import BF16, F16, F32, call

_DT = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}


def _s():
    return _lib.P(torch.cuda.current_stream().cuda_stream)


def _p(t):
    return None if t is None else _lib.P(t.data_ptr())


# ------------------------------------------------------------------ MLX affine

@dataclass
class QuantBase:
    """Frozen quantised matrix (X070Backbone.swift:79-85)."""
    wq: torch.Tensor       # int32 storage of u32 words [OUT, IN*bits/32]
    scales: torch.Tensor   # [OUT, IN/group]
    biases: torch.Tensor   # [OUT, IN/group]
    groupSize: int
    bits: int

    @property
    def outFeatures(self):
        return self.wq.shape[0]

    @property
    def inFeatures(self):
        return self.wq.shape[1] * 32 // self.bits


def quantized(W: torch.Tensor, groupSize: int = 64, bits: int = 4):
    """MLX `quantized` (affine): returns (wq, scales, biases); scales/biases in
    W's dtype."""
    if W.dim() != 2:
        raise ValueError("quantized: W must be [OUT, IN]")
    if W.dtype not in _DT:
        W = W.to(torch.float32)
    W = W.contiguous()
    OUT, IN = W.shape
    wq = torch.empty((OUT, IN * bits // 32), device=W.device, dtype=torch.int32)
    sc = torch.empty((OUT, IN // groupSize), device=W.device, dtype=W.dtype)
    bi = torch.empty_like(sc)
    call("rwkv_q_quantize", _DT[W.dtype], _p(W), _p(wq), _p(sc), _p(bi), OUT, IN, groupSize, bits, _s())
    return wq, sc, bi


def dequantized(wq, scales, biases, groupSize=64, bits=4, dtype=None):
    """MLX `dequantized`: dense [OUT, IN] in `dtype` (default: scales' dtype)."""
    dtype = dtype or scales.dtype
    OUT = wq.shape[0]
    IN = wq.shape[1] * 32 // bits
    out = torch.empty((OUT, IN), device=wq.device, dtype=dtype)
    call("rwkv_q_dequant", _p(wq.contiguous()), _p(scales.contiguous()), _p(biases.contiguous()),
         _DT[scales.dtype], _DT[dtype], _p(out), OUT, IN, groupSize, bits, _s())
    return out


def quantizedMM(x, wq, scales, biases, transpose=True, groupSize=64, bits=4, out_dtype=None):
    """MLX `quantizedMM(x, w, transpose: true)`: y = x W^T, [..., OUT] in x's
    dtype (or `out_dtype`); accumulation in fp32."""
    if not transpose:
        raise ValueError("quantizedMM: only transpose=true is used by the reference")
    lead = x.shape[:-1]
    IN = x.shape[-1]
    OUT = wq.shape[0]
    if x.dtype not in _DT:
        x = x.to(torch.float32)
    x2 = x.reshape(-1, IN).contiguous()
    rows = x2.shape[0]
    ydt = out_dtype or x.dtype
    y = torch.empty((rows, OUT), device=x.device, dtype=ydt)
    call("rwkv_q_gemm", _DT[x2.dtype], _p(x2), _p(wq), _p(scales), _p(biases), _DT[scales.dtype],
         _DT[ydt], _p(y), rows, OUT, IN, groupSize, bits, _s())
    return y.reshape(*lead, OUT)


def baseMatmulVJP(cotangent, weight=None, q: QuantBase | None = None, primal_dtype=None, out=None):
    """The backward of a frozen base projection y = x W^T, the VJP
    X070Backbone gives baseMatmul (X070Backbone.swift:337-356, bf16 backward):
    dX = matmul(cotangent.asType(bf16), W_bf16), a bf16 result cast to the
    primal's dtype (`primal_dtype`, default the cotangent's).  `weight`: the
    dense bf16 [OUT, IN] (a dense target, or a base dequantised to bf16);
    `q`: the 4-bit group-64 container, dequantised inside the kernel.  With
    `out` (an fp32 [..., IN] tensor) the result is added into it instead."""
    if (weight is None) == (q is None):
        raise ValueError("baseMatmulVJP: give exactly one of weight / q")
    OUT = cotangent.shape[-1]
    lead = cotangent.shape[:-1]
    dy = cotangent.reshape(-1, OUT).to(torch.bfloat16).contiguous()
    rows = dy.shape[0]
    IN = weight.shape[1] if weight is not None else q.inFeatures
    if out is not None:
        if out.dtype != torch.float32 or not out.is_contiguous() or out.numel() != rows * IN:
            raise ValueError("baseMatmulVJP: out must be a contiguous fp32 tensor of [..., IN]")
        dx, acc = out, 1
    else:
        dt = primal_dtype or cotangent.dtype
        if dt not in _DT:
            dt = torch.float32
        dx, acc = torch.empty((rows, IN), device=dy.device, dtype=dt), 0
    if weight is not None:
        w = weight.to(torch.bfloat16).contiguous()
        call("rwkv_gemm_dx", BF16, _p(dy), BF16, _p(w), _DT[dx.dtype], _p(dx), rows, OUT, IN, acc, _s())
    else:
        call("rwkv_q_gemm_dx", BF16, _p(dy), _p(q.wq), _p(q.scales), _p(q.biases), _DT[q.scales.dtype],
             _DT[dx.dtype], _p(dx), rows, OUT, IN, q.groupSize, q.bits, acc, _s())
    return dx.reshape(*lead, IN)


def quantized_rows(ids, q: QuantBase, dtype=torch.float16):
    """Embedding rows of a quantised table (X070Backbone.embed, :758-767)."""
    ids32 = ids.reshape(-1).to(torch.int32).contiguous()
    out = torch.empty((ids32.numel(), q.inFeatures), device=q.wq.device, dtype=dtype)
    call("rwkv_q_rows", _p(ids32), ids32.numel(), _p(q.wq), _p(q.scales), _p(q.biases),
         _DT[q.scales.dtype], _DT[dtype], _p(out), q.outFeatures, q.inFeatures, q.groupSize,
         q.bits, _s())
    return out.reshape(*ids.shape, q.inFeatures)


# ------------------------------------------------------------------------ sb6

def rwkvqDequantDense(qblk, qsqm, ddm, outFeatures, inFeatures, superBlock, xbits,
                      dtype=torch.float32):
    """RwkvqDequant.swift:160-183."""
    if not (qblk.dtype == torch.uint8 and qsqm.dtype == torch.uint8 and ddm.dtype == torch.float16):
        raise ValueError("sb6 dequant: buffers must be uint8/uint8/float16")
    if superBlock != 8:
        raise ValueError(f"sb6 dequant: superblock {superBlock}, kernel built for 8")
    out = torch.empty((outFeatures, inFeatures), device=qblk.device, dtype=dtype)
    call("rwkv_sb6_dequant", _p(qblk), _p(qsqm), _p(ddm), _DT[dtype], _p(out), outFeatures,
         inFeatures, xbits, _s())
    return out


def rwkvqSb6GEMVApplies(outFeatures, inFeatures, xbits, superBlock, rows):
    """RwkvqSb6GEMV.swift:159-164 (any rows >= 1 are taken here)."""
    return 0 <= xbits <= 2 and superBlock == 8 and rows >= 1 and inFeatures % 256 == 0


def rwkvqSb6GEMV(x, qblk, qsqm, ddm, outFeatures, inFeatures, xbits):
    """y = x W^T over the K3 interleave (RwkvqSb6GEMV.swift:170-190); x [rows, IN]
    -> [rows, OUT] fp32."""
    if x.dim() != 2 or x.shape[1] != inFeatures:
        raise ValueError(f"sb6-GEMV: input {tuple(x.shape)}, expected [N, {inFeatures}]")
    if not (qblk.dtype == torch.uint8 and qsqm.dtype == torch.uint8 and ddm.dtype == torch.float16):
        raise ValueError("sb6-GEMV: buffers must be uint8/uint8/float16")
    x = x if x.dtype in _DT else x.to(torch.float32)
    x = x.contiguous()
    y = torch.empty((x.shape[0], outFeatures), device=x.device, dtype=torch.float32)
    call("rwkv_sb6_gemv", _DT[x.dtype], _p(x), _p(qblk), _p(qsqm), _p(ddm), _p(y), x.shape[0],
         outFeatures, inFeatures, xbits, _s())
    return y


@dataclass
class RwkvqNativeWeight:
    """sb6 relaid into the MLX affine container (RwkvqNative.swift:38-60)."""
    wq: torch.Tensor
    scales: torch.Tensor
    biases: torch.Tensor
    bits: int
    outFeatures: int
    inFeatures: int
    groupSize: int = 32

    def __call__(self, x):
        return quantizedMM(x, self.wq, self.scales, self.biases, True, 32, self.bits)


def nativeAffine(qblk, qsqm, ddm, outFeatures, inFeatures, xbits, exactScales=True):
    """RwkvqSidecar.nativeAffine (RwkvqNative.swift:78-196): lossless relayout;
    scales/biases stay fp32 only where fp16 would change a weight."""
    OUT, IN, bits = outFeatures, inFeatures, 4 + xbits
    wq = torch.empty((OUT, IN // 32 * bits), device=qblk.device, dtype=torch.int32)
    sc = torch.empty((OUT, IN // 32), device=qblk.device, dtype=torch.float32)
    bi = torch.empty_like(sc)
    import ctypes
    ok = ctypes.c_int(0)
    call("rwkv_sb6_to_affine", _p(qblk), _p(qsqm), _p(ddm), _p(wq), _p(sc), _p(bi),
         ctypes.cast(ctypes.pointer(ok), ctypes.c_void_p), OUT, IN, xbits, _s())
    use_half = (not exactScales) or bool(ok.value)
    if use_half:
        sc, bi = sc.to(torch.float16), bi.to(torch.float16)
    return RwkvqNativeWeight(wq, sc, bi, bits, OUT, IN)


# ------------------------------------------------------------------------ sym

rwkvqSymGEMVMaxRows = 4  # RwkvqSymGEMV.swift:40 (kept for callers; any rows are taken)


def rwkvqDequantSym(qblk, qs, d, outFeatures, inFeatures, bits, dtype=torch.float32):
    """RwkvqDequant.swift:409-431 (and the :442-466 chain for IN % 256 != 0)."""
    out = torch.empty((outFeatures, inFeatures), device=qblk.device, dtype=dtype)
    call("rwkv_sym_dequant", _p(qblk), _p(qs), _p(d), _DT[dtype], _p(out), outFeatures,
         inFeatures, bits, _s())
    return out


def rwkvqSymGEMVApplies(outFeatures, inFeatures, bits, rows):
    """RwkvqSymGEMV.swift:213-218 without the 4-row limit."""
    return bits in (6, 8) and inFeatures % 256 == 0 and outFeatures % 16 == 0 and rows >= 1


def rwkvqSymGEMV(x, qblk, qs, d, outFeatures, inFeatures, bits):
    """RwkvqSymGEMV.swift:223-247: x [N, IN] -> [N, OUT] fp32."""
    if x.dim() != 2 or x.shape[1] != inFeatures:
        raise ValueError(f"sym-GEMV: input {tuple(x.shape)}, expected [N, {inFeatures}]")
    if not rwkvqSymGEMVApplies(outFeatures, inFeatures, bits, x.shape[0]):
        raise ValueError(f"sym-GEMV: shape {outFeatures}x{inFeatures}, bits={bits} not taken")
    x = (x if x.dtype in _DT else x.to(torch.float32)).contiguous()
    y = torch.empty((x.shape[0], outFeatures), device=x.device, dtype=torch.float32)
    call("rwkv_sym_gemv", _DT[x.dtype], _p(x), _p(qblk), _p(qs), _p(d), _p(y), x.shape[0],
         outFeatures, inFeatures, bits, outFeatures, _s())
    return y


def symGEMVFused(xstack, qblk, qs, d, outPer, inFeatures, bits):
    """K matrices in one launch (RwkvqSymGEMV.swift:343-358): xstack [K, IN] ->
    [K, outPer] fp32; the buffers are the K matrices' rows concatenated."""
    K = xstack.shape[0]
    OUT = outPer * K
    x = (xstack if xstack.dtype in _DT else xstack.to(torch.float32)).contiguous()
    y = torch.empty((1, OUT), device=x.device, dtype=torch.float32)
    call("rwkv_sym_gemv", _DT[x.dtype], _p(x), _p(qblk), _p(qs), _p(d), _p(y), 1, OUT,
         inFeatures, bits, outPer, _s())
    return y.reshape(K, outPer)


@dataclass
class RwkvqSymRowTable:
    """8-bit sym embedding rows on demand (RwkvqSymRows.swift:26-78)."""
    codes: torch.Tensor  # uint8 [rows, IN]
    qs: torch.Tensor     # uint8 [rows, IN/16]
    d: torch.Tensor      # fp16 [rows, ceil(IN/256)]
    rowCount: int
    inFeatures: int

    def rows(self, ids):
        ids32 = ids.reshape(-1).to(torch.int32).contiguous()
        out = torch.empty((ids32.numel(), self.inFeatures), device=self.codes.device,
                          dtype=torch.float16)
        call("rwkv_sym_rows", _p(ids32), ids32.numel(), _p(self.codes), _p(self.qs), _p(self.d),
             _p(out), self.rowCount, self.inFeatures, _s())
        return out.reshape(*ids.shape, self.inFeatures)

    def dense(self):
        return rwkvqDequantSym(self.codes, self.qs, self.d, self.rowCount, self.inFeatures, 8,
                               torch.float16)
