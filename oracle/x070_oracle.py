"""x070 recurrent decode, CPU restatement -- TEST INFRASTRUCTURE ONLY.

Restates the one-token step of Sources/RWKVGen/X070Generation.swift
(stepEager :483-498, tmixStep :201-307, cmixStep :310-319) with the manual
fp32 LayerNorm (:503-511), l2norm (:500-502) and the wkv7 step / tail of
rwkv_oracle.c, over weights whose big matrices are quantised to the MLX
affine container by the restated quantiser and used dequantised.  Matmul
inputs are rounded to the activation dtype (fp16 or fp32) before the product,
as the CUDA runtime feeds its GEMVs; products and sums run in float64.

Also holds the fixture generators: `tiny_weights` mirrors the reference's
TinyBackbone (Tests/RWKVGenTests/TinyBackbone.swift:37-111) with numpy's
PCG64 instead of MLXRandom, and `splitmix_ids` is its SplitMix64 id stream
(:120-136), bit for bit.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O

QUANT_TARGETS = ("r_proj", "k_proj", "v_proj", "o_proj", "cmix.key", "cmix.value", "head", "emb")


def lora_ranks(D: int):
    """x070 low-rank sizes (X070Init.swift:46-52, rwkvMetal formula)."""
    def f(c, p):
        return max(32, int(np.floor(c * D ** p / 32 + 0.5)) * 32)
    return {"w": f(1.8, 0.5), "a": f(1.8, 0.5), "v": f(1.3, 0.5), "g": f(0.6, 0.8)}


class Cfg:
    def __init__(self, n_layer, n_embd, vocab, head_size=64, ffn=None):
        self.n_layer, self.n_embd, self.vocab, self.head_size = n_layer, n_embd, vocab, head_size
        self.n_head = n_embd // head_size
        self.ffn = ffn or 4 * n_embd
        self.ranks = lora_ranks(n_embd)


def tiny_weights(cfg: Cfg, seed: int = 42, fan_in_scale: bool = False):
    """Random weights on the TinyBackbone recipe (all matrices non-zero).

    TinyBackbone draws every matrix with std 0.05, which suits its width
    (D = 128 .. 256).  fan_in_scale=True keeps that conditioning at any width:
    a matrix's std becomes 0.05 * sqrt(256 / fan_in), so projections keep
    unit gain at D = 2048 as they do at D = 256."""
    rng = np.random.default_rng(seed)
    D, H, S, V, F = cfg.n_embd, cfg.n_head, cfg.head_size, cfg.vocab, cfg.ffn
    r = cfg.ranks

    def n(shape, scale=0.05):
        if fan_in_scale and np.ndim(shape) == 1 and len(shape) == 2 and scale == 0.05:
            scale = 0.05 * np.sqrt(256.0 / shape[1])
        return (rng.standard_normal(shape) * scale).astype(np.float32)

    w = {"emb.weight": n((V, D), 0.1), "ln0.weight": np.ones(D, np.float32),
         "ln0.bias": np.zeros(D, np.float32), "ln_out.weight": np.ones(D, np.float32),
         "ln_out.bias": np.zeros(D, np.float32), "head.weight": n((V, D), 0.1)}
    for i in range(cfg.n_layer):
        bp = f"blocks.{i}."
        for ln in ("ln1", "ln2"):
            w[bp + ln + ".weight"] = np.ones(D, np.float32)
            w[bp + ln + ".bias"] = np.zeros(D, np.float32)
        tp = bp + "tmix."
        for name in ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g"):
            w[tp + name] = n(D, 0.3) + 0.5
        w[tp + "k_k"] = np.ones((H, S), np.float32) + n((H, S), 0.1)
        w[tp + "k_a"] = n((H, S), 0.1)
        w[tp + "r_k"] = n((H, S), 0.1)
        for name in ("w", "a", "g"):
            w[tp + f"{name}_lora_A.weight"] = n((r[name], D))
            w[tp + f"{name}_lora_B.weight"] = n((D, r[name]))
        w[tp + "w_lora_B.bias"] = n(D, 0.1)
        w[tp + "a_lora_B.bias"] = n(D, 0.1)
        if i > 0:
            w[tp + "v_lora_A.weight"] = n((r["v"], D))
            w[tp + "v_lora_B.weight"] = n((D, r["v"]))
            w[tp + "v_lora_B.bias"] = n(D, 0.1)
        for name in ("r_proj", "k_proj", "v_proj", "o_proj"):
            w[tp + name + ".weight"] = n((D, D))
        w[tp + "ln_x.weight"] = np.ones(D, np.float32)
        w[tp + "ln_x.bias"] = np.zeros(D, np.float32)
        cp = bp + "cmix."
        w[cp + "x_k"] = n(D, 0.3) + 0.5
        w[cp + "key.weight"] = n((F, D))
        w[cp + "value.weight"] = n((D, F))
    return w


def to_bf16(x):
    """Round float32 values to bfloat16 (nearest, ties to even), as float32."""
    u = np.ascontiguousarray(np.asarray(x, np.float32)).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return r.astype(np.uint32).view(np.float32)


def splitmix_ids(B, T, vocab=64, seed=1):
    """TinyBackbone.ids: SplitMix64 stream, ids = next() % vocab, [B, T] int32."""
    mask = (1 << 64) - 1
    state = (seed * 0x2545F4914F6CDD1D + 0x9E3779B9) & mask
    out = []
    for _ in range(B * T):
        state = (state + 0x9E3779B97F4A7C15) & mask
        z = state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & mask
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & mask
        z = z ^ (z >> 31)
        out.append(z % vocab)
    return np.array(out, np.int32).reshape(B, T)


def _is_quant(name):
    stem = name[:-len(".weight")] if name.endswith(".weight") else name
    return any(stem == t or stem.endswith("." + t) for t in QUANT_TARGETS)


class X070Oracle:
    """Recurrent decode for `rows` independent rows."""

    # fp16 activations and more rows than this: the quantised projections are
    # products with the weight dequantised INTO fp16 (MLX's quantized matmul,
    # which the runtime's tensor-core path follows); up to it, with the exact
    # dequantised weight (MLX's quantized matrix-vector product).
    GEMV_MAX_ROWS = 8

    def __init__(self, cfg: Cfg, weights: dict, act="f16", quant_bits=4, group=64, exact=None):
        """quant_bits 4: the big matrices in the 4-bit container (used
        dequantised); quant_bits 0: a dense bf16 base.  The low-rank and
        adapter matrices are stored fp16, or bf16 with a bf16 model (the
        runtime's storage).  exact: {name: fp32 [OUT, IN]} matrices used as
        given at every row count -- the dequantised .rwkvq sb6 / sym matrices,
        whose GEMVs (RwkvqSb6GEMV.swift:103-145, RwkvqSymGEMV.swift:100-199)
        multiply the exact dequantised weight."""
        self.cfg, self.act = cfg, act
        self.w = {}
        self.w16 = {}
        lr_bf16 = act == "bf16" or (quant_bits == 0 and act != "f16")
        for k, v in weights.items():
            v = np.asarray(v, np.float32)
            if quant_bits and v.ndim == 2 and _is_quant(k):
                v16 = v.astype(np.float16).astype(np.float32)
                wq, sc, bi = O.affine_quantize(v16, group, quant_bits)
                v = O.affine_dequant(wq, sc, bi, group, quant_bits)
                if act == "f16" and k != "emb.weight":
                    self.w16[k] = v.astype(np.float16).astype(np.float64)
            elif not quant_bits and v.ndim == 2 and _is_quant(k):
                v = to_bf16(v)          # dense bf16 base
            elif v.ndim == 2:          # dense low-rank branches: 16-bit storage
                v = to_bf16(v) if lr_bf16 else v.astype(np.float16).astype(np.float32)
            self.w[k] = v.astype(np.float64)
        for k, v in (exact or {}).items():
            self.w[k] = np.asarray(v, np.float32).astype(np.float64)
            self.w16.pop(k, None)

    def new_state(self, rows):
        c = self.cfg
        return {"wkv": np.zeros((c.n_layer, rows, c.n_head, c.head_size, c.head_size), np.float32),
                "tshift": np.zeros((c.n_layer, rows, c.n_embd), np.float64),
                "cshift": np.zeros((c.n_layer, rows, c.n_embd), np.float64)}

    def _a(self, x):
        """Round a matmul input to the activation dtype."""
        if self.act == "f16":
            return x.astype(np.float16).astype(np.float64)
        if self.act == "bf16":
            return to_bf16(x).astype(np.float64)
        return x.astype(np.float32).astype(np.float64)

    def _mm(self, x, key):
        w = self.w16.get(key) if x.shape[0] > self.GEMV_MAX_ROWS else None
        return self._a(x) @ (self.w[key] if w is None else w).T

    def _proj(self, x, key):
        """Projection with its optional LoRA adapter (X070Backbone.swift:746-752):
        base + scale * (x A^T) B^T, adapter keys "<target>.lora_a" / ".lora_b" /
        ".lora_scale" (LoRA.swift:118-127).  A and B are stored in fp16 like the
        other dense matrices; z = scale * (x A^T) is rounded to the activation
        type, where the runtime stores it."""
        y = self._mm(x, key)
        stem = key[:-len(".weight")]
        A, B = self.w.get(stem + ".lora_a"), self.w.get(stem + ".lora_b")
        if A is None or B is None:
            return y
        scale = float(np.asarray(self.w.get(stem + ".lora_scale", 1.0)).reshape(-1)[0])
        z = self._a(scale * (self._a(x) @ A.T))
        return y + z @ B.T

    @staticmethod
    def _ln(x, w, b, eps=1e-5):
        mean = x.mean(-1, keepdims=True)
        var = ((x - mean) ** 2).mean(-1, keepdims=True)
        return (x - mean) / np.sqrt(var + eps) * w + b

    def step(self, ids, st):
        """One token per row: ids [rows] -> logits [rows, vocab] (float64)."""
        c, W = self.cfg, self.w
        H, S, D = c.n_head, c.head_size, c.n_embd
        rows = len(ids)
        x = self._ln(W["emb.weight"][ids], W["ln0.weight"], W["ln0.bias"])
        v_first = None
        sig = lambda z: 1.0 / (1.0 + np.exp(-z))
        for L in range(c.n_layer):
            p = f"blocks.{L}.tmix."
            xl = self._ln(x, W[f"blocks.{L}.ln1.weight"], W[f"blocks.{L}.ln1.bias"])
            xx = st["tshift"][L] - xl
            st["tshift"][L] = xl
            mix = {m: xl + xx * W[p + "x_" + m] for m in "rwkvag"}
            r = self._proj(mix["r"], p + "r_proj.weight")
            k = self._proj(mix["k"], p + "k_proj.weight")
            v = self._proj(mix["v"], p + "v_proj.weight")
            gate = self._mm(sig(self._mm(mix["g"], p + "g_lora_A.weight")), p + "g_lora_B.weight")
            if L == 0:
                v_first = v.copy()
            else:
                vv = sig(self._mm(self._mm(mix["v"], p + "v_lora_A.weight"), p + "v_lora_B.weight")
                         + W[p + "v_lora_B.bias"])
                v = v + (v_first - v) * vv
            a = sig(self._mm(self._mm(mix["a"], p + "a_lora_A.weight"), p + "a_lora_B.weight")
                    + W[p + "a_lora_B.bias"])
            ww = self._mm(np.tanh(self._mm(mix["w"], p + "w_lora_A.weight")), p + "w_lora_B.weight") \
                + W[p + "w_lora_B.bias"]
            w_dec = np.exp(-0.606531 * sig(ww))
            kk = (k * W[p + "k_k"].reshape(D)).reshape(rows, H, S)
            kk = kk / np.sqrt((kk * kk).sum(-1, keepdims=True) + 1e-12)
            k2 = k * (1.0 + (a - 1.0) * W[p + "k_a"].reshape(D))
            kk = kk.reshape(rows, D)
            f32 = lambda t: t.reshape(rows, H, S).astype(np.float32)
            y, h = O.wkv7_step(f32(r), f32(w_dec), f32(k2), f32(v), f32(-kk), f32(kk * a),
                               st["wkv"][L])
            st["wkv"][L] = h
            tail = O.wkv_tail(y.reshape(rows, D), r.astype(np.float32), k2.astype(np.float32),
                              v.astype(np.float32), W[p + "r_k"].reshape(D), W[p + "ln_x.weight"],
                              W[p + "ln_x.bias"], gate.astype(np.float32), H, S).astype(np.float64)
            x = x + self._proj(tail, p + "o_proj.weight")
            cp = f"blocks.{L}.cmix."
            xl2 = self._ln(x, W[f"blocks.{L}.ln2.weight"], W[f"blocks.{L}.ln2.bias"])
            xx2 = st["cshift"][L] - xl2
            st["cshift"][L] = xl2
            xk = xl2 + xx2 * W[cp + "x_k"]
            hk = np.maximum(self._proj(xk, cp + "key.weight"), 0.0)
            x = x + self._proj(hk * hk, cp + "value.weight")
        xo = self._ln(x, W["ln_out.weight"], W["ln_out.bias"])
        return self._proj(xo, "head.weight")
