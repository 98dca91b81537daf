"""Host mirror of X070Config / X070Backbone's decode API over the C runtime.

`X070Backbone.step` / `generate` / `generateBatch` keep the reference's names
(Sources/RWKVGen/X070Generation.swift:449-498, Generate.swift:112-202,
BatchGenerate.swift:69-116); the model, its state and every kernel live in
librwkvcuda (rwkv_x070_*).  torch only provides device buffers and the stream.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import BF16, F16, F32, call


def _native_matrix(key: str) -> bool:
    """Base matrices a .rwkvq sb6 / sym tensor can stay native for."""
    if key == "head.weight":
        return True
    parts = key.split(".")
    return len(parts) >= 4 and parts[0] == "blocks" and ".".join(parts[2:]) in (
        "tmix.r_proj.weight", "tmix.k_proj.weight", "tmix.v_proj.weight", "tmix.o_proj.weight",
        "cmix.key.weight", "cmix.value.weight")


def lora_ranks(D: int):
    """x070 low-rank sizes, rwkvMetal formula (X070Init.swift:46-52)."""
    def f(c, p):
        return max(32, int(np.floor(c * D ** p / 32 + 0.5)) * 32)
    return {"w": f(1.8, 0.5), "a": f(1.8, 0.5), "v": f(1.3, 0.5), "g": f(0.6, 0.8)}


@dataclass
class X070Config:
    """X070Backbone.swift:24-37."""
    nLayer: int
    nEmbd: int
    vocab: int
    headSize: int = 64
    ffnMultiplier: float = 4.0

    @property
    def nHead(self):
        return self.nEmbd // self.headSize

    @property
    def ffn(self):
        return int(self.nEmbd * self.ffnMultiplier / 32) * 32


class _Cfg(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "n_layer", "n_embd", "head_size", "vocab", "ffn", "rank_w", "rank_a", "rank_v", "rank_g",
        "quant_bits", "quant_group", "act_dtype", "max_rows")]


class X070Backbone:
    """x070 model, decoded recurrently and prefilled in parallel.

    base="q4": a 4-bit group-64 QLoRA base (LoRA.swift:28-91); act="f16"
    feeds the projections fp16 activations (tensor-core GEMMs), act="f32"
    keeps activations fp32 end to end (the parity path).
    base="bf16": a dense bf16 base (the reference's bf16 model, BASELINE
    config 3); act="bf16" (tensor-core GEMMs) or "f32"."""

    def __init__(self, cfg: X070Config, max_rows: int = 1, act: str = "f16", base: str = "q4"):
        self.cfg = cfg
        if base not in ("q4", "bf16"):
            raise ValueError(f"base {base!r}: 'q4' or 'bf16'")
        r = lora_ranks(cfg.nEmbd)
        adt = {"f16": F16, "f32": F32, "bf16": BF16}[act]
        c = _Cfg(cfg.nLayer, cfg.nEmbd, cfg.headSize, cfg.vocab, cfg.ffn, r["w"], r["a"], r["v"],
                 r["g"], 4 if base == "q4" else 0, 64, adt, max_rows)
        h = ctypes.c_void_p()
        call("rwkv_x070_create", ctypes.byref(c), ctypes.byref(h))
        self.h = h
        self.max_rows = max_rows
        self.ranks = r

    def close(self):
        if self.h:
            _lib.lib().rwkv_x070_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---------------------------------------------------------------- weights
    def load(self, weights: dict):
        """Reference-named weights (numpy / torch, any float dtype)."""
        for name, v in weights.items():
            a = np.ascontiguousarray(np.asarray(v.cpu() if torch.is_tensor(v) else v, np.float32))
            call("rwkv_x070_set_param", self.h, name.encode(), a.ctypes.data_as(ctypes.c_void_p),
                 a.size)
        return self

    def load_rwkvq(self, path: str, weights: dict | None = None, native: bool = True):
        """The projection matrices, embedding and head found in a `.rwkvq`
        file (swiftrwkv_b200.rwkvq; world names mapped as RwkvqNaming does).
        With `native`, sb6 and sym projection / head matrices are kept as
        stored (rwkv_x070_set_param_rwkvq: the step runs them through the
        sb6 / sym GEMV kernels, as the reference's decode does); the others --
        and every matrix without `native` -- are dequantised on the GPU by the
        reference's dequant arithmetic (RwkvqDequant.swift) into this model's
        base: rounded once into bf16 for the dense base, re-quantised into
        the 4-bit container otherwise (lossy: sb6 / sym are not 4-bit group
        64).  `weights` (reference names) is loaded first and supplies the
        rest of the model; the file's tensors take precedence.  Returns the
        x070 names loaded."""
        from .rwkvq import RwkvqFile, x070_key
        f = RwkvqFile(path)
        if weights:
            self.load(weights)
        done = []
        for wk in f.keys():
            key = x070_key(wk) if f.naming == "world" else wk
            if key is None:
                continue
            kind = f.info(wk)["kind"]
            if native and kind in ("sb6", "sym") and _native_matrix(key) and f.info(wk)["shape"][1] % 256 == 0:
                t = f.tensor(wk)
                if kind == "sb6":
                    bufs, fmt, bits = (t["qblk"], t["qsqm"], t["ddm"]), 1, int(t["xbits"])
                else:
                    bufs, fmt, bits = (t["qblk"], t["qs"], t["d"]), 2, int(t["bits"])
                bufs = [np.ascontiguousarray(b) for b in bufs]
                args = []
                for b in bufs:
                    args += [b.ctypes.data_as(ctypes.c_void_p), b.nbytes]
                call("rwkv_x070_set_param_rwkvq", self.h, key.encode(), fmt, bits, *args)
            else:
                w = f.dequantize(wk, torch.float32).cpu().numpy()
                call("rwkv_x070_set_param", self.h, key.encode(), w.ctypes.data_as(ctypes.c_void_p), w.size)
            done.append(key)
        return done

    def init_random(self, seed: int = 0):
        """Device-side random init with the x070 recipe (X070Init.weights)."""
        call("rwkv_x070_init_random", self.h, ctypes.c_uint64(seed))
        return self

    @property
    def weight_bytes(self) -> int:
        return int(_lib.lib().rwkv_x070_weight_bytes(self.h))

    @property
    def launches_per_step(self) -> int:
        return int(_lib.lib().rwkv_x070_launches_per_step(self.h))

    def set_decode_path(self, path: int):
        """0: one captured graph of per-op launches per step (default);
        1: the persistent one-launch step where it applies (1..64 rows, fp16
        activations, 4-bit base, no adapters or .rwkvq matrices), the per-op
        graph elsewhere."""
        call("rwkv_x070_set_decode_path", self.h, int(path))
        return self

    def decode_path(self, rows: int) -> int:
        """The path a step of `rows` rows takes now (0 or 1)."""
        return int(_lib.lib().rwkv_x070_decode_path(self.h, rows))

    # ----------------------------------------------------------------- decode
    @staticmethod
    def _s():
        return _lib.P(torch.cuda.current_stream().cuda_stream)

    def reset(self, rows: int):
        """Fresh (zero) state for rows 0..rows-1."""
        call("rwkv_x070_reset_state", self.h, rows, self._s())

    def step(self, ids, use_graph: bool = False):
        """One token per row (ids: int tensor [rows]) -> logits [rows, vocab] fp32.
        The state advances in place (X070Backbone.step(_:state:))."""
        ids = torch.as_tensor(ids, dtype=torch.int32, device="cuda").reshape(-1).contiguous()
        rows = ids.numel()
        logits = torch.empty((rows, self.cfg.vocab), device="cuda", dtype=torch.float32)
        call("rwkv_x070_step", self.h, _lib.P(ids.data_ptr()), rows, _lib.P(logits.data_ptr()),
             None, int(use_graph), self._s())
        return logits

    def step_greedy(self, rows: int, ids=None, use_graph: bool = True, next_ids=None):
        """Device-resident greedy loop: feeds `ids` (or the previous argmax);
        the argmax of this step also goes to `next_ids` (device int32 [rows])
        when given."""
        p = None
        if ids is not None:
            ids = torch.as_tensor(ids, dtype=torch.int32, device="cuda").reshape(-1).contiguous()
            p = _lib.P(ids.data_ptr())
        q = None
        if next_ids is not None:
            if next_ids.dtype != torch.int32 or not next_ids.is_cuda or not next_ids.is_contiguous() \
                    or next_ids.numel() < rows:
                raise ValueError("next_ids must be a contiguous device int32 tensor of >= rows elements")
            q = _lib.P(next_ids.data_ptr())
        call("rwkv_x070_step", self.h, p, rows, None, q, int(use_graph), self._s())

    def profile_step(self, rows: int):
        """One eager step with per-launch device times: {kernel: (launches, ms)}
        plus the ordered list [(name, ms)].  The state advances as in step()."""
        cap = 4096
        ms = (ctypes.c_float * cap)()
        names = ctypes.create_string_buffer(cap * 24)
        n = ctypes.c_int(0)
        call("rwkv_x070_profile_step", self.h, rows, ctypes.cast(ms, ctypes.c_void_p), cap,
             ctypes.cast(names, ctypes.c_void_p), len(names), ctypes.byref(n), self._s())
        seq = list(zip(names.value.decode().split("\n"), ms[:n.value]))
        agg = {}
        for name, t in seq:
            c, tot = agg.get(name, (0, 0.0))
            agg[name] = (c + 1, tot + t)
        return agg, seq

    def prefill(self, ids, lengths=None, logits: bool = True):
        """Parallel prefill of right-padded prompts (prefillBatch over
        bodyWithState, BatchGenerate.swift:36-51): ids int [rows, T] (device
        or host), lengths int [rows] (None: all T).  Continues from the rows'
        current state; returns the logits [rows, vocab] of each row's last
        real token (or None), whose argmax becomes the next step's input."""
        ids = torch.as_tensor(ids, dtype=torch.int32).to("cuda").contiguous()
        rows, T = ids.shape
        lens = None
        if lengths is not None:
            lens = np.ascontiguousarray(np.asarray(lengths, np.int32))
            if lens.shape != (rows,):
                raise ValueError(f"lengths must be [{rows}]")
        out = torch.empty((rows, self.cfg.vocab), device="cuda", dtype=torch.float32) if logits else None
        call("rwkv_x070_prefill", self.h, _lib.P(ids.data_ptr()),
             None if lens is None else lens.ctypes.data_as(ctypes.c_void_p), rows, T,
             None if out is None else _lib.P(out.data_ptr()), None, self._s())
        return out

    def generateBatch(self, prompts, n_new: int, stopTokens=()):
        """Greedy generation, host in / host out (BatchGenerate.swift:69-116).
        prompts: int [rows, T] (equal lengths) -> int32 [rows, n_new], or a
        list of token lists (ragged, right-padded internally) -> a list of
        token lists, each ending at its first stop token (kept) or after
        n_new tokens; stopped rows leave the batch.  State starts from zero."""
        ragged = not isinstance(prompts, np.ndarray) and (
            len(prompts) > 0 and not np.isscalar(prompts[0]) and len({len(p) for p in prompts}) > 1)
        if not ragged and not stopTokens:
            p = np.ascontiguousarray(np.asarray(prompts, np.int32))
            rows, T = p.shape
            self.reset(rows)
            out = np.zeros((rows, n_new), np.int32)
            call("rwkv_x070_generate", self.h, p.ctypes.data_as(ctypes.c_void_p), rows, T, n_new,
                 out.ctypes.data_as(ctypes.c_void_p), self._s())
            return out
        rows = len(prompts)
        lens = np.array([len(p) for p in prompts], np.int32)
        if rows == 0 or lens.min() < 1:
            raise ValueError("generateBatch: every prompt needs at least one token")
        T = int(lens.max())
        p = np.zeros((rows, T), np.int32)
        for i, q in enumerate(prompts):
            p[i, :len(q)] = q
        stops = np.ascontiguousarray(np.asarray(list(stopTokens), np.int32))
        out = np.zeros((rows, max(n_new, 1)), np.int32)
        cnt = np.zeros(rows, np.int32)
        call("rwkv_x070_generate_batch", self.h, p.ctypes.data_as(ctypes.c_void_p),
             lens.ctypes.data_as(ctypes.c_void_p), rows, T, n_new,
             stops.ctypes.data_as(ctypes.c_void_p) if stops.size else None, int(stops.size),
             out.ctypes.data_as(ctypes.c_void_p), cnt.ctypes.data_as(ctypes.c_void_p), self._s())
        return [list(out[i, :cnt[i]]) for i in range(rows)]

    def generate(self, prompt, n_new: int):
        """Single-row greedy generation (Generate.swift:112-202, argmax sampler)."""
        return self.generateBatch(np.asarray(prompt, np.int32).reshape(1, -1), n_new)[0]
