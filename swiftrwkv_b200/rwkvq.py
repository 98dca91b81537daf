"""`.rwkvq` reader: the quantised base file of the reference, read directly.

Mirrors RwkvqContainer / RwkvqSidecar(rwkvq:) (Sources/RWKVQuant/RwkvqFile.swift
:31-160, :214-492): a `.rwkvq` is a safetensors container (8-byte little-endian
header length, a JSON header, raw buffers) whose `__metadata__["rwkvq"]` holds
the JSON manifest (`format` "rwkvq", `format_version` <= 2, `naming`, and a
`tensors` table: shape, kind, bits, gw_gs, gw_sb, n_blocks per tensor); a
tensor's buffers are named "<key>::<field>".

The file is mapped (numpy memmap) and every buffer is read on its own.  The
disk layout is canonical; the kernels read the loader's interleave, built here
as a byte permutation (no arithmetic), exactly as the reference builds it:

  sb6 (block 32, superblock 8): qblk = [16 nibble bytes | 4 B qh | 4 B qh2]
      per block; qsqm = (qs, qm - 31 as a byte) per block, both unpacked from
      6-bit streams (RwkvqFile.swift:171-212); ddm = (d, dm) fp16 pairs per
      superblock -- the layout rwkv_sb6_* take;
  sym (block 16, superblock 16): 8-bit codes as bytes, or for 6 bits
      [16 nibble bytes | 4 B qh | 4 B qh2] per pair of blocks; qs int8 per
      block; d fp16 per superblock -- the layout rwkv_sym_* take;
  dense: the buffer as stored.

The `asym` and `rtn` kinds (low-rank LoRA and per-row quantisation in the
reference) have no kernels here: reading one raises, naming the tensor.
Name mapping world <-> x070 follows RwkvqNaming (RwkvqSidecar.swift:344-399).
"""
from __future__ import annotations

import json
import os

import numpy as np

MAX_FORMAT_VERSION = 2   # RwkvqSidecar.maxFormatVersion (RwkvqSidecar.swift:117)

_DTYPES = {"BOOL": np.bool_, "U8": np.uint8, "I8": np.int8, "I16": np.int16, "U16": np.uint16,
           "F16": np.float16, "BF16": np.uint16, "I32": np.int32, "U32": np.uint32,
           "F32": np.float32, "F64": np.float64, "I64": np.int64, "U64": np.uint64}

_TMIX = {"r_proj": "receptance", "k_proj": "key", "v_proj": "value", "o_proj": "output"}


class RwkvqError(ValueError):
    """A malformed or unsupported `.rwkvq` file (RwkvqError in the reference)."""


def world_key(x070_key: str):
    """x070 name -> world name, or None (RwkvqNaming.worldKey)."""
    if x070_key in ("emb.weight", "head.weight"):
        return x070_key
    p = x070_key.split(".")
    if len(p) != 5 or p[0] != "blocks" or p[4] != "weight" or not p[1].isdigit():
        return None
    if p[2] == "tmix" and p[3] in _TMIX:
        return f"blocks.{p[1]}.att.{_TMIX[p[3]]}.weight"
    if p[2] == "cmix" and p[3] in ("key", "value"):
        return f"blocks.{p[1]}.ffn.{p[3]}.weight"
    return None


def x070_key(world: str):
    """world name -> x070 name, or None (RwkvqNaming.x070Key)."""
    if world in ("emb.weight", "head.weight"):
        return world
    p = world.split(".")
    if len(p) != 5 or p[0] != "blocks" or p[4] != "weight" or not p[1].isdigit():
        return None
    if p[2] == "att":
        inv = {v: k for k, v in _TMIX.items()}
        return f"blocks.{p[1]}.tmix.{inv[p[3]]}.weight" if p[3] in inv else None
    if p[2] == "ffn" and p[3] in ("key", "value"):
        return f"blocks.{p[1]}.cmix.{p[3]}.weight"
    return None


class RwkvqContainer:
    """A safetensors container, mapped; buffers handed out one at a time."""

    def __init__(self, path: str):
        path = os.path.expanduser(path)
        if not os.path.isfile(path):
            raise RwkvqError(f"{path}: no such file")
        size = os.path.getsize(path)
        if size < 8:
            raise RwkvqError(f"{path}: shorter than a safetensors header")
        with open(path, "rb") as f:
            head = f.read(8)
            if head[:4] == b"PK\x03\x04":
                raise RwkvqError(f"{path}: a pickle container (torch.save), not safetensors")
            n = int.from_bytes(head, "little")
            if n <= 0 or n > size - 8:
                raise RwkvqError(f"{path}: header length {n} outside the file")
            header = json.loads(f.read(n))
        if not isinstance(header, dict):
            raise RwkvqError(f"{path}: the safetensors header is not an object")
        self.path, self.base = path, 8 + n
        self.metadata = header.pop("__metadata__", {}) or {}
        self.entries = {}
        for name, d in header.items():
            try:
                dt, shape, off = d["dtype"], list(d["shape"]), list(d["data_offsets"])
            except (KeyError, TypeError):
                raise RwkvqError(f"{path}: incomplete buffer record {name}") from None
            if dt not in _DTYPES:
                raise RwkvqError(f"{path}: dtype {dt} of buffer {name} is not supported")
            count = int(np.prod(shape)) if shape else 1
            if len(off) != 2 or off[0] < 0 or off[1] < off[0] or self.base + off[1] > size or \
                    off[1] - off[0] != count * np.dtype(_DTYPES[dt]).itemsize:
                raise RwkvqError(f"{path}: buffer {name}: offsets {off} disagree with shape {shape} and {dt}")
            self.entries[name] = (dt, shape, off)
        self._mm = np.memmap(path, dtype=np.uint8, mode="r")

    def names(self):
        return sorted(self.entries)

    def contains(self, name: str) -> bool:
        return name in self.entries

    def shape(self, name: str):
        e = self.entries.get(name)
        return None if e is None else list(e[1])

    def array(self, name: str):
        """The buffer as a numpy array (BF16 as raw uint16 bits)."""
        dt, shape, off = self.entries[name]
        raw = self._mm[self.base + off[0]: self.base + off[1]]
        return np.frombuffer(raw.tobytes(), dtype=_DTYPES[dt]).reshape(shape)


def unpack6x8(b):
    """6-bit stream uint8 [..., 6] -> int32 [..., 8], LSB first
    (rwkvqUnpack6x8, RwkvqFile.swift:171-183)."""
    b = np.asarray(b)
    if b.shape[-1] != 6:
        raise RwkvqError(f"unpack6: expected 6 bytes per superblock, got {b.shape[-1]}")
    x = b.astype(np.int32).reshape(b.shape[:-1] + (2, 3))
    x0, x1, x2 = x[..., 0], x[..., 1], x[..., 2]
    v = np.stack([x0 & 0x3F, ((x0 >> 6) | (x1 << 2)) & 0x3F, ((x1 >> 4) | (x2 << 4)) & 0x3F,
                  (x2 >> 2) & 0x3F], axis=-1)
    return v.reshape(b.shape[:-1] + (8,))


def sb6_to_k3(codes_packed, qsqm, d, dm, qh, qh2, shape, gs=32, sb=8):
    """sb6 disk layout -> (qblk, qsqm, ddm, xbits), the loader's interleave
    (rwkvqSb6ToK3, RwkvqFile.swift:185-212): a byte permutation."""
    OUT, IN = shape
    NB = IN // gs
    xbits = (qh is not None) + (qh2 is not None)
    parts = [np.asarray(codes_packed, np.uint8).reshape(OUT, NB, 16)]
    if qh is not None:
        parts.append(np.asarray(qh, np.uint8).reshape(OUT, NB, 4))
    if qh2 is not None:
        parts.append(np.asarray(qh2, np.uint8).reshape(OUT, NB, 4))
    qblk = np.concatenate(parts, axis=2).reshape(OUT, NB * (16 + 4 * xbits))
    q = np.asarray(qsqm, np.uint8)
    qs = unpack6x8(q[..., 0:6]).reshape(OUT, NB)
    qm = unpack6x8(q[..., 6:12]).reshape(OUT, NB)
    k3 = np.stack([qs, (qm - 31 + 256) % 256], axis=-1).astype(np.uint8).reshape(OUT, NB * 2)
    ddm = np.stack([np.asarray(d, np.float16), np.asarray(dm, np.float16)], axis=-1).reshape(OUT, (NB // sb) * 2)
    return qblk, k3, ddm.view(np.uint16), xbits


class RwkvqFile:
    """A `.rwkvq` base (RwkvqSidecar(rwkvq:)): the manifest is checked whole
    when the file opens; tensors are read on demand with `tensor(key)`."""

    def __init__(self, path: str):
        self.box = RwkvqContainer(path)
        text = self.box.metadata.get("rwkvq")
        if text is None:
            raise RwkvqError(f"{path}: not .rwkvq -- no rwkvq key in __metadata__")
        root = json.loads(text)
        if root.get("format") != "rwkvq":
            raise RwkvqError(f"{path}: format {root.get('format')}")
        version = int(root.get("format_version", 0))
        if version > MAX_FORMAT_VERSION:
            raise RwkvqError(f"{path}: format_version {version} newer than {MAX_FORMAT_VERSION}")
        tensors = root.get("tensors")
        if not isinstance(tensors, dict):
            raise RwkvqError(f'{path}: no "tensors" section')
        self.path = path
        self.naming = root.get("naming", "world")
        self.n_layer = root.get("n_layer", 0)
        self.n_embd = root.get("n_embd", 0)
        self.head_size = root.get("head_size", 64)
        self.vocab_size = root.get("vocab_size", 0)
        self.tensors = tensors
        for key in tensors:
            self._check(key)

    def keys(self):
        return sorted(self.tensors)

    def _dims(self, key, field):
        s = self.box.shape(f"{key}::{field}")
        if s is None:
            raise RwkvqError(f"{key}: missing buffer {field}")
        return s

    def _check(self, key):
        """The manifest checks of RwkvqSidecar(rwkvq:) (RwkvqFile.swift:292-459)."""
        m = self.tensors[key]
        if not isinstance(m, dict) or "shape" not in m or "kind" not in m:
            raise RwkvqError(f"{self.path}: no shape or layout for {key}")
        kind, shape, bits = m["kind"], list(m["shape"]), int(m.get("bits", 16))
        gs, sb = int(m.get("gw_gs", 0)), int(m.get("gw_sb", 0))
        nb = int(m.get("n_blocks", 0))
        if kind == "dense":
            self._dims(key, "dense")
        elif kind == "sb6":
            if len(shape) != 2 or gs != 32 or sb != 8 or shape[1] % (gs * sb):
                raise RwkvqError(f"{key}: sb6 needs block 32 and superblock 8 (gw_gs={gs}, gw_sb={sb}, shape {shape})")
            if nb > 0 and nb != shape[1] // gs:
                raise RwkvqError(f"{key}: sb6 covers {shape[1] // gs} blocks, the manifest says {nb}")
            want = [shape[0], shape[1] // (gs * sb), 12]
            if self._dims(key, "gw_qsqm") != want:
                raise RwkvqError(f"{key}: gw_qsqm {self._dims(key, 'gw_qsqm')}, expected {want}")
            for f in ("codes_packed", "gw_d", "gw_dm"):
                self._dims(key, f)
            xbits = self.box.contains(f"{key}::gw_qh") + self.box.contains(f"{key}::gw_qh2")
            if bits != 4 + xbits:
                raise RwkvqError(f"{key}: bits={bits}, but the file has {xbits} bit planes")
        elif kind == "sym":
            if len(shape) != 2 or gs != 16 or sb != 16:
                raise RwkvqError(f"{key}: sym needs block 16 and superblock 16 (gw_gs={gs}, gw_sb={sb})")
            OUT, IN = shape
            if IN % gs:
                raise RwkvqError(f"{key}: sym, IN={IN} is not a multiple of 16")
            qs, d = self._dims(key, "gw_qs"), self._dims(key, "gw_d")
            if nb > 0 and nb != qs[-1]:
                raise RwkvqError(f"{key}: gw_qs covers {qs[-1]} blocks, the manifest says {nb}")
            if qs != [OUT, IN // gs] or len(d) != 2 or d[1] * sb != IN // gs:
                raise RwkvqError(f"{key}: gw_qs {qs} / gw_d {d} do not fit {shape}")
            if self.box.contains(f"{key}::codes"):
                if bits != 8:
                    raise RwkvqError(f"{key}: sym with an 8-bit codes buffer at bits={bits}")
            else:
                if bits != 6 or IN % 32:
                    raise RwkvqError(f"{key}: sym with codes_packed at bits={bits}, IN={IN}")
                for f in ("codes_packed", "gw_qh", "gw_qh2"):
                    self._dims(key, f)
        elif kind in ("asym", "rtn"):
            pass  # checked when read: no kernels take these here
        else:
            raise RwkvqError(f"unknown layout {kind} of {key}")

    def info(self, key: str) -> dict:
        return dict(self.tensors[key])

    def tensor(self, key: str) -> dict:
        """The tensor's buffers in the loader's layout, as numpy arrays:
        sb6 -> {kind, shape, xbits, qblk, qsqm, ddm}; sym -> {kind, shape,
        bits, qblk, qs, d}; dense -> {kind, shape, dense}."""
        m = self.tensors[key]
        kind, shape = m["kind"], list(m["shape"])
        a = lambda f: self.box.array(f"{key}::{f}")
        if kind == "dense":
            return {"kind": kind, "shape": shape, "dense": a("dense")}
        if kind == "sb6":
            qh = a("gw_qh") if self.box.contains(f"{key}::gw_qh") else None
            qh2 = a("gw_qh2") if self.box.contains(f"{key}::gw_qh2") else None
            qblk, qsqm, ddm, xbits = sb6_to_k3(a("codes_packed"), a("gw_qsqm"), a("gw_d").view(np.float16),
                                               a("gw_dm").view(np.float16), qh, qh2, shape,
                                               int(m["gw_gs"]), int(m["gw_sb"]))
            return {"kind": kind, "shape": shape, "xbits": xbits, "qblk": qblk, "qsqm": qsqm, "ddm": ddm}
        if kind == "sym":
            OUT, IN = shape
            if self.box.contains(f"{key}::codes"):
                qblk, bits = a("codes").view(np.uint8).reshape(OUT, IN), 8
            else:
                NP = IN // 32
                qblk = np.concatenate([a("codes_packed").reshape(OUT, NP, 16), a("gw_qh").reshape(OUT, NP, 4),
                                       a("gw_qh2").reshape(OUT, NP, 4)], axis=2).reshape(OUT, NP * 24)
                bits = 6
            return {"kind": kind, "shape": shape, "bits": bits, "qblk": np.ascontiguousarray(qblk, np.uint8),
                    "qs": a("gw_qs").view(np.uint8).reshape(OUT, IN // 16), "d": a("gw_d").view(np.uint16)}
        raise RwkvqError(f"{key}: layout {kind} has no kernel here (sb6, sym and dense are read)")

    def dequantize(self, key: str, dtype=None):
        """The dense weight [OUT, IN] on the GPU (rwkv_sb6_dequant /
        rwkv_sym_dequant; dense buffers as stored), default fp32."""
        import torch
        from . import quant as Q
        t = self.tensor(key)
        dtype = dtype or torch.float32
        dev = lambda x: torch.from_numpy(np.array(x, copy=True)).cuda()
        if t["kind"] == "dense":
            d = t["dense"]
            dt = self.box.entries[f"{key}::dense"][0]
            if dt == "BF16":
                w = torch.from_numpy(d.astype(np.int16)).view(torch.bfloat16)
            else:
                w = torch.from_numpy(np.asarray(d))
            return w.to("cuda", dtype)
        OUT, IN = t["shape"]
        if t["kind"] == "sb6":
            return Q.rwkvqDequantDense(dev(t["qblk"]), dev(t["qsqm"]), dev(t["ddm"].view(np.float16)), OUT, IN, 8,
                                       t["xbits"], dtype=dtype)
        return Q.rwkvqDequantSym(dev(t["qblk"]), dev(t["qs"]), dev(t["d"].view(np.float16)), OUT, IN, t["bits"],
                                 dtype=dtype)
