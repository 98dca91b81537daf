"""Writer of `.rwkvq` test files -- TEST INFRASTRUCTURE.

The reference's writer (rwkv-quant, formats/codec.py) is not part of the
reference tree.  This writes the container the reader expects
(RwkvqFile.swift:31-160, :214-459): a safetensors file whose
`__metadata__["rwkvq"]` is the manifest, buffers "<key>::<field>" in the
canonical disk layout -- which is the inverse of the loader's byte
permutation (sb6: 6-bit packed qs / qm streams, qm stored without the -31
shift, codes and bit planes in separate buffers; sym 6-bit: nibble bytes and
bit planes separate).  Round trips through swiftrwkv_b200.rwkvq check that the
reader rebuilds the loader layout byte for byte.
"""
from __future__ import annotations

import json
import struct

import numpy as np


def pack6x8(v):
    """int [..., 8] values 0..63 -> uint8 [..., 6], LSB first (inverse of unpack6x8)."""
    v = np.asarray(v, np.int64).reshape(np.shape(v)[:-1] + (2, 4))
    v0, v1, v2, v3 = (v[..., i] for i in range(4))
    x0 = (v0 | (v1 << 6)) & 0xFF
    x1 = ((v1 >> 2) | (v2 << 4)) & 0xFF
    x2 = ((v2 >> 4) | (v3 << 2)) & 0xFF
    return np.stack([x0, x1, x2], axis=-1).astype(np.uint8).reshape(np.shape(v)[:-2] + (6,))


def sb6_disk(qblk, qsqm, ddm, OUT, IN, xbits):
    """Loader layout (K3) -> disk buffers of one sb6 tensor."""
    NB, NSB = IN // 32, IN // 256
    BB = 16 + 4 * xbits
    q = np.asarray(qblk, np.uint8).reshape(OUT, NB, BB)
    out = {"codes_packed": q[:, :, :16].reshape(OUT, NB * 16)}
    if xbits >= 1:
        out["gw_qh"] = q[:, :, 16:20].reshape(OUT, NB * 4)
    if xbits >= 2:
        out["gw_qh2"] = q[:, :, 20:24].reshape(OUT, NB * 4)
    k3 = np.asarray(qsqm, np.uint8).reshape(OUT, NB, 2)
    qs = k3[:, :, 0].astype(np.int64).reshape(OUT, NSB, 8)
    qm = ((k3[:, :, 1].astype(np.int64) + 31) % 256).reshape(OUT, NSB, 8)
    out["gw_qsqm"] = np.concatenate([pack6x8(qs), pack6x8(qm)], axis=-1)
    dd = np.asarray(ddm, np.uint16).reshape(OUT, NSB, 2)
    out["gw_d"] = dd[:, :, 0].view(np.float16)
    out["gw_dm"] = dd[:, :, 1].view(np.float16)
    return out


def sym_disk(qblk, qs, d, OUT, IN, bits):
    out = {"gw_qs": np.asarray(qs, np.uint8).view(np.int8).reshape(OUT, IN // 16),
           "gw_d": np.asarray(d, np.uint16).view(np.float16).reshape(OUT, -1)}
    if bits == 8:
        out["codes"] = np.asarray(qblk, np.uint8).view(np.int8).reshape(OUT, IN)
    else:
        NP = IN // 32
        q = np.asarray(qblk, np.uint8).reshape(OUT, NP, 24)
        out["codes_packed"] = q[:, :, :16].reshape(OUT, NP * 16)
        out["gw_qh"] = q[:, :, 16:20].reshape(OUT, NP * 4)
        out["gw_qh2"] = q[:, :, 20:24].reshape(OUT, NP * 4)
    return out


_ST = {np.dtype(np.uint8): "U8", np.dtype(np.int8): "I8", np.dtype(np.float16): "F16",
       np.dtype(np.float32): "F32", np.dtype(np.uint16): "U16", np.dtype(np.int32): "I32"}


def write_rwkvq(path, tensors: dict, naming="world", format_version=2, extra_meta=None, **root):
    """tensors: key -> (manifest entry dict, {field: ndarray}).  Writes the
    safetensors container with the manifest in __metadata__["rwkvq"]."""
    manifest = {"format": "rwkvq", "format_version": format_version, "naming": naming,
                "tensors": {k: m for k, (m, _) in tensors.items()}, **root}
    header, blobs, off = {}, [], 0
    for k, (_, bufs) in tensors.items():
        for field, a in bufs.items():
            a = np.ascontiguousarray(a)
            raw = a.tobytes()
            header[f"{k}::{field}"] = {"dtype": _ST[a.dtype], "shape": list(a.shape),
                                       "data_offsets": [off, off + len(raw)]}
            blobs.append(raw)
            off += len(raw)
    meta = {"rwkvq": json.dumps(manifest)}
    meta.update(extra_meta or {})
    header["__metadata__"] = meta
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
