"""The `.rwkvq` reader (swiftrwkv_b200.rwkvq) on files written in the
canonical disk layout: the loader's byte layout is rebuilt exactly (sb6 K3
interleave with the 6-bit qs / qm streams and the -31 shift, sym 6- and
8-bit), the manifest checks of the reference reject malformed files
(RwkvqFile.swift:52-110, :262-459), names map world <-> x070
(RwkvqSidecar.swift:344-399).  CPU only; the GPU side is in
test_rwkvq_gpu.py."""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

from rwkvq_fixture import pack6x8, sb6_disk, sym_disk, write_rwkvq
from swiftrwkv_b200 import rwkvq as RQ


def _sb6(rng, OUT, IN, xbits):
    from test_quant_gpu import make_sb6
    return make_sb6(rng, OUT, IN, xbits)


def _sym(rng, OUT, IN, bits):
    from test_quant_gpu import make_sym
    return make_sym(rng, OUT, IN, bits)


def test_unpack6_inverts_pack6(rng):
    v = rng.integers(0, 64, (5, 3, 8))
    assert np.array_equal(RQ.unpack6x8(pack6x8(v)), v)


@pytest.mark.parametrize("xbits", [0, 1, 2])
def test_sb6_round_trip_rebuilds_the_loader_layout(tmp_path, rng, xbits):
    OUT, IN = 48, 512
    qblk, qsqm, ddm = _sb6(rng, OUT, IN, xbits)
    p = tmp_path / "m.rwkvq"
    m = {"shape": [OUT, IN], "kind": "sb6", "bits": 4 + xbits, "gw_gs": 32, "gw_sb": 8, "n_blocks": IN // 32}
    write_rwkvq(p, {"blocks.0.att.receptance.weight": (m, sb6_disk(qblk, qsqm, ddm, OUT, IN, xbits))},
                n_layer=1, n_embd=IN)
    f = RQ.RwkvqFile(str(p))
    t = f.tensor("blocks.0.att.receptance.weight")
    assert t["xbits"] == xbits
    assert np.array_equal(t["qblk"], qblk) and np.array_equal(t["qsqm"], qsqm)
    assert np.array_equal(t["ddm"], ddm)
    assert f.n_layer == 1 and f.naming == "world"


@pytest.mark.parametrize("bits", [6, 8])
def test_sym_round_trip_rebuilds_the_loader_layout(tmp_path, rng, bits):
    OUT, IN = 32, 512
    qblk, qs, d = _sym(rng, OUT, IN, bits)
    p = tmp_path / "m.rwkvq"
    m = {"shape": [OUT, IN], "kind": "sym", "bits": bits, "gw_gs": 16, "gw_sb": 16}
    write_rwkvq(p, {"blocks.1.ffn.key.weight": (m, sym_disk(qblk, qs, d, OUT, IN, bits))})
    t = RQ.RwkvqFile(str(p)).tensor("blocks.1.ffn.key.weight")
    assert t["bits"] == bits
    assert np.array_equal(t["qblk"], qblk) and np.array_equal(t["qs"], qs)
    assert np.array_equal(t["d"], np.asarray(d, np.uint16).reshape(t["d"].shape))


def test_manifest_checks(tmp_path, rng):
    OUT, IN = 16, 256
    qblk, qsqm, ddm = _sb6(rng, OUT, IN, 1)
    good = {"shape": [OUT, IN], "kind": "sb6", "bits": 5, "gw_gs": 32, "gw_sb": 8}
    bufs = sb6_disk(qblk, qsqm, ddm, OUT, IN, 1)

    def opens(entry=good, b=bufs, **kw):
        p = tmp_path / "x.rwkvq"
        write_rwkvq(p, {"t": (entry, b)}, **kw)
        return RQ.RwkvqFile(str(p))

    opens()
    with pytest.raises(RQ.RwkvqError, match="bit planes"):
        opens(dict(good, bits=6))
    with pytest.raises(RQ.RwkvqError, match="superblock"):
        opens(dict(good, gw_sb=4))
    with pytest.raises(RQ.RwkvqError, match="newer"):
        opens(format_version=3)
    with pytest.raises(RQ.RwkvqError, match="missing buffer"):
        opens(b={k: v for k, v in bufs.items() if k != "gw_dm"})
    with pytest.raises(RQ.RwkvqError, match="unknown layout"):
        opens(dict(good, kind="nf4"))
    # a pickle container and a file that is not .rwkvq
    p = tmp_path / "z.rwkvq"
    p.write_bytes(b"PK\x03\x04" + b"\0" * 16)
    with pytest.raises(RQ.RwkvqError, match="pickle"):
        RQ.RwkvqContainer(str(p))
    write_rwkvq(p, {"t": (good, bufs)})
    raw = p.read_bytes()
    n = int.from_bytes(raw[:8], "little")
    h = json.loads(raw[8:8 + n])
    h["__metadata__"] = {}
    hb = json.dumps(h).encode()
    p.write_bytes(len(hb).to_bytes(8, "little") + hb + raw[8 + n:])
    with pytest.raises(RQ.RwkvqError, match="not .rwkvq"):
        RQ.RwkvqFile(str(p))


def test_asym_and_rtn_are_refused_when_read(tmp_path, rng):
    p = tmp_path / "a.rwkvq"
    write_rwkvq(p, {"blocks.0.att.w1": ({"shape": [4, 4], "kind": "asym", "gw_gs": 4},
                                        {"codes": np.zeros((4, 4), np.uint8)})})
    f = RQ.RwkvqFile(str(p))
    with pytest.raises(RQ.RwkvqError, match="no kernel"):
        f.tensor("blocks.0.att.w1")


def test_names_map_world_and_x070():
    pairs = [("blocks.3.tmix.r_proj.weight", "blocks.3.att.receptance.weight"),
             ("blocks.0.tmix.o_proj.weight", "blocks.0.att.output.weight"),
             ("blocks.7.cmix.value.weight", "blocks.7.ffn.value.weight"),
             ("head.weight", "head.weight"), ("emb.weight", "emb.weight")]
    for x, w in pairs:
        assert RQ.world_key(x) == w and RQ.x070_key(w) == x
    assert RQ.world_key("blocks.0.tmix.x_r") is None
    assert RQ.x070_key("blocks.0.att.w1") is None
