"""`.rwkvq` files on the GPU: tensors read by swiftrwkv_b200.rwkvq dequantise
bit-exactly to the oracle's unpacking of the same buffers (sb6:
RwkvqDequant.swift:110-141; sym: :339-389), and a model loaded from a
`.rwkvq` base (X070Backbone.load_rwkvq) equals the same model loaded from the
dequantised weights directly; matrices kept native run the sb6 / sym GEMVs
inside the decode step and match the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err
from rwkvq_fixture import sb6_disk, sym_disk, write_rwkvq

pytestmark = pytest.mark.gpu


def test_reader_dequantises_bit_exactly(cuda, oracle, rng, tmp_path):
    from swiftrwkv_b200 import rwkvq as RQ
    from test_quant_gpu import make_sb6, make_sym
    OUT, IN = 64, 512
    sb = make_sb6(rng, OUT, IN, 2)
    sy = make_sym(rng, OUT, IN, 6)
    p = tmp_path / "q.rwkvq"
    write_rwkvq(p, {
        "blocks.0.att.key.weight": ({"shape": [OUT, IN], "kind": "sb6", "bits": 6, "gw_gs": 32, "gw_sb": 8},
                                    sb6_disk(*sb, OUT, IN, 2)),
        "blocks.0.ffn.value.weight": ({"shape": [OUT, IN], "kind": "sym", "bits": 6, "gw_gs": 16, "gw_sb": 16},
                                      sym_disk(*sy, OUT, IN, 6))})
    f = RQ.RwkvqFile(str(p))
    got = f.dequantize("blocks.0.att.key.weight").cpu().numpy()
    assert np.array_equal(got, oracle.sb6_dequant(*sb, OUT, IN, 2))
    got = f.dequantize("blocks.0.ffn.value.weight").cpu().numpy()
    assert np.array_equal(got, oracle.sym_dequant(*sy, OUT, IN, 6))


@pytest.mark.parametrize("base,act", [("bf16", "bf16"), ("q4", "f16")])
def test_model_from_rwkvq_equals_model_from_dequantised_weights(cuda, oracle, rng, tmp_path, base, act):
    from oracle import x070_oracle as XO
    from swiftrwkv_b200.x070 import X070Backbone, X070Config
    from test_quant_gpu import make_sb6, make_sym
    L, C, V = 2, 256, 256
    cfg = XO.Cfg(L, C, V)
    w = XO.tiny_weights(cfg, 5)
    tensors, deq = {}, {}
    for l in range(L):
        for x070k, worldk, (OUT, IN) in ((f"blocks.{l}.tmix.r_proj.weight", f"blocks.{l}.att.receptance.weight", (C, C)),
                                         (f"blocks.{l}.cmix.key.weight", f"blocks.{l}.ffn.key.weight", (4 * C, C))):
            # the synthetic scales shrunk so that the model's activations stay
            # in fp16 range (the codes are uniform over their full width)
            shrink = lambda u16: (u16.view(np.float16) * np.float16(0.02)).view(np.uint16)
            if l == 0:
                qblk, qsqm, ddm = make_sb6(rng, OUT, IN, 1)
                q = (qblk, qsqm, shrink(ddm))
                tensors[worldk] = ({"shape": [OUT, IN], "kind": "sb6", "bits": 5, "gw_gs": 32, "gw_sb": 8},
                                   sb6_disk(*q, OUT, IN, 1))
                deq[x070k] = oracle.sb6_dequant(*q, OUT, IN, 1)
            else:
                qblk, qs, d = make_sym(rng, OUT, IN, 8)
                q = (qblk, qs, shrink(d))
                tensors[worldk] = ({"shape": [OUT, IN], "kind": "sym", "bits": 8, "gw_gs": 16, "gw_sb": 16},
                                   sym_disk(*q, OUT, IN, 8))
                deq[x070k] = oracle.sym_dequant(*q, OUT, IN, 8)
    p = tmp_path / "m.rwkvq"
    write_rwkvq(p, tensors, n_layer=L, n_embd=C)
    rest = {k: v for k, v in w.items() if k not in deq}
    a = X070Backbone(X070Config(L, C, V), max_rows=3, act=act, base=base)
    loaded = a.load_rwkvq(str(p), rest, native=False)
    assert sorted(loaded) == sorted(deq)
    b = X070Backbone(X070Config(L, C, V), max_rows=3, act=act, base=base).load({**rest, **deq})
    ids = XO.splitmix_ids(3, 3, vocab=V, seed=2)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        a.reset(3)
        b.reset(3)
        for t in range(3):
            la = a.step(torch.from_numpy(ids[:, t]).cuda())
            lb = b.step(torch.from_numpy(ids[:, t]).cuda())
    s.synchronize()
    assert torch.isfinite(la).all()
    assert torch.equal(la, lb)


@pytest.mark.parametrize("rows,act,tol", [(1, "f16", 2e-3), (3, "f16", 2e-3), (9, "f16", 2e-3), (2, "f32", 1e-4)])
def test_native_rwkvq_matrices_match_oracle(cuda, oracle, rng, tmp_path, rows, act, tol):
    """sb6 / sym matrices kept as stored (rwkv_x070_set_param_rwkvq): the step
    runs them through the sb6 / sym GEMV kernels with the projection's
    epilogue -- plain (r), += x (o, value), relu^2 into fp16 (key), the head --
    at every row count, against the oracle with the exact dequantised weights
    (the reference's sidecar decode, X070Backbone.swift:708-732)."""
    from oracle import x070_oracle as XO
    from swiftrwkv_b200.x070 import X070Backbone, X070Config
    from test_quant_gpu import make_sb6, make_sym
    L, C, V = 2, 256, 256
    cfg = XO.Cfg(L, C, V)
    w = XO.tiny_weights(cfg, 9)
    shrink = lambda u16: (u16.view(np.float16) * np.float16(0.02)).view(np.uint16)
    tensors, deq = {}, {}
    plan = {  # x070 name: (world name, kind, bits, OUT, IN)
        "blocks.0.tmix.r_proj.weight": ("blocks.0.att.receptance.weight", "sb6", 0, C, C),
        # r and k of layer 0, k and v of layer 1 share a format: one launch at 1 row
        "blocks.0.tmix.k_proj.weight": ("blocks.0.att.key.weight", "sb6", 0, C, C),
        "blocks.1.tmix.r_proj.weight": ("blocks.1.att.receptance.weight", "sym", 6, C, C),
        "blocks.1.tmix.k_proj.weight": ("blocks.1.att.key.weight", "sb6", 1, C, C),
        "blocks.0.tmix.o_proj.weight": ("blocks.0.att.output.weight", "sym", 8, C, C),
        "blocks.0.cmix.key.weight": ("blocks.0.ffn.key.weight", "sym", 6, 4 * C, C),
        "blocks.1.cmix.value.weight": ("blocks.1.ffn.value.weight", "sb6", 2, C, 4 * C),
        "blocks.1.tmix.v_proj.weight": ("blocks.1.att.value.weight", "sb6", 1, C, C),
        "head.weight": ("head.weight", "sym", 8, V, C),
    }
    for k, (wk, kind, bits, OUT, IN) in plan.items():
        if kind == "sb6":
            qblk, qsqm, ddm = make_sb6(rng, OUT, IN, bits)
            q = (qblk, qsqm, shrink(ddm))
            tensors[wk] = ({"shape": [OUT, IN], "kind": "sb6", "bits": 4 + bits, "gw_gs": 32, "gw_sb": 8},
                           sb6_disk(*q, OUT, IN, bits))
            deq[k] = oracle.sb6_dequant(*q, OUT, IN, bits)
        else:
            qblk, qs, d = make_sym(rng, OUT, IN, bits)
            q = (qblk, qs, shrink(d))
            tensors[wk] = ({"shape": [OUT, IN], "kind": "sym", "bits": bits, "gw_gs": 16, "gw_sb": 16},
                           sym_disk(*q, OUT, IN, bits))
            deq[k] = oracle.sym_dequant(*q, OUT, IN, bits)
    p = tmp_path / "n.rwkvq"
    write_rwkvq(p, tensors, n_layer=L, n_embd=C)
    rest = {k: v for k, v in w.items() if k not in deq}
    m = X070Backbone(X070Config(L, C, V), max_rows=rows, act=act)
    assert sorted(m.load_rwkvq(str(p), rest)) == sorted(deq)
    assert m.decode_path(rows) == 0
    ref = XO.X070Oracle(cfg, rest, act=act, exact=deq)
    ids = XO.splitmix_ids(rows, 3, vocab=V, seed=rows)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        m.reset(rows)
        got = [m.step(torch.from_numpy(ids[:, t]).cuda(), use_graph=True) for t in range(3)]
    s.synchronize()
    st = ref.new_state(rows)
    for t in range(3):
        want = ref.step(ids[:, t], st)
        e = rel_err(got[t].cpu().numpy(), want)
        assert e < tol, (rows, act, t, e)
