"""The x070 runtime over a dense bf16 base (BASELINE config 3's model class:
the reference's bf16 x070, X070Backbone.swift:24-37 with unquantised
weights) against the decode oracle.

bf16 activations run every projection -- base, low-rank, head -- on the
tcgen05 GEMM with bf16 operands (both A and B bf16, fp32 accumulation) at any
row count; fp32 activations take the CUDA-core path over the same bf16
weights.  Bounds: bf16 2e-2 (the bf16 bound of the WKV parity tests); fp32
1e-4 for the prefill and 3e-4 over five decode steps of 20 rows (fp32
rounding of the recurrent state carried through the steps: 1.3e-4 seen);
greedy ids identical on the fp32 path.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def model(act, rows, n_layer=2, n_embd=128, vocab=64, seed=11):
    from oracle import x070_oracle as XO
    from swiftrwkv_b200.x070 import X070Backbone, X070Config
    cfg = XO.Cfg(n_layer, n_embd, vocab)
    w = XO.tiny_weights(cfg, seed)
    m = X070Backbone(X070Config(n_layer, n_embd, vocab), max_rows=rows, act=act, base="bf16").load(w)
    return m, XO.X070Oracle(cfg, w, act=act, quant_bits=0)


@pytest.mark.parametrize("act,tol", [("bf16", 2e-2), ("f32", 3e-4)])
@pytest.mark.parametrize("rows", [1, 3, 20])
def test_dense_bf16_decode_matches_oracle(cuda, act, tol, rows):
    from oracle import x070_oracle as XO
    m, ref = model(act, rows)
    ids = XO.splitmix_ids(rows, 5, seed=rows)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        m.reset(rows)
        got = [m.step(torch.from_numpy(ids[:, t]).cuda(), use_graph=True) for t in range(ids.shape[1])]
    s.synchronize()
    st = ref.new_state(rows)
    for t in range(ids.shape[1]):
        want = ref.step(ids[:, t], st)
        assert rel_err(got[t].cpu().numpy(), want) < tol, (act, rows, t, rel_err(got[t].cpu().numpy(), want))


@pytest.mark.parametrize("act,tol", [("bf16", 2e-2), ("f32", 1e-4)])
def test_dense_bf16_prefill_matches_oracle(cuda, act, tol):
    from oracle import x070_oracle as XO
    rows, T = 2, 24
    m, ref = model(act, rows)
    ids = XO.splitmix_ids(rows, T, seed=29)
    lengths = [24, 17]
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        m.reset(rows)
        got = m.prefill(torch.from_numpy(ids).cuda(), lengths)
    s.synchronize()
    want = []
    for i in range(rows):
        st = ref.new_state(1)
        for t in range(lengths[i]):
            lg = ref.step(ids[i:i + 1, t], st)
        want.append(lg[0])
    assert rel_err(got.cpu().numpy(), np.stack(want)) < tol


def test_dense_bf16_greedy_ids_identical_fp32(cuda):
    from oracle import x070_oracle as XO
    m, ref = model("f32", 1)
    prompt = XO.splitmix_ids(1, 6, seed=4)[0]
    got = m.generate(prompt, 10)
    st = ref.new_state(1)
    for t in prompt:
        lg = ref.step(np.array([t], np.int32), st)
    want = []
    for _ in range(10):
        nxt = int(np.argmax(lg[0]))
        want.append(nxt)
        lg = ref.step(np.array([nxt], np.int32), st)
    assert [int(x) for x in got] == want


def test_base_and_activation_types_must_match(cuda):
    """A tensor-core product takes both operands in one type: the runtime
    refuses fp16 activations over the bf16 base and bf16 over the 4-bit one."""
    from swiftrwkv_b200 import _lib
    from swiftrwkv_b200.x070 import X070Backbone, X070Config
    cfg = X070Config(1, 128, 64)
    for act, base in (("f16", "bf16"), ("bf16", "q4")):
        with pytest.raises(_lib.RWKVError) as e:
            X070Backbone(cfg, max_rows=1, act=act, base=base)
        assert e.value.status == _lib.E_DTYPE
