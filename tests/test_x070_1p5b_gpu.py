"""GPU parity of the x070 decode runtime at the benchmarked 1.5B shapes.

The bench times x070 1.5B (C=2048, H=32, FFN 8192, vocab 65536, low-rank
96/96/64/256) over the 4-bit group-64 base.  These tests run that width with
L=2 (so the CPU oracle stays fast) and compare every step with the decode
oracle (oracle/x070_oracle.py, X070Generation.swift:201-319, 483-498):

  * fp16 activations, rows 1, 8, 64 and 256 -- the kernel choices the bench
    makes at those row counts: the exact-GEMV mma.sync path (<= 8 rows), the
    tcgen05 GEMM with each split-K cluster plan the 1.5B step uses (r/k/v,
    o, key, value, low-rank down/up, the 65536-row head), the C=2048 glue
    kernels (two 16-byte column groups per thread) and the warp-per-row WKV
    step at H=32; logits within 2e-3 (max-norm relative) of the oracle,
    which (like MLX) takes the product with the exact dequantised weight up to
    8 rows and with the weight dequantised into fp16 above;
  * fp32 activations: greedy token ids identical to the oracle's.

Weights follow the TinyBackbone recipe with fan-in scaling (std
0.05 * sqrt(256 / fan-in)), so that the 2048-wide projections keep the
conditioning the recipe has at its own width.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu

L, C, V = 2, 2048, 65536
MAX_ROWS = 256


@pytest.fixture(scope="module")
def weights():
    from oracle import x070_oracle as XO
    return XO.tiny_weights(XO.Cfg(L, C, V), seed=1515, fan_in_scale=True)


@pytest.fixture(scope="module")
def oracle16(weights):
    from oracle import x070_oracle as XO
    return XO.X070Oracle(XO.Cfg(L, C, V), weights, act="f16")


@pytest.fixture(scope="module")
def model16(cuda, weights):
    from swiftrwkv_b200.x070 import X070Backbone, X070Config
    m = X070Backbone(X070Config(L, C, V), max_rows=MAX_ROWS, act="f16").load(weights)
    yield m
    m.close()


@pytest.mark.parametrize("rows", [1, 2, 8, 64, 256])
def test_1p5b_width_logits_match_oracle(model16, oracle16, rows):
    from oracle import x070_oracle as XO
    ids = XO.splitmix_ids(rows, 3, vocab=V, seed=rows)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        model16.reset(rows)
        got = [model16.step(torch.from_numpy(ids[:, t]).cuda(), use_graph=True) for t in range(ids.shape[1])]
    s.synchronize()
    st = oracle16.new_state(rows)
    for t in range(ids.shape[1]):
        want = oracle16.step(ids[:, t], st)
        err = rel_err(got[t].cpu().numpy(), want)
        assert err < 2e-3, (rows, t, err)


def test_1p5b_width_greedy_ids_identical_fp32(cuda, weights):
    """north_star: greedy decode token ids identical for the fp32 path."""
    from oracle import x070_oracle as XO
    from swiftrwkv_b200.x070 import X070Backbone, X070Config
    m = X070Backbone(X070Config(L, C, V), max_rows=2, act="f32").load(weights)
    ref = XO.X070Oracle(XO.Cfg(L, C, V), weights, act="f32")
    prompts = XO.splitmix_ids(2, 4, vocab=V, seed=99)
    n_new = 6
    got = m.generateBatch(prompts, n_new)
    m.close()
    st = ref.new_state(2)
    for t in range(prompts.shape[1]):
        logits = ref.step(prompts[:, t], st)
    want = []
    for _ in range(n_new):
        nxt = np.argmax(logits, axis=1)
        want.append(nxt)
        logits = ref.step(nxt.astype(np.int32), st)
    assert np.array_equal(got, np.stack(want, axis=1).astype(np.int32))


def test_1p5b_width_prefill_matches_oracle(model16, oracle16):
    """Parallel prefill at the 1.5B width: 64 rows x 16 tokens (1024 token
    rows through the tcgen05 GEMMs, the chunked WKV at H=32), then a decode
    step from the prefilled state."""
    from oracle import x070_oracle as XO
    rows, T = 64, 16
    ids = XO.splitmix_ids(rows, T, vocab=V, seed=77)
    nxt = XO.splitmix_ids(rows, 1, vocab=V, seed=78)[:, 0]
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        model16.reset(rows)
        got = model16.prefill(torch.from_numpy(ids).cuda())
        cont = model16.step(torch.from_numpy(nxt).cuda(), use_graph=True)
    s.synchronize()
    st = oracle16.new_state(rows)
    oracle16.GEMV_MAX_ROWS = -1      # every prefill projection: fp16-dequantised weight
    for t in range(T):
        want = oracle16.step(ids[:, t], st)
    oracle16.GEMV_MAX_ROWS = 8
    assert rel_err(got.cpu().numpy(), want) < 2e-3, rel_err(got.cpu().numpy(), want)
    want = oracle16.step(nxt, st)
    assert rel_err(cont.cpu().numpy(), want) < 2e-3, rel_err(cont.cpu().numpy(), want)


@pytest.mark.parametrize("rows", [1, 8, 16, 32, 64])
def test_1p5b_width_persistent_step(model16, oracle16, rows):
    """The persistent decode step (rwkv_x070_set_decode_path 1) at the 1.5B
    width: the 1..8-row kernel (exact-code GEMVs, the 8192-wide value matrix
    in two staged activation windows) and the 9..64-row kernel at each of its
    tile widths (16, 32, 64 rows)."""
    from oracle import x070_oracle as XO
    from swiftrwkv_b200 import _lib
    _lib.call("rwkv_x070_set_decode_path", model16.h, 1)
    assert _lib.lib().rwkv_x070_decode_path(model16.h, rows) == 1
    ids = XO.splitmix_ids(rows, 2, vocab=V, seed=100 + rows)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        model16.reset(rows)
        got = [model16.step(torch.from_numpy(ids[:, t]).cuda(), use_graph=True) for t in range(2)]
    s.synchronize()
    _lib.call("rwkv_x070_set_decode_path", model16.h, 0)
    st = oracle16.new_state(rows)
    for t in range(2):
        want = oracle16.step(ids[:, t], st)
        assert rel_err(got[t].cpu().numpy(), want) < 2e-3, (rows, t)
