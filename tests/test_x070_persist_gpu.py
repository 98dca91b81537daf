"""The persistent decode steps (one cooperative launch per step: the 1..8-row
kernel with exact-code GEMVs and the 9..64-row tcgen05 kernel, fp16
activations) against the decode oracle and against the per-kernel step.

Each persistent kernel computes the projections with the per-kernel path's
arithmetic for its row count (up to 8 rows the exact dequantised weight,
above 8 the fp16-dequantised weight), which the oracle models; the sums are
grouped differently, so they agree to fp32 rounding carried through fp16
activations, not bitwise.  Checked: logits within 2e-3 of the oracle over
several steps (tiny width; the 1.5B width is in test_x070_1p5b_gpu.py),
greedy ids equal to the per-kernel path's where the top two logits are not a
near tie, and the state the persistent steps leave behind continues
correctly on the per-kernel path.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _model(rows, n_embd=256, vocab=256, n_layer=2, seed=7, fan_in=False):
    from oracle import x070_oracle as XO
    from swiftrwkv_b200.x070 import X070Backbone, X070Config
    cfg = XO.Cfg(n_layer, n_embd, vocab)
    w = XO.tiny_weights(cfg, seed, fan_in_scale=fan_in)
    m = X070Backbone(X070Config(n_layer, n_embd, vocab), max_rows=rows, act="f16").load(w)
    return m, XO.X070Oracle(cfg, w, act="f16")


def _steps(m, ids, path):
    from swiftrwkv_b200 import _lib
    _lib.call("rwkv_x070_set_decode_path", m.h, path)
    rows = ids.shape[0]
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        m.reset(rows)
        out = [m.step(torch.from_numpy(ids[:, t]).cuda(), use_graph=True) for t in range(ids.shape[1])]
    s.synchronize()
    return [o.cpu().numpy() for o in out]


@pytest.mark.parametrize("rows", [1, 3, 8, 9, 20, 64])
def test_persistent_step_matches_oracle(cuda, rows):
    from oracle import x070_oracle as XO
    from swiftrwkv_b200 import _lib
    m, ref = _model(rows)
    _lib.call("rwkv_x070_set_decode_path", m.h, 1)
    assert _lib.lib().rwkv_x070_decode_path(m.h, rows) == 1
    ids = XO.splitmix_ids(rows, 4, vocab=256, seed=rows)
    got = _steps(m, ids, 1)
    st = ref.new_state(rows)
    for t in range(ids.shape[1]):
        want = ref.step(ids[:, t], st)
        assert rel_err(got[t], want) < 2e-3, (rows, t, rel_err(got[t], want))
    per_kernel = _steps(m, ids, 0)
    for t in range(ids.shape[1]):
        assert rel_err(got[t], per_kernel[t]) < 2e-3
        # greedy ids agree wherever the top two logits are not a near tie
        top2 = np.sort(per_kernel[t], 1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 1e-2 * np.abs(per_kernel[t]).max()
        assert np.array_equal(np.argmax(got[t], 1)[clear], np.argmax(per_kernel[t], 1)[clear])


def test_persistent_state_continues_on_the_per_kernel_path(cuda):
    from oracle import x070_oracle as XO
    from swiftrwkv_b200 import _lib
    rows = 16
    m, ref = _model(rows)
    ids = XO.splitmix_ids(rows, 5, vocab=256, seed=3)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        m.reset(rows)
        _lib.call("rwkv_x070_set_decode_path", m.h, 1)
        for t in range(3):
            m.step(torch.from_numpy(ids[:, t]).cuda(), use_graph=True)
        _lib.call("rwkv_x070_set_decode_path", m.h, 0)
        got = [m.step(torch.from_numpy(ids[:, t]).cuda(), use_graph=True) for t in range(3, 5)]
    s.synchronize()
    st = ref.new_state(rows)
    for t in range(5):
        want = ref.step(ids[:, t], st)
        if t >= 3:
            assert rel_err(got[t - 3].cpu().numpy(), want) < 2e-3


def test_persistent_step_is_not_taken_outside_its_range(cuda):
    from swiftrwkv_b200 import _lib
    m, _ = _model(65)
    L = _lib.lib()
    assert L.rwkv_x070_decode_path(m.h, 40) == 0     # the per-kernel graph by default
    assert L.rwkv_x070_decode_path(m.h, 1) == 0
    _lib.call("rwkv_x070_set_decode_path", m.h, 1)
    assert L.rwkv_x070_decode_path(m.h, 1) == 1      # the 1..8-row kernel
    assert L.rwkv_x070_decode_path(m.h, 8) == 1
    assert L.rwkv_x070_decode_path(m.h, 65) == 0     # beyond one 64-row tile
    assert L.rwkv_x070_decode_path(m.h, 40) == 1
    _lib.call("rwkv_x070_set_decode_path", m.h, 0)
    assert L.rwkv_x070_decode_path(m.h, 40) == 0
