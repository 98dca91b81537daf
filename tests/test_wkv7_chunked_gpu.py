"""The chunked (DPLR) prefill form of the WKV-7 forward against the oracle and
against the sequential kernel: same bounds as the forward parity tests
(WKV7KernelParityTests.swift:32-62: <= 1e-4 absolute on y, the state to the
same relative bound), over ragged lengths, initial states, every input dtype
and decays small enough to take the token-by-token guard."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import config1_inputs, rel_err, wkv_inputs

pytestmark = pytest.mark.gpu


def dev(x, dtype=torch.float32):
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).cuda().to(dtype)


def host(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("B,T,H", [(1, 1, 2), (1, 5, 3), (1, 16, 2), (1, 17, 4), (2, 53, 3),
                                   (1, 512, 12), (3, 32, 1), (2, 100, 5),
                                   # 24+ chunks: the grouped three-level scan (ragged last chunk and group)
                                   (1, 1000, 3), (2, 390, 2)])
@pytest.mark.parametrize("with_h0", [False, True])
def test_chunked_matches_oracle(cuda, oracle, rng, B, T, H, with_h0):
    from swiftrwkv_b200 import kernel as K
    ins = wkv_inputs(rng, B, T, H)
    h0 = (rng.standard_normal((B, H, 64, 64)) * 0.1).astype(np.float32) if with_h0 else None
    y_ref, h_ref = oracle.wkv7_forward(*ins, h0)
    y, h = K.wkv7PrefillChunked(*map(dev, ins), dev(h0))
    torch.cuda.synchronize()
    assert np.abs(host(y) - y_ref).max() < 1e-4
    assert rel_err(host(h), h_ref) < 1e-5


def test_chunked_config1_matches_sequential(cuda, rng):
    """BASELINE config 1 (B=1, T=1024, H=12): chunked vs the sequential kernel."""
    from swiftrwkv_b200 import kernel as K
    ins = [dev(x) for x in config1_inputs(rng)]
    y1, h1 = K.wkv7SequenceForward(*ins)
    y2, h2 = K.wkv7PrefillChunked(*ins)
    assert (y1 - y2).abs().max().item() < 1e-4
    assert rel_err(host(h2), host(h1)) < 1e-5


def test_chunked_tiny_decays_take_the_guard(cuda, oracle, rng):
    """Decays near zero (cumulative products below 1e-30 inside a chunk) are
    stepped token by token; results stay within the same bound."""
    from swiftrwkv_b200 import kernel as K
    r, w, k, v, a, b = wkv_inputs(rng, 1, 48, 2)
    w = w.copy()
    w[:, 16:32] = 1e-3      # chunk 1: c_16 = 1e-48
    w[:, 40, 0] = 0.0       # chunk 2: an exact zero
    y_ref, h_ref = oracle.wkv7_forward(r, w, k, v, a, b, None)
    y, h = K.wkv7PrefillChunked(*map(dev, (r, w, k, v, a, b)))
    assert np.abs(host(y) - y_ref).max() < 1e-4
    assert rel_err(host(h), h_ref) < 1e-5


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_chunked_low_precision_inputs(cuda, oracle, rng, dt):
    from swiftrwkv_b200 import kernel as K
    ins = wkv_inputs(rng, 2, 64, 4)
    ins16 = [dev(x).to(dt) for x in ins]
    y_ref, h_ref = oracle.wkv7_forward(*[host(x) for x in ins16], None)
    y, h = K.wkv7PrefillChunked(*ins16)
    assert rel_err(host(y), y_ref) < 2e-2
    assert rel_err(host(h), h_ref) < 1e-4


def test_chunked_state_chains(cuda, rng):
    """Two chunked calls with the state passed on agree with one call (to
    fp32 rounding: the chunk boundaries differ)."""
    from swiftrwkv_b200 import kernel as K
    ins = [dev(x) for x in wkv_inputs(rng, 1, 80, 3)]
    y, h = K.wkv7PrefillChunked(*ins)
    y1, h1 = K.wkv7PrefillChunked(*(x[:, :37] for x in ins))
    y2, h2 = K.wkv7PrefillChunked(*(x[:, 37:].contiguous() for x in ins), h1)
    assert (torch.cat([y1, y2], 1) - y).abs().max().item() < 1e-4
    assert rel_err(host(h2), host(h)) < 1e-5
