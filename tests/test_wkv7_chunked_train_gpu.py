"""The chunked (DPLR) training path -- train forward with 16-token
checkpoints and the chunked backward -- against the oracle's train path and
against the sequential kernels, with the reference's bounds
(WKV7TrainKernelTests.swift:67-82: gradients, dh_in included, within 1e-3
relative in fp32; 2e-2 for bf16 / fp16 inputs), over initial states, upstream
state gradients, decays that take the token-by-token guard, and the
config-1 shape (B=1, T=1024, H=12)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import config1_inputs, rel_err, wkv_inputs

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-3
NAMES = ("dr", "dw", "dk", "dv", "da", "db", "dh_in")


def dev(x, dtype=torch.float32):
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).cuda().to(dtype)


def host(t):
    return t.detach().float().cpu().numpy()


def _case(rng, B, T, H, with_h0=True, with_dh=True):
    ins = wkv_inputs(rng, B, T, H)
    h0 = (rng.standard_normal((B, H, 64, 64)) * 0.1).astype(np.float32) if with_h0 else None
    dy = rng.standard_normal((B, T, H, 64)).astype(np.float32)
    dh = (rng.standard_normal((B, H, 64, 64)) * 0.1).astype(np.float32) if with_dh else None
    return ins, h0, dy, dh


@pytest.mark.parametrize("B,T,H", [(1, 16, 1), (1, 64, 2), (2, 48, 3), (1, 256, 4), (3, 32, 2),
                                   # 24+ chunks: the grouped three-level scans, forward and reverse
                                   (1, 400, 2), (2, 528, 2)])
@pytest.mark.parametrize("with_h0,with_dh", [(True, True), (False, False), (True, False)])
def test_chunked_backward_matches_oracle(cuda, oracle, rng, B, T, H, with_h0, with_dh):
    from swiftrwkv_b200 import kernel as K
    ins, h0, dy, dh = _case(rng, B, T, H, with_h0, with_dh)
    want = oracle.wkv7_train(*ins, h0, dy, dh)[2:]
    d = [dev(x) for x in ins]
    y, h_out, sa, ck = K.wkv7TrainForwardChunked(*d, dev(h0))
    got = K.wkv7BackwardChunked(*d, dev(h0), ck, dev(dy), dev(dh))
    torch.cuda.synchronize()
    for name, g, wv in zip(NAMES, got, want):
        g = host(g)
        assert np.isfinite(g).all(), name
        assert rel_err(g, wv) < GRAD_TOL, (name, rel_err(g, wv))


@pytest.mark.parametrize("T", [96, 784])
def test_chunked_train_forward_matches_sequential(cuda, rng, T):
    """y, h_out, sa and every 16-token checkpoint against the sequential train
    forward (T = 784: 49 chunks, the grouped scan with 7 groups of 7)."""
    from swiftrwkv_b200 import kernel as K
    ins, h0, _, _ = _case(rng, 2, T, 3)
    d = [dev(x) for x in ins]
    a = K._train_forward(*d, dev(h0))
    b = K.wkv7TrainForwardChunked(*d, dev(h0))
    assert (a[0] - b[0]).abs().max().item() < 1e-4
    for x, z in zip(a[1:], b[1:]):
        assert rel_err(host(z), host(x)) < 1e-5


def test_chunked_backward_config1_matches_sequential(cuda, rng):
    """BASELINE config 1 (B=1, T=1024, H=12), dy ~ N(0,1): the chunked and the
    sequential backward from the same checkpoints."""
    from swiftrwkv_b200 import kernel as K
    ins = [dev(x) for x in config1_inputs(rng)]
    dy = torch.randn_like(ins[0])
    _, _, _, ck = K._train_forward(*ins, None)
    a = K.wkv7Backward(*ins, None, ck, dy, None)
    b = K.wkv7BackwardChunked(*ins, None, ck, dy, None)
    for name, x, z in zip(NAMES, a, b):
        assert rel_err(host(z), host(x)) < GRAD_TOL, name


def test_chunked_backward_tiny_decays_take_the_guard(cuda, oracle, rng):
    """Chunks whose cumulative decay underflows go token by token.  The
    reference is the double-precision exact backward: the restated v2 kernel
    (oracle.wkv7_train) itself returns NaN where a decay is exactly zero."""
    from swiftrwkv_b200 import kernel as K
    ins, h0, dy, dh = _case(rng, 1, 64, 2)
    r, w, k, v, a, b = ins
    w = w.copy()
    w[:, 16:32] = 1e-3      # chunk 1: c_16 = 1e-48, token by token
    w[:, 40, 0] = 0.0       # chunk 2: an exact zero
    ins = (r, w, k, v, a, b)
    want = oracle.wkv7_exact(*ins, h0, dy, dh)[2:]
    d = [dev(x) for x in ins]
    _, _, _, ck = K.wkv7TrainForwardChunked(*d, dev(h0))
    got = K.wkv7BackwardChunked(*d, dev(h0), ck, dev(dy), dev(dh))
    for name, g, wv in zip(NAMES, got, want):
        assert rel_err(host(g), wv) < GRAD_TOL, (name, rel_err(host(g), wv))


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_chunked_backward_low_precision_inputs(cuda, oracle, rng, dt):
    from swiftrwkv_b200 import kernel as K
    ins, h0, dy, dh = _case(rng, 2, 64, 3)
    d = [dev(x).to(dt) for x in ins]
    dyd = dev(dy).to(dt)
    want = oracle.wkv7_train(*[host(x) for x in d], h0, host(dyd), dh)[2:]
    _, _, _, ck = K.wkv7TrainForwardChunked(*d, dev(h0))
    got = K.wkv7BackwardChunked(*d, dev(h0), ck, dyd, dev(dh))
    for name, g, wv in zip(NAMES, got, want):
        assert g.dtype == (torch.float32 if name == "dh_in" else dt)
        assert rel_err(host(g), wv) < 2e-2, name


def test_chunked_backward_is_deterministic(cuda, rng):
    from swiftrwkv_b200 import kernel as K
    ins, h0, dy, dh = _case(rng, 2, 128, 4)
    d = [dev(x) for x in ins]
    _, _, _, ck = K.wkv7TrainForwardChunked(*d, dev(h0))
    g1 = K.wkv7BackwardChunked(*d, dev(h0), ck, dev(dy), dev(dh))
    g2 = K.wkv7BackwardChunked(*d, dev(h0), ck, dev(dy), dev(dh))
    for x, z in zip(g1, g2):
        assert torch.equal(x, z)


def test_autograd_uses_both_training_paths(cuda, oracle, rng):
    from swiftrwkv_b200 import kernel as K
    ins, h0, dy, dh = _case(rng, 1, 48, 2)
    want = oracle.wkv7_train(*ins, h0, dy, dh)[2:]
    saved = K.useChunkedTraining
    try:
        for chunked in (True, False):
            K.useChunkedTraining = chunked
            d = [dev(x).requires_grad_() for x in ins]
            h = dev(h0).requires_grad_()
            y, h_out = K.wkv7TrainWithState(*d, h)
            ((y * dev(dy)).sum() + (h_out * dev(dh)).sum()).backward()
            for name, t, wv in zip(NAMES, d + [h], want):
                assert rel_err(host(t.grad), wv) < GRAD_TOL, (chunked, name)
    finally:
        K.useChunkedTraining = saved
