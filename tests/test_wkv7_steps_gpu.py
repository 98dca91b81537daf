"""wkv7Step / wkv7Steps, the differentiable few-token steps (WKV7Step.swift:
45-123), against the oracle's double-precision exact forward and backward:
outputs within 1e-4 absolute and gradients (hIn included) within 1e-3
relative, as the reference bounds its kernels (WKV7KernelParityTests.swift:
32-62); any T (the reranker head's probe tokens), both input ranks."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err, wkv_inputs

pytestmark = pytest.mark.gpu


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.parametrize("B,T,H", [(2, 1, 3), (1, 2, 2), (3, 5, 2), (1, 17, 4), (2, 32, 1)])
def test_steps_forward_and_gradients_match_exact(cuda, oracle, rng, B, T, H):
    from swiftrwkv_b200 import kernel as K
    ins = wkv_inputs(rng, B, T, H)
    h0 = (rng.standard_normal((B, H, 64, 64)) * 0.1).astype(np.float32)
    dy = rng.standard_normal((B, T, H, 64)).astype(np.float32)
    dh = (rng.standard_normal((B, H, 64, 64)) * 0.1).astype(np.float32)
    want = oracle.wkv7_exact(*ins, h0, dy, dh)
    xs = [dev(x).requires_grad_() for x in ins]
    h = dev(h0).requires_grad_()
    out, h_out = K.wkv7Steps(*xs, h)
    assert out.shape == (B, T, H, 64) and out.dtype == torch.float32
    assert np.abs(out.detach().cpu().numpy() - want[0]).max() < 1e-4
    assert rel_err(h_out.detach().cpu().numpy(), want[1]) < 1e-5
    ((out * dev(dy)).sum() + (h_out * dev(dh)).sum()).backward()
    for name, t, wv in zip(("dr", "dw", "dk", "dv", "da", "db", "dh_in"), xs + [h], want[2:]):
        assert rel_err(t.grad.cpu().numpy(), wv) < 1e-3, name


def test_step_ranks_and_zero_state(cuda, oracle, rng):
    from swiftrwkv_b200 import kernel as K
    ins = wkv_inputs(rng, 2, 1, 3)
    y_ref, h_ref = oracle.wkv7_exact(*ins)
    y4, h4 = K.wkv7Step(*map(dev, ins))                       # [B,1,H,D], hIn = zeros
    y3, h3 = K.wkv7Step(*(dev(x[:, 0]) for x in ins))         # [B,H,D]
    assert y4.shape == (2, 1, 3, 64) and y3.shape == (2, 3, 64)
    assert torch.equal(y4[:, 0], y3) and torch.equal(h4, h3)
    assert np.abs(y3.cpu().numpy() - y_ref[:, 0]).max() < 1e-4
    assert rel_err(h3.cpu().numpy(), h_ref) < 1e-5
