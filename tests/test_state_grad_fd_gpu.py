"""State gradient of the tuner's WKV path, pinned without autograd: the
reference's testBatchGradientIsMeanOfRowsAndMatchesFiniteDifference
(Tests/RWKVGenTests/StateTuningTests.swift:243-294) restated on the layers of
the WKV-7 path.

Loss over two layers of a batch of two rows, each layer's state broadcast to
every row (h_in[b] = S_l): L(S) = mean over rows of sum over layers and
tokens of |y|^2 / 2, so dL/dy = y / B and dL/dS_l is the tuner's layer
gradient (sum over rows of the backward's dh_in) with that upstream gradient.

  * the gradient of the two-row batch is the mean of the one-row gradients
    (1e-4), and the two rows' gradients differ (> 1e-2);
  * for each layer, along a random direction d, the central difference
    (L(S + eps d) - L(S - eps d)) / (2 eps) matches <dL/dS_l, d> within
    0.03 |analytic| + 2e-3 -- the reference's tolerance -- with every L
    evaluated by the forward kernel alone.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err, wkv_inputs

pytestmark = pytest.mark.gpu

LAYERS, B, T, H = 2, 2, 32, 3


def _layers(seed=21):
    rng = np.random.default_rng(seed)
    return [[torch.from_numpy(x).cuda() for x in wkv_inputs(rng, B, T, H, scale=0.6)] for _ in range(LAYERS)]


def _loss(layers, states, rows):
    from swiftrwkv_b200 import kernel as K
    tot = 0.0
    for l, ins in enumerate(layers):
        ins = [x[rows] for x in ins]
        h = states[l].expand(ins[0].shape[0], H, 64, 64).contiguous()
        y, _ = K.wkv7SequenceForward(*ins, h)
        tot += float((y.double() ** 2).sum() / 2) / ins[0].shape[0]
    return tot


def _grads(layers, states, rows):
    from swiftrwkv_b200 import kernel as K
    from swiftrwkv_b200.state_tune import CudaStateOps
    ops = CudaStateOps()
    out = []
    for l, ins in enumerate(layers):
        ins = [x[rows].contiguous() for x in ins]
        nb = ins[0].shape[0]
        h = states[l].expand(nb, H, 64, 64).contiguous()
        y, _ = K.wkv7SequenceForward(*ins, h)
        dy = (y / nb).contiguous()
        g = torch.empty((H, 64, 64), device="cuda")
        ops.layer_grad(ins, dy, states[l].contiguous(), g)
        out.append(g)
    torch.cuda.synchronize()
    return out


def test_batch_gradient_is_mean_of_rows_and_matches_finite_difference(cuda):
    layers = _layers()
    rng = np.random.default_rng(3)
    states = [torch.from_numpy((rng.standard_normal((H, 64, 64)) * 0.2).astype(np.float32)).cuda()
              for _ in range(LAYERS)]
    both = _grads(layers, states, slice(0, 2))
    first = _grads(layers, states, slice(0, 1))
    second = _grads(layers, states, slice(1, 2))
    for l in range(LAYERS):
        b, f, s = (x[l].cpu().numpy() for x in (both, first, second))
        assert rel_err(b, (f + s) * 0.5) < 1e-4, l
        assert rel_err(f, s) > 1e-2, "the rows gave one gradient: nothing to compare"

    eps = 1e-2
    drng = np.random.default_rng(1)
    for l in range(LAYERS):
        d = torch.from_numpy(drng.standard_normal((H, 64, 64)).astype(np.float32)).cuda()
        analytic = float((both[l].double() * d.double()).sum())

        def at(e):
            moved = list(states)
            moved[l] = states[l] + e * d
            return _loss(layers, moved, slice(0, 2))

        numeric = (at(eps) - at(-eps)) / (2 * eps)
        assert abs(numeric - analytic) <= 0.03 * abs(analytic) + 2e-3, (l, numeric, analytic)
