"""State tuning over the WKV-7 path: host logic on CPU.

The tuner's rank logic (local batch slices, per-layer allreduce buckets, the
1/world average, the schedule and bias corrections, checkpoint/restore) runs
here against the oracle's implementation of its two device operations, over
`gloo` with world size 2, and must equal one process over the whole batch.
The CUDA operations themselves are checked against the same oracle in
test_state_tune_gpu.py.
"""
from __future__ import annotations

import math
import os
import socket

import numpy as np
import pytest
import torch

from conftest import wkv_inputs

import oracle.oracle as orc
from swiftrwkv_b200.state_tune import StateTuneConfig, WKVStateTuner


class OracleOps:
    """The tuner's device operations restated by the oracle (CPU tensors)."""

    def layer_grad(self, inputs, dy, state, grad):
        g = orc.state_layer_grad(*(x.numpy() for x in inputs), dy.numpy(), state.numpy())
        grad.copy_(torch.from_numpy(g))

    def adamw(self, param, m, v, grad, norm_out, **kw):
        p, m2, v2, n = orc.adamw_clip_step(param.numpy(), m.numpy(), v.numpy(), grad.numpy(), **kw)
        param.copy_(torch.from_numpy(p))
        m.copy_(torch.from_numpy(m2))
        v.copy_(torch.from_numpy(v2))
        norm_out.fill_(float(n))


L, H, T, BG = 2, 2, 32, 4   # layers, heads, tokens, global batch


def _global_batch(seed=11):
    rng = np.random.default_rng(seed)
    layers = []
    for _ in range(L):
        r, w, k, v, a, b = wkv_inputs(rng, BG, T, H)
        dy = rng.standard_normal((BG, T, H, 64)).astype(np.float32)
        layers.append([torch.from_numpy(np.ascontiguousarray(x)) for x in (r, w, k, v, a, b, dy)])
    init = torch.from_numpy((rng.standard_normal((L, H, 64, 64)) * 0.1).astype(np.float32))
    return layers, init


def _cfg():
    return StateTuneConfig(lr=1e-2, lrMin=1e-3, warmupSteps=1, maxSteps=4, gradClip=1.0)


# ------------------------------------------------------------------ schedule

def test_learning_rate_follows_the_reference_schedule():
    f = np.float32
    c = StateTuneConfig(lr=3e-4, lrMin=3e-5, schedule="cosine", warmupSteps=10, maxSteps=110)
    assert c.learningRate(0) == float(f(3e-4) * f(1) / f(10))
    assert c.learningRate(9) == float(f(3e-4) * f(10) / f(10))
    # after warm-up: lrMin + (lr - lrMin) * 0.5 (1 + cos(pi p)), p = (s - 10) / 100
    for s, p in [(10, 0.0), (60, 0.5), (110, 1.0), (500, 1.0)]:
        want = 3e-5 + (3e-4 - 3e-5) * 0.5 * (1 + math.cos(math.pi * p))
        assert abs(c.learningRate(s) - want) < 1e-9
    lin = StateTuneConfig(lr=1.0, lrMin=0.0, schedule="linear", warmupSteps=0, maxSteps=4)
    assert [lin.learningRate(s) for s in range(5)] == [1.0, 0.75, 0.5, 0.25, 0.0]
    const = StateTuneConfig(lr=0.5, schedule="constant", warmupSteps=2)
    assert [const.learningRate(s) for s in range(4)] == [0.25, 0.5, 0.5, 0.5]
    with pytest.raises(ValueError):
        StateTuneConfig(schedule="step")


def test_bias_corrections_are_fp32_of_the_double_power():
    c = StateTuneConfig()
    c1, c2 = c.bias_corrections(3)
    assert c1 == float(np.float32(1) - np.float32(float(np.float32(0.9)) ** 3))
    assert c2 == float(np.float32(1) - np.float32(float(np.float32(0.99)) ** 3))


# ------------------------------------------------------------------ optimizer oracle

def test_adamw_oracle_clips_by_global_norm_and_updates():
    rng = np.random.default_rng(3)
    p = rng.standard_normal(1000).astype(np.float32)
    g = (rng.standard_normal(1000) * 5).astype(np.float32)
    z = np.zeros_like(p)
    kw = dict(grad_scale=0.5, clip=1.0, lr=0.1, beta1=0.9, beta2=0.99, eps=1e-8,
              weight_decay=0.0, c1=0.1, c2=0.01)
    p1, m1, v1, norm = orc.adamw_clip_step(p, z, z, g, **kw)
    assert abs(norm - np.linalg.norm(g.astype(np.float64) * 0.5)) < 1e-3
    gc = g * 0.5 * (1.0 / (norm + 1e-6))          # clipped to norm 1
    np.testing.assert_allclose(m1, 0.1 * gc, rtol=1e-5, atol=1e-9)
    np.testing.assert_allclose(v1, 0.01 * gc * gc, rtol=1e-5, atol=1e-12)
    # first step: mhat / sqrt(vhat) = sign(g) where |g| >> eps: those entries move by lr
    big = np.abs(gc) > 1e-4
    np.testing.assert_allclose((p - p1)[big], 0.1 * np.sign(g)[big], rtol=1e-4)
    # no clipping when clip <= 0: the moments see the unclipped, scaled gradient
    _, m2, _, _ = orc.adamw_clip_step(p, z, z, g, **{**kw, "clip": 0.0})
    np.testing.assert_allclose(m2, 0.1 * g * 0.5, rtol=1e-6)
    # decoupled weight decay adds wd * p to the update
    p3, _, _, _ = orc.adamw_clip_step(p, z, z, g, **{**kw, "weight_decay": 0.1})
    np.testing.assert_allclose(p1 - p3, 0.1 * 0.1 * p, rtol=1e-3, atol=1e-6)


# ------------------------------------------------------------------ tuner on one process

def _run_single(steps=2, grad_scale=None):
    layers, init = _global_batch()
    tu = WKVStateTuner(L, H, config=_cfg(), initial=init, device="cpu", ops=OracleOps(),
                       grad_scale=grad_scale)
    norms = [float(tu.step(layers)) for _ in range(steps)]
    return tu, norms


def test_tuner_moves_the_states_and_reports_the_norm():
    layers, init = _global_batch()
    tu, norms = _run_single()
    assert tu.t == 2 and tu.step_index == 2
    assert all(n > 0 and math.isfinite(n) for n in norms)
    assert not torch.equal(tu.params, init)
    # the first step's gradient equals the oracle's per-layer state gradient
    tu0 = WKVStateTuner(L, H, config=_cfg(), initial=init, device="cpu", ops=OracleOps())
    tu0.step(layers)
    for l in range(L):
        want = orc.state_layer_grad(*(x.numpy() for x in layers[l][:6]), layers[l][6].numpy(),
                                    init[l].numpy())
        np.testing.assert_array_equal(tu0.grads[l].numpy(), want)


def test_tuner_checkpoint_restore_continues_identically():
    layers, init = _global_batch()
    a = WKVStateTuner(L, H, config=_cfg(), initial=init, device="cpu", ops=OracleOps())
    a.step(layers)
    ck = a.checkpoint()
    a.step(layers)
    b = WKVStateTuner(L, H, config=_cfg(), device="cpu", ops=OracleOps())
    b.restore(ck)
    b.step(layers)
    assert (b.step_index, b.t) == (a.step_index, a.t)
    assert torch.equal(a.params, b.params) and torch.equal(a.m, b.m) and torch.equal(a.v, b.v)
    with pytest.raises(KeyError):
        b.restore({"param": ck["param"]})


def test_tuner_rejects_bad_inputs():
    layers, init = _global_batch()
    tu = WKVStateTuner(L, H, config=_cfg(), initial=init, device="cpu", ops=OracleOps())
    with pytest.raises(ValueError, match="layers given"):
        tu.step(layers[:1])
    bad = [list(t) for t in layers]
    bad[0] = [x[:, :24] for x in bad[0]]
    with pytest.raises(ValueError, match="multiple of CHUNK"):
        tu.step(bad)
    with pytest.raises(ValueError, match="head_size"):
        WKVStateTuner(L, H, head_size=32, device="cpu", ops=OracleOps())
    with pytest.raises(ValueError):
        WKVStateTuner(L, H, initial=torch.zeros(L, H + 1, 64, 64), ops=OracleOps())
    with pytest.raises(ValueError, match="does not split"):
        WKVStateTuner.local_slice(5, 0, 2)


# ------------------------------------------------------------------ data parallel (gloo)

def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dp_worker(rank, world, port, out_dir, steps):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layers, init = _global_batch()
        sl = WKVStateTuner.local_slice(BG, rank, world)
        local = [[x[sl].contiguous() for x in t] for t in layers]
        tu = WKVStateTuner(L, H, config=_cfg(), initial=init, device="cpu", ops=OracleOps())
        assert tu.world == world and tu.grad_scale == 1.0 / world
        norms = [float(tu.step(local)) for _ in range(steps)]
        torch.save({"params": tu.params, "m": tu.m, "v": tu.v, "norms": norms},
                   os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        torch.distributed.destroy_process_group()


def test_data_parallel_two_ranks_equal_one_process_over_the_whole_batch(tmp_path):
    world, steps = 2, 2
    port = _free_port()
    torch.multiprocessing.start_processes(_dp_worker, args=(world, port, str(tmp_path), steps),
                                          nprocs=world, join=True, start_method="spawn")
    ranks = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    # every rank made the same update
    for key in ("params", "m", "v"):
        assert torch.equal(ranks[0][key], ranks[1][key]), key
    assert ranks[0]["norms"] == ranks[1]["norms"]
    # and it is the single-process step over the whole batch, averaged over the ranks
    single, norms = _run_single(steps, grad_scale=1.0 / world)
    np.testing.assert_allclose(ranks[0]["params"].numpy(), single.params.numpy(), rtol=0, atol=1e-6)
    np.testing.assert_allclose(ranks[0]["norms"], norms, rtol=1e-5)
