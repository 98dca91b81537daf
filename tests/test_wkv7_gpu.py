"""GPU parity of the WKV-7 kernels against the oracle and the autograd golden
fixture, through the C ABI (swiftrwkv_b200.kernel mirrors RWKVKernel)."""
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


# WKV7SequenceTests.swift:29-47 shapes
SEQ_SHAPES = [(1, 1, 2), (1, 5, 3), (1, 16, 2), (1, 17, 4), (2, 53, 3), (1, 512, 12), (3, 32, 1)]


@pytest.mark.parametrize("B,T,H", SEQ_SHAPES)
@pytest.mark.parametrize("with_h0", [False, True])
def test_forward_matches_oracle(cuda, oracle, rng, B, T, H, with_h0):
    from swiftrwkv_b200 import kernel as K
    ins = wkv_inputs(rng, B, T, H)
    h0 = (rng.standard_normal((B, H, 64, 64)) * 0.1).astype(np.float32) if with_h0 else None
    y_ref, h_ref = oracle.wkv7_forward(*ins, h0)
    y, h = K.wkv7SequenceForward(*map(dev, ins), dev(h0))
    torch.cuda.synchronize()
    assert np.abs(host(y) - y_ref).max() < 1e-4
    assert rel_err(host(h), h_ref) < 1e-5


def test_forward_and_backward_match_autograd_golden(cuda, golden):
    """WKV7KernelParityTests / WKV7TrainKernelTests: forward <= 1e-4 absolute,
    all seven gradients <= 1e-3 relative to autograd of the unrolled recurrence."""
    from swiftrwkv_b200 import kernel as K
    g = golden("wkv7_autograd.npz")
    names = ("r", "w", "k", "v", "a", "b", "h0")
    ts = [dev(g[n]).requires_grad_(True) for n in names]
    out, h_out = K.wkv7TrainWithState(*ts)
    loss = (out * dev(g["dy"])).sum() + (h_out * dev(g["dh_out"])).sum()
    loss.backward()
    assert np.abs(host(out) - g["y"]).max() < 1e-4
    assert np.abs(host(h_out) - g["h_out"]).max() < 1e-4
    for n, t in zip(names, ts):
        assert rel_err(host(t.grad), g["d" + n]) < 1e-3, n


def test_train_forward_bitwise_equals_frozen_and_checkpoints(cuda, oracle, rng):
    """WKV7TrainKernelTests.swift:117-136 / WKV7StateTests: same kernel, same
    bits; checkpoints and sa agree with the oracle."""
    from swiftrwkv_b200 import kernel as K
    ins = wkv_inputs(rng, 2, 48, 3)
    y, h = K.wkv7SequenceForward(*map(dev, ins))
    y2, h2, sa, ck = K._train_forward(*map(dev, ins), None)
    assert torch.equal(y, y2) and torch.equal(h, h2)
    assert torch.equal(ck[:, :, -1], h)
    _, _, sa_ref, ck_ref = oracle.wkv7_forward(*ins, want_sa=True, ckpt_every=16)
    assert rel_err(host(sa), sa_ref) < 1e-5
    assert rel_err(host(ck), ck_ref) < 1e-5


def test_split_equals_contiguous_bitwise(cuda, rng):
    """WKV7SequenceTests.swift:50-62: a pass split through the state is the
    whole pass, bit for bit, at aligned and unaligned cuts."""
    from swiftrwkv_b200 import kernel as K
    ins = [dev(x) for x in wkv_inputs(rng, 2, 53, 3)]
    h0 = dev((rng.standard_normal((2, 3, 64, 64)) * 0.1).astype(np.float32))
    y, h = K.wkv7SequenceForward(*ins, h0)
    for cut in (16, 17, 1):
        y1, h1 = K.wkv7SequenceForward(*(x[:, :cut] for x in ins), h0)
        y2, h2 = K.wkv7SequenceForward(*(x[:, cut:] for x in ins), h1)
        assert torch.equal(torch.cat([y1, y2], 1), y)
        assert torch.equal(h2, h)


@pytest.mark.parametrize("H", [12, 3, 32])
def test_step_equals_forward_at_t1_bitwise(cuda, rng, H):
    """DecodeKernelTests.swift:27-39."""
    from swiftrwkv_b200 import kernel as K
    ins = [dev(x) for x in wkv_inputs(rng, 1, 1, H)]
    h0 = dev((rng.standard_normal((1, H, 64, 64)) * 0.1).astype(np.float32))
    y, h = K.wkv7SequenceForward(*ins, h0)
    ys, hs = K.wkv7StepForward(*(x[0, 0] for x in ins), h0[0])
    assert torch.equal(ys, y[0, 0]) and torch.equal(hs, h[0])


def test_step_many_items_equals_forward_bitwise(cuda, rng):
    """A full decode batch (64 rows x 32 heads, more CTAs than fit on the
    GPU at once): still the forward at T = 1 bit for bit."""
    from swiftrwkv_b200 import kernel as K
    rows, H = 64, 32
    ins = [dev(x) for x in wkv_inputs(rng, rows, 1, H)]
    h0 = dev((rng.standard_normal((rows, H, 64, 64)) * 0.1).astype(np.float32))
    y, h = K.wkv7SequenceForward(*ins, h0)
    ys, hs = K.wkv7StepForward(*(x[:, 0] for x in ins), h0)
    assert torch.equal(ys, y[:, 0]) and torch.equal(hs, h)


def test_step_dtype_independence(cuda, rng):
    """DecodeKernelTests.swift:43-53: the result does not depend on the input
    dtype once values are the same (bf16-exact inputs in bf16 and fp32)."""
    from swiftrwkv_b200 import kernel as K
    ins = [dev(x).to(torch.bfloat16) for x in wkv_inputs(rng, 4, 1, 8)]
    h0 = dev((rng.standard_normal((4, 8, 64, 64)) * 0.1).astype(np.float32))
    y16, h16 = K.wkv7StepForward(*(x[:, 0] for x in ins), h0)
    y32, h32 = K.wkv7StepForward(*(x[:, 0].float() for x in ins), h0)
    assert torch.equal(y16, y32) and torch.equal(h16, h32)


@pytest.mark.parametrize("rows", [5, 64])
def test_step_tail_matches_oracle(cuda, oracle, rng, rows):
    """The fused step+tail against the oracle's step followed by its tail
    (<= 1e-5), on a few rows and on a full 64-row decode batch."""
    from swiftrwkv_b200 import kernel as K
    H = 32
    ins = [x[:, 0] for x in wkv_inputs(rng, rows, 1, H)]
    h0 = (rng.standard_normal((rows, H, 64, 64)) * 0.1).astype(np.float32)
    g = rng.standard_normal((rows, H, 64)).astype(np.float32)
    rk, lnw, lnb = (rng.standard_normal(H * 64).astype(np.float32) for _ in range(3))
    y_ref, h_ref = oracle.wkv7_step(*ins, h0)
    want = oracle.wkv_tail(y_ref, ins[0], ins[2], ins[3], rk, lnw, lnb, g, H, 64)
    h = dev(h0)
    out = K.wkv7StepTail(*map(dev, ins), h, dev(rk), dev(lnw), dev(lnb), dev(g))
    assert rel_err(host(h), h_ref) < 1e-5
    assert np.abs(host(out) - want).max() < 1e-5 * max(1, np.abs(want).max())
    tail = K.wkvTail(dev(y_ref), *map(dev, (ins[0], ins[2], ins[3])), dev(rk), dev(lnw), dev(lnb),
                     dev(g), nHead=H, headSize=64, rows=rows)
    assert np.abs(host(tail) - want).max() < 1e-5 * max(1, np.abs(want).max())


@pytest.mark.parametrize("B,T,H", [(2, 64, 4), (1, 48, 3), (1, 1024, 12)])
def test_backward_matches_oracle(cuda, oracle, rng, B, T, H):
    """All seven gradients within 1e-3 relative of the oracle (config 1 shapes
    included), with a non-zero initial state and a cotangent on h_out."""
    from swiftrwkv_b200 import kernel as K
    ins = config1_inputs(rng, B, T, H) if T == 1024 else wkv_inputs(rng, B, T, H)
    h0 = (rng.standard_normal((B, H, 64, 64)) * 0.1).astype(np.float32)
    dy = rng.standard_normal((B, T, H, 64)).astype(np.float32)
    dh = (rng.standard_normal((B, H, 64, 64)) * 0.1).astype(np.float32)
    ref = oracle.wkv7_train(*ins, h0, dy, dh)
    y, h_out, sa, ck = K._train_forward(*map(dev, ins), dev(h0))
    assert rel_err(host(y), ref[0]) < 1e-4
    grads = K.wkv7Backward(*map(dev, ins), dev(h0), ck, dev(dy), dev(dh))
    for name, got, want in zip(("dr", "dw", "dk", "dv", "da", "db", "dh_in"), grads, ref[2:]):
        assert rel_err(host(got), want) < 1e-3, name


def test_backward_is_deterministic(cuda, rng):
    """WKV7KernelParityTests.swift:66-78: identical runs, identical bits."""
    from swiftrwkv_b200 import kernel as K
    ins = [dev(x) for x in wkv_inputs(rng, 2, 64, 4)]
    dy = dev(rng.standard_normal((2, 64, 4, 64)).astype(np.float32))
    _, _, _, ck = K._train_forward(*ins, None)
    g1 = K.wkv7Backward(*ins, None, ck, dy)
    g2 = K.wkv7Backward(*ins, None, ck, dy)
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)


def test_bf16_inputs_within_tolerance(cuda, oracle, rng):
    """bf16 path within 2e-2 relative of fp32 on the same (bf16-rounded) values."""
    from swiftrwkv_b200 import kernel as K
    ins = [dev(x).to(torch.bfloat16) for x in config1_inputs(rng, 1, 256, 4)]
    ref, h_ref = oracle.wkv7_forward(*(host(x) for x in ins))
    y, h = K.wkv7SequenceForward(*ins)
    assert y.dtype == torch.bfloat16
    assert rel_err(host(y), ref) < 2e-2
    assert rel_err(host(h), h_ref) < 1e-4


def test_padding_steps_are_identity(cuda, rng):
    """Right-padding neutral steps (w=1, k=0, b=0) freeze the state."""
    from swiftrwkv_b200 import kernel as K
    r, w, k, v, a, b = wkv_inputs(rng, 1, 20, 2)
    w[:, 7:] = 1.0
    k[:, 7:] = 0.0
    b[:, 7:] = 0.0
    _, h_all = K.wkv7SequenceForward(*map(dev, (r, w, k, v, a, b)))
    _, h_7 = K.wkv7SequenceForward(*(dev(x[:, :7]) for x in (r, w, k, v, a, b)))
    assert torch.equal(h_all, h_7)


def test_errors_are_raised_not_trapped(cuda):
    from swiftrwkv_b200 import kernel as K
    from swiftrwkv_b200._lib import RWKVError
    x = torch.zeros((1, 20, 2, 64), device="cuda")
    with pytest.raises(ValueError):
        K.wkv7TrainWithState(x, x, x, x, x, x)          # T % 16 != 0
    with pytest.raises(ValueError):
        K.wkv7SequenceForward(*(torch.zeros((1, 4, 2, 32), device="cuda"),) * 6)
    from swiftrwkv_b200 import _lib
    st = _lib.status("rwkv_wkv7_forward", 0, *([_lib.P(x.data_ptr())] * 6), None,
                     _lib.P(x.data_ptr() + 4), None, 1, 20, 2, 64, None)
    assert st == _lib.E_UNSUPPORTED  # misaligned output is refused, not written
    assert issubclass(RWKVError, RuntimeError)
