"""rwkv_wkv7_backward_noalloc, the WKV-7 backward for hosts that cannot
allocate device memory (a framework bridge that hands the op only its own
tensors, or a process with a fixed memory budget), checked through the C ABI
against rwkv_wkv7_backward with a caller-supplied workspace.

Two calls in a row on different inputs: the second reuses the built-in scratch
the first one left behind, and both must match the workspace entry point
within the gradient tolerance of the backward parity tests (1e-3 relative).
The file name sorts last so that pytest runs it after every other test; it
also passes on its own in a fresh process.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import rel_err, wkv_inputs

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-3


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _case(rng, B, T, H):
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()
    ins = [dev(x) for x in wkv_inputs(rng, B, T, H)]
    h0 = dev((rng.standard_normal((B, H, 64, 64)) * 0.1).astype(np.float32))
    dy = dev(rng.standard_normal((B, T, H, 64)).astype(np.float32))
    dh = dev((rng.standard_normal((B, H, 64, 64)) * 0.1).astype(np.float32))
    return ins, h0, dy, dh


def _grads_like(r, B, H):
    return [torch.full_like(r, float("nan")) for _ in range(6)] + [
        torch.full((B, H, 64, 64), float("nan"), device=r.device, dtype=torch.float32)]


def _backward(noalloc, ins, h0, ck, dy, dh, B, T, H, dtype=None):
    from swiftrwkv_b200 import _lib
    out = _grads_like(ins[0], B, H)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    dtype = _lib.F32 if dtype is None else dtype
    common = (dtype, *map(_p, ins), _p(h0), _p(ck), _p(dy), _p(dh), *map(_p, out), B, T, H, 64)
    if noalloc:
        _lib.call("rwkv_wkv7_backward_noalloc", *common, st)
    else:
        ws_bytes = int(_lib.lib().rwkv_wkv7_backward_workspace_size(B, T, H, 64))
        ws = torch.empty(ws_bytes, device=ins[0].device, dtype=torch.uint8)
        _lib.call("rwkv_wkv7_backward", *common, _p(ws), ws_bytes, st)
    return out


def test_noalloc_backward_matches_workspace_backward_twice():
    from swiftrwkv_b200 import _lib, kernel as K
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    _lib.lib()
    rng = np.random.default_rng(2024)
    for B, T, H in [(2, 64, 4), (3, 48, 5)]:
        ins, h0, dy, dh = _case(rng, B, T, H)
        _, _, _, ck = K._train_forward(*ins, h0)
        want = _backward(False, ins, h0, ck, dy, dh, B, T, H)
        got = _backward(True, ins, h0, ck, dy, dh, B, T, H)
        torch.cuda.synchronize()
        for name, g, w in zip(("dr", "dw", "dk", "dv", "da", "db", "dh_in"), got, want):
            g, w = g.cpu().numpy(), w.cpu().numpy()
            assert np.isfinite(g).all(), name
            assert rel_err(g, w) < GRAD_TOL, (B, T, H, name)


def _compare(got, want, tol, what):
    torch.cuda.synchronize()
    for name, g, w in zip(("dr", "dw", "dk", "dv", "da", "db", "dh_in"), got, want):
        g, w = g.float().cpu().numpy(), w.float().cpu().numpy()
        assert np.isfinite(g).all(), (what, name)
        assert rel_err(g, w) < tol, (what, name, rel_err(g, w))


def test_noalloc_backward_bf16_matches_workspace_backward():
    """bf16 inputs and gradients (the bf16 bound of the backward, 2e-2)."""
    from swiftrwkv_b200 import _lib, kernel as K
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    _lib.lib()
    rng = np.random.default_rng(7)
    B, T, H = 2, 32, 3
    ins, h0, dy, dh = _case(rng, B, T, H)
    ins = [x.to(torch.bfloat16) for x in ins]
    dy = dy.to(torch.bfloat16)
    _, _, _, ck = K._train_forward(*ins, h0)
    want = _backward(False, ins, h0, ck, dy, dh, B, T, H, _lib.BF16)
    got = _backward(True, ins, h0, ck, dy, dh, B, T, H, _lib.BF16)
    _compare(got, want, 2e-2, "bf16")


def test_noalloc_backward_zero_state_after_a_nonzero_call():
    """h_in = NULL and dh_out = NULL (zero state, no upstream state gradient)
    right after a call with non-zero ones: the scratch keeps that call's
    states, and the zero-start call must not see them."""
    from swiftrwkv_b200 import _lib, kernel as K
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    _lib.lib()
    rng = np.random.default_rng(11)
    B, T, H = 2, 48, 4
    ins, h0, dy, dh = _case(rng, B, T, H)
    _, _, _, ck = K._train_forward(*ins, h0)
    _compare(_backward(True, ins, h0, ck, dy, dh, B, T, H), _backward(False, ins, h0, ck, dy, dh, B, T, H),
             GRAD_TOL, "non-zero state")
    ins2, _, dy2, _ = _case(rng, B, T, H)
    _, _, _, ck2 = K._train_forward(*ins2, None)
    want = _backward(False, ins2, None, ck2, dy2, None, B, T, H)
    got = _backward(True, ins2, None, ck2, dy2, None, B, T, H)
    _compare(got, want, GRAD_TOL, "zero state")


def test_noalloc_backward_rejects_more_heads_than_its_scratch():
    from swiftrwkv_b200 import _lib
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    lib = _lib.lib()
    t = torch.zeros(64, device="cuda")
    p = _p(t)
    B, H = _lib.RWKV_NOALLOC_MAX_HEADS + 1, 1
    rc = lib.rwkv_wkv7_backward_noalloc(_lib.F32, p, p, p, p, p, p, None, p, p, None, p, p, p, p, p,
                                        p, None, B, 16, H, 64, None)
    assert rc == _lib.E_SHAPE
    header = open(_lib.HEADER_PATH).read()
    assert f"#define RWKV_NOALLOC_MAX_HEADS {_lib.RWKV_NOALLOC_MAX_HEADS}\n" in header
    assert b"scratch" in lib.rwkv_last_error()
