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


def _backward(noalloc, ins, h0, ck, dy, dh, B, T, H):
    from swiftrwkv_b200 import _lib
    out = _grads_like(ins[0], B, H)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    common = (_lib.F32, *map(_p, ins), _p(h0), _p(ck), _p(dy), _p(dh), *map(_p, out), B, T, H, 64)
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
