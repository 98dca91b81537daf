"""Reporting of a tensor-core GEMM wait that gave up, without a device fault.

The tcgen05 GEMM's pipeline waits are bounded in time; a wait that gives up
sets a device flag (which the other roles watch, so the launch winds down) and
a mapped host record.  These tests set the flag from the host instead of
making a wait run out:
  * host record set: the next call reports RWKV_E_TIMEOUT once, clears it and
    launches nothing; the call after that is correct;
  * device flag only: the next launch finds it at entry, every role skips its
    work (no copies, no MMAs, no output), the launch ends and records it; the
    status query reports it and clears it; the next call is correct.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _gemm_case(oracle, rng, rows=64, OUT=2048, IN=2048):
    from test_quant_gpu import dev, make_affine, want_gemm
    W, wq, sc, bi = make_affine(oracle, rng, OUT, IN)
    x = (rng.standard_normal((rows, IN))).astype(np.float16)
    want = want_gemm(oracle, x, wq, sc, bi)
    t = (dev(x), dev(wq.view(np.int32)), dev(sc.view(np.float16)), dev(bi.view(np.float16)))
    y = torch.empty((rows, OUT), device="cuda", dtype=torch.float32)
    return t, y, want


def _q_gemm(t, y, rows, OUT, IN):
    from swiftrwkv_b200 import _lib
    P = _lib.P
    st = P(torch.cuda.current_stream().cuda_stream)
    x, wq, sc, bi = t
    return _lib.status("rwkv_q_gemm", 2, P(x.data_ptr()), P(wq.data_ptr()), P(sc.data_ptr()),
                       P(bi.data_ptr()), 2, 0, P(y.data_ptr()), rows, OUT, IN, 64, 4, st)


def test_q_gemm_reports_a_recorded_wait_error_once(cuda, oracle, rng):
    from swiftrwkv_b200 import _lib
    rows, OUT, IN = 64, 2048, 2048
    t, y, want = _gemm_case(oracle, rng, rows, OUT, IN)
    st = _lib.P(torch.cuda.current_stream().cuda_stream)
    assert _q_gemm(t, y, rows, OUT, IN) == _lib.OK          # sets up the per-device record
    assert _lib.status("rwkv_q_gemm_status", st) == _lib.OK
    _lib.call("rwkv_q_gemm_inject_wait_error", 1, st)
    y.fill_(float("nan"))
    assert _q_gemm(t, y, rows, OUT, IN) == _lib.E_TIMEOUT
    torch.cuda.synchronize()
    assert torch.isnan(y).all(), "the reporting call launched nothing"
    assert _q_gemm(t, y, rows, OUT, IN) == _lib.OK
    assert _lib.status("rwkv_q_gemm_status", st) == _lib.OK
    assert rel_err(y.cpu().numpy(), want) < 2e-5


def test_q_gemm_launch_with_the_flag_set_skips_and_is_reported(cuda, oracle, rng):
    from swiftrwkv_b200 import _lib
    rows, OUT, IN = 64, 2048, 8192          # split-K cluster path
    t, y, want = _gemm_case(oracle, rng, rows, OUT, IN)
    st = _lib.P(torch.cuda.current_stream().cuda_stream)
    assert _q_gemm(t, y, rows, OUT, IN) == _lib.OK
    assert _lib.status("rwkv_q_gemm_status", st) == _lib.OK
    _lib.call("rwkv_q_gemm_inject_wait_error", 0, st)       # device flag only
    y.fill_(float("nan"))
    assert _q_gemm(t, y, rows, OUT, IN) == _lib.OK          # launched; the kernel finds the flag
    assert _lib.status("rwkv_q_gemm_status", st) == _lib.E_TIMEOUT
    assert torch.isnan(y).all(), "a launch that found the flag set wrote no output"
    assert _lib.status("rwkv_q_gemm_status", st) == _lib.OK  # cleared
    for _ in range(2):
        assert _q_gemm(t, y, rows, OUT, IN) == _lib.OK
        assert _lib.status("rwkv_q_gemm_status", st) == _lib.OK
        assert rel_err(y.cpu().numpy(), want) < 2e-5


def _tiny_wide(rows=20):
    from test_x070_gpu import tiny
    return tiny("f16", rows=rows, n_embd=256, vocab=200, seed=7)


def test_x070_step_reports_a_wait_error_and_recovers(cuda):
    """More than 8 rows: the step's GEMMs are tcgen05 launches."""
    from oracle import x070_oracle as XO
    from swiftrwkv_b200 import _lib
    rows = 20
    m, ref = _tiny_wide(rows)
    ids = XO.splitmix_ids(rows, 3, vocab=200)
    s = torch.cuda.Stream()
    P = _lib.P
    with torch.cuda.stream(s):
        st = P(s.cuda_stream)
        # host record: the next step reports it and runs nothing
        m.reset(rows)
        _lib.call("rwkv_x070_inject_wait_error", m.h, 1, st)
        with pytest.raises(_lib.RWKVError) as e:
            m.step(torch.from_numpy(ids[:, 0]).cuda(), use_graph=True)
        assert e.value.status == _lib.E_TIMEOUT
        assert _lib.status("rwkv_x070_status", m.h, st) == _lib.OK
        # device flag only: the captured step's GEMM launches skip; the status
        # query reports it
        _lib.call("rwkv_x070_inject_wait_error", m.h, 0, st)
        m.step(torch.from_numpy(ids[:, 0]).cuda(), use_graph=True)
        assert _lib.status("rwkv_x070_status", m.h, st) == _lib.E_TIMEOUT
        assert _lib.status("rwkv_x070_status", m.h, st) == _lib.OK
        # after the report the model is correct again from a fresh state
        m.reset(rows)
        got = [m.step(torch.from_numpy(ids[:, t]).cuda(), use_graph=True) for t in range(3)]
        assert _lib.status("rwkv_x070_status", m.h, st) == _lib.OK
    s.synchronize()
    st_ref = ref.new_state(rows)
    for t in range(3):
        want = ref.step(ids[:, t], st_ref)
        assert rel_err(got[t].cpu().numpy(), want) < 2e-3, (t, rel_err(got[t].cpu().numpy(), want))
