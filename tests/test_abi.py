"""CPU tests of the C ABI: the library loads without a GPU, exports every
symbol include/rwkv_cuda.h declares, and rejects bad arguments on the host
(status codes, never a trap) before anything would launch."""
from __future__ import annotations

import ctypes

import pytest

from swiftrwkv_b200 import _lib


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = _lib.header_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert set(names) == set(_lib._SIGS), "binding table out of sync with the header"


def test_status_strings_and_version():
    L = _lib.lib()
    assert L.rwkv_version() >= 100
    assert L.rwkv_status_string(0) == b"ok"
    assert L.rwkv_status_string(-4) == b"unsupported"


FAKE = ctypes.c_void_p(0x1000)  # aligned, never dereferenced: checks fail first


def _wkv_args(N=64, T=4, dtype=0):
    return [dtype] + [FAKE] * 6 + [None, FAKE, None, 1, T, 2, N, None]


def test_wkv_forward_rejects_bad_arguments():
    s = _lib.status
    args = _wkv_args()
    args[1] = None
    assert s("rwkv_wkv7_forward", *args) == _lib.E_NULL
    assert b"NULL" in _lib.lib().rwkv_last_error()
    assert s("rwkv_wkv7_forward", *_wkv_args(N=32)) == _lib.E_UNSUPPORTED
    assert s("rwkv_wkv7_forward", *_wkv_args(T=0)) == _lib.E_SHAPE
    assert s("rwkv_wkv7_forward", *_wkv_args(dtype=7)) == _lib.E_DTYPE
    args = _wkv_args()
    args[2] = ctypes.c_void_p(0x1004)
    assert s("rwkv_wkv7_forward", *args) == _lib.E_UNSUPPORTED


def test_train_and_backward_require_chunk_multiple_and_workspace():
    s = _lib.status
    tf = [0] + [FAKE] * 6 + [None, FAKE, None, None, FAKE, 1, 20, 2, 64, None]
    assert s("rwkv_wkv7_train_forward", *tf) == _lib.E_SHAPE  # T % 16
    need = _lib.lib().rwkv_wkv7_backward_workspace_size(1, 32, 2, 64)
    assert need == 1 * 2 * 17 * 64 * 64 * 4
    bw = [0] + [FAKE] * 6 + [None, FAKE, FAKE, None] + [FAKE] * 6 + [None, 1, 32, 2, 64, FAKE,
                                                                  need - 1, None]
    assert s("rwkv_wkv7_backward", *bw) == _lib.E_WORKSPACE
    bw[-3] = None
    bw[-2] = need
    assert s("rwkv_wkv7_backward", *bw) == _lib.E_WORKSPACE


@pytest.mark.parametrize("bits,group,IN,code", [
    (7, 64, 2048, _lib.E_UNSUPPORTED),
    (4, 48, 2048, _lib.E_UNSUPPORTED),
    (4, 64, 2000, _lib.E_SHAPE),
])
def test_q_gemm_rejects_unsupported_formats(bits, group, IN, code):
    args = [2, FAKE, FAKE, FAKE, FAKE, 2, 0, FAKE, 1, 128, IN, group, bits, None]
    assert _lib.status("rwkv_q_gemm", *args) == code


def test_sb6_and_sym_shape_rules():
    s = _lib.status
    # sb6 needs IN % 256 (RwkvqSb6GEMV.swift:74)
    assert s("rwkv_sb6_gemv", 0, FAKE, FAKE, FAKE, FAKE, FAKE, 1, 16, 128, 0, None) == _lib.E_UNSUPPORTED
    assert s("rwkv_sb6_gemv", 0, FAKE, FAKE, FAKE, FAKE, FAKE, 1, 16, 256, 3, None) == _lib.E_SHAPE
    # sym bits in {6, 8}; fused rows must split evenly
    assert s("rwkv_sym_gemv", 0, FAKE, FAKE, FAKE, FAKE, FAKE, 1, 16, 256, 7, 16, None) == _lib.E_SHAPE
    assert s("rwkv_sym_gemv", 0, FAKE, FAKE, FAKE, FAKE, FAKE, 1, 48, 256, 8, 20, None) == _lib.E_UNSUPPORTED
    # the off-superblock sym dequant is taken (IN = 48), as the reference's chain does
    assert s("rwkv_sym_dequant", FAKE, FAKE, FAKE, 0, None, 2, 48, 8, None) == _lib.E_NULL


def test_tail_requires_warp_multiple_head():
    args = [FAKE] * 9 + [1, 2, 48, ctypes.c_float(64e-5), None]
    assert _lib.status("rwkv_wkv_tail", *args) == _lib.E_UNSUPPORTED


def test_wkv7_step_api_validates_shapes_before_any_launch():
    """wkv7Step / wkv7Steps reject bad ranks and lengths on the host (the
    reference's preconditions, WKV7Step.swift:49-57, :85)."""
    import torch
    from swiftrwkv_b200 import kernel as K
    x3 = torch.zeros(1, 2, 64)
    with pytest.raises(ValueError, match="exactly one token"):
        K.wkv7Step(*(torch.zeros(1, 2, 2, 64) for _ in range(6)))
    with pytest.raises(ValueError, match="expects"):
        K.wkv7Step(*(torch.zeros(64) for _ in range(6)))
    with pytest.raises(ValueError, match="expects"):
        K.wkv7Steps(*(x3 for _ in range(6)))
    with pytest.raises(ValueError, match="every input"):
        K.wkv7Steps(torch.zeros(1, 3, 2, 64), *(torch.zeros(1, 2, 2, 64) for _ in range(5)))


def test_projection_backward_validates_before_any_launch():
    """rwkv_gemm_dx / rwkv_q_gemm_dx: bf16 cotangent only, fp32 dX for
    accumulation, IN % 128 and OUT % 64, 4-bit group 64 with fp16 scales."""
    s = _lib.status
    F32, BF16, F16 = _lib.F32, _lib.BF16, _lib.F16
    dense = lambda dyt=BF16, wt=BF16, dxt=F32, rows=16, OUT=256, IN=256, acc=0: s(
        "rwkv_gemm_dx", dyt, FAKE, wt, FAKE, dxt, FAKE, rows, OUT, IN, acc, None)
    assert dense(dyt=F32) == _lib.E_DTYPE          # the host casts the cotangent to bf16
    assert dense(wt=F16) == _lib.E_DTYPE
    assert dense(dxt=BF16, acc=1) == _lib.E_DTYPE  # accumulation into fp32 only
    assert dense(dxt=9) == _lib.E_DTYPE
    assert dense(rows=0) == _lib.E_SHAPE
    assert dense(IN=200) == _lib.E_UNSUPPORTED
    assert dense(OUT=96) == _lib.E_UNSUPPORTED
    assert s("rwkv_gemm_dx", BF16, None, BF16, FAKE, F32, FAKE, 1, 64, 128, 0, None) == _lib.E_NULL
    q = lambda group=64, bits=4, sdt=F16: s("rwkv_q_gemm_dx", BF16, FAKE, FAKE, FAKE, FAKE, sdt, F32, FAKE,
                                          8, 256, 256, group, bits, 0, None)
    assert q(group=32) == _lib.E_UNSUPPORTED
    assert q(bits=8) == _lib.E_UNSUPPORTED
    assert q(sdt=BF16) == _lib.E_UNSUPPORTED
