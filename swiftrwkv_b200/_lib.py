"""ctypes binding of librwkvcuda.so (the C ABI in include/rwkv_cuda.h).

The library is loaded from this package directory.  There is no fallback: if
the shared object is missing or was built without a kernel, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librwkvcuda.so")
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "rwkv_cuda.h")

OK, E_NULL, E_SHAPE, E_DTYPE, E_UNSUPPORTED, E_CUDA, E_TIMEOUT, E_WORKSPACE = 0, -1, -2, -3, -4, -5, -6, -7
F32, BF16, F16 = 0, 1, 2
RWKV_NOALLOC_MAX_HEADS = 240  # rwkv_cuda.h: (batch, head) pairs of rwkv_wkv7_backward_noalloc


class RWKVError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed with status {status}: {msg}")
        self.status = status
        self.fn = fn


P = ctypes.c_void_p
I = ctypes.c_int
I64 = ctypes.c_int64
F = ctypes.c_float

# name -> argtypes (restype int unless listed in _RESTYPES)
_SIGS = {
    "rwkv_version": [],
    "rwkv_status_string": [I],
    "rwkv_last_error": [],
    "rwkv_wkv7_forward": [I, P, P, P, P, P, P, P, P, P, I, I, I, I, P],
    "rwkv_wkv7_train_forward": [I, P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, P],
    "rwkv_wkv7_forward_chunked_workspace_size": [I, I, I, I],
    "rwkv_wkv7_forward_chunked": [I, P, P, P, P, P, P, P, P, P, P, I, I, I, I, P, I64, P],
    "rwkv_wkv7_train_forward_chunked": [I, P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, P, I64, P],
    "rwkv_wkv7_backward_workspace_size": [I, I, I, I],
    "rwkv_wkv7_backward_chunked_workspace_size": [I, I, I, I],
    "rwkv_wkv7_backward_chunked": [I, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, P, I64, P],
    "rwkv_wkv7_backward": [I, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, P, I64, P],
    "rwkv_wkv7_backward_noalloc": [I, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, P],
    "rwkv_wkv7_step": [I, P, P, P, P, P, P, P, P, I, I, I, P],
    "rwkv_wkv_tail": [P, P, P, P, P, P, P, P, P, I, I, I, F, P],
    "rwkv_wkv7_step_tail": [P, P, P, P, P, P, P, P, P, P, P, P, I, I, I, F, P],
    "rwkv_q_gemm": [I, P, P, P, P, I, I, P, I, I, I, I, I, P],
    "rwkv_q_gemm_status": [P],
    "rwkv_q_gemm_inject_wait_error": [I, P],
    "rwkv_gemm_dx": [I, P, I, P, I, P, I, I, I, I, P],
    "rwkv_x070_set_param_rwkvq": [P, ctypes.c_char_p, I, I, P, I64, P, I64, P, I64],
    "rwkv_q_gemm_dx": [I, P, P, P, P, I, I, P, I, I, I, I, I, I, P],
    "rwkv_q_dequant": [P, P, P, I, I, P, I, I, I, I, P],
    "rwkv_q_rows": [P, I, P, P, P, I, I, P, I, I, I, I, P],
    "rwkv_q_quantize": [I, P, P, P, P, I, I, I, I, P],
    "rwkv_sb6_dequant": [P, P, P, I, P, I, I, I, P],
    "rwkv_sb6_gemv": [I, P, P, P, P, P, I, I, I, I, P],
    "rwkv_sb6_to_affine": [P, P, P, P, P, P, P, I, I, I, P],
    "rwkv_sym_dequant": [P, P, P, I, P, I, I, I, P],
    "rwkv_sym_gemv": [I, P, P, P, P, P, I, I, I, I, I, P],
    "rwkv_sym_rows": [P, I, P, P, P, P, I, I, P],
    "rwkv_x070_create": [P, P],
    "rwkv_x070_destroy": [P],
    "rwkv_x070_set_param": [P, ctypes.c_char_p, P, I64],
    "rwkv_x070_init_random": [P, ctypes.c_uint64],
    "rwkv_x070_reset_state": [P, I, P],
    "rwkv_x070_step": [P, P, I, P, P, I, P],
    "rwkv_x070_generate": [P, P, I, I, I, P, P],
    "rwkv_x070_prefill": [P, P, P, I, I, P, P, P],
    "rwkv_x070_generate_batch": [P, P, P, I, I, I, P, I, P, P, P],
    "rwkv_x070_profile_step": [P, I, P, I, P, I, P, P],
    "rwkv_x070_status": [P, P],
    "rwkv_x070_inject_wait_error": [P, I, P],
    "rwkv_x070_weight_bytes": [P],
    "rwkv_x070_set_decode_path": [P, I],
    "rwkv_x070_trace": [P, P, I, P],
    "rwkv_x070_decode_path": [P, I],
    "rwkv_x070_launches_per_step": [P],
    "rwkv_state_broadcast": [P, P, I, I, I, P],
    "rwkv_state_grad_sum": [P, P, I, I, I, I, P],
    "rwkv_adamw_workspace_size": [I64],
    "rwkv_adamw_clip_step": [P, P, P, P, I64, F, F, F, F, F, F, F, F, F, P, P, I64, P],
}
_RESTYPES = {
    "rwkv_status_string": ctypes.c_char_p,
    "rwkv_last_error": ctypes.c_char_p,
    "rwkv_wkv7_backward_workspace_size": I64,
    "rwkv_wkv7_forward_chunked_workspace_size": I64,
    "rwkv_wkv7_backward_chunked_workspace_size": I64,
    "rwkv_x070_weight_bytes": I64,
    "rwkv_adamw_workspace_size": I64,
}

_lib = None


def header_functions() -> list[str]:
    """Names of every function declared in include/rwkv_cuda.h."""
    with open(HEADER_PATH) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rwkv_[a-z0-9_]+)\s*\(", text)))


def lib() -> ctypes.CDLL:
    """Load librwkvcuda.so (once) and set every declared signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"librwkvcuda.so not found at {LIB_PATH}: build it with "
            "`python -m swiftrwkv_b200.build` (there is no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    for name, args in _SIGS.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, I)
    _lib = L
    return L


def call(name: str, *args) -> int:
    """Call an entry point; raise RWKVError on a non-zero status."""
    L = lib()
    st = getattr(L, name)(*args)
    if st != OK:
        msg = L.rwkv_last_error().decode()
        raise RWKVError(name, st, msg)
    return st


def status(name: str, *args) -> int:
    """Call an entry point and return its status without raising."""
    return getattr(lib(), name)(*args)
