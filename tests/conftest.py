"""Shared fixtures.  `-m "not gpu"` runs the oracle / host-logic / ABI tests on
CPU; `-m gpu` runs the parity tests through the C ABI on a B200."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")
SEED = 0x5EED2026


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and librwkvcuda.so")


def rel_err(x, ref):
    """max|x - ref| / max|ref|, the reference's parity measure
    (WKV7KernelParityTests.swift:55-60)."""
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(x - ref).max() / (np.abs(ref).max() + 1e-12))


@pytest.fixture
def rng():
    return np.random.default_rng(SEED)


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return dict(np.load(os.path.join(GOLDEN, name)))
    return load


@pytest.fixture(scope="session")
def cuda():
    """The CUDA library on a GPU: fails (never skips) when it cannot load."""
    import torch
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    from swiftrwkv_b200 import _lib
    _lib.lib()
    return torch.device("cuda:0")


def wkv_inputs(rng, B, T, H, N=64, scale=0.5):
    """WKV-7 inputs with the model's value ranges (RWKVBlock.swift:207-219):
    kk unit-norm per head, a = -kk, b = kk*sigmoid, w = exp(-0.606531*sigmoid)."""
    def rnd(s):
        return (rng.standard_normal((B, T, H, N)) * s).astype(np.float32)
    r, v, k = rnd(scale), rnd(scale), rnd(scale)
    kk = k / np.sqrt((k * k).sum(-1, keepdims=True) + 1e-12)
    a = (-kk).astype(np.float32)
    b = (kk / (1 + np.exp(-rnd(1.0)))).astype(np.float32)
    w = np.exp(-0.606531 / (1 + np.exp(-rnd(1.0)))).astype(np.float32)
    return r, w, k, v, a, b


def config1_inputs(rng, B=1, T=1024, H=12, N=64):
    """r,k,v ~ N(0,1); w = exp(-exp(u)), u = -softplus(-z) - 0.5;
    kk ~ N(0,1) L2-normalised; a = -kk; b = kk*sigmoid(g)."""
    def n():
        return rng.standard_normal((B, T, H, N)).astype(np.float32)
    r, k, v = n(), n(), n()
    z = n()
    u = -np.logaddexp(0, -z) - 0.5
    w = np.exp(-np.exp(u)).astype(np.float32)
    kk = n()
    kk = kk / np.sqrt((kk * kk).sum(-1, keepdims=True))
    a = (-kk).astype(np.float32)
    b = (kk / (1 + np.exp(-n()))).astype(np.float32)
    return r, w, k, v, a, b
