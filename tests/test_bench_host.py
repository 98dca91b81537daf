"""Host-side pieces of bench.py (no GPU): the CPU baseline's projection
dispatch over the three weight containers, the .rwkvq decode bases, and the
traffic table lookup that feeds the roofline's `traffic` figure."""
from __future__ import annotations

import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def test_cpu_gemv_dispatches_on_the_container(oracle, rng):
    """_cpu_gemv on a 4-bit affine tuple, an sb6 and a sym matrix equals the
    exact product of the oracle's dequantised weight."""
    OUT, IN = 32, 256
    x = rng.standard_normal((2, IN)).astype(np.float32)
    W = (rng.standard_normal((OUT, IN)) * 0.02).astype(np.float16).astype(np.float32)
    wq, sc, bi = oracle.affine_quantize(W)
    got = bench._cpu_gemv(x, (wq, sc, bi))
    want = x.astype(np.float64) @ oracle.affine_dequant(wq, sc.view(np.float16), bi.view(np.float16)).T
    assert np.abs(got - want).max() <= 2e-5 * np.abs(want).max()

    NB = IN // 32
    qblk = rng.integers(0, 256, (OUT, NB * 20), dtype=np.uint8)
    qsqm = rng.integers(0, 64, (OUT, NB * 2), dtype=np.uint8)
    ddm = (rng.random((OUT, NB // 8 * 2)) * 1e-3).astype(np.float16).view(np.uint16)
    got = bench._cpu_gemv(x, ("sb6", qblk, qsqm, ddm, OUT, IN, 1))
    want = x.astype(np.float64) @ oracle.sb6_dequant(qblk, qsqm, ddm, OUT, IN, 1).astype(np.float64).T
    assert got.shape == (2, OUT)
    assert np.abs(got - want).max() <= 2e-5 * np.abs(want).max()

    qblk = rng.integers(0, 256, OUT * IN // 32 * 24, dtype=np.uint8)
    qs = rng.integers(0, 128, OUT * IN // 16, dtype=np.uint8)
    d = (rng.random(OUT * (IN // 256)) * 1e-4).astype(np.float16).view(np.uint16)
    got = bench._cpu_gemv(x, ("sym", qblk, qs, d, OUT, IN, 6))
    want = x.astype(np.float64) @ oracle.sym_dequant(qblk, qs, d, OUT, IN, 6).astype(np.float64).T
    assert np.abs(got - want).max() <= 2e-5 * np.abs(want).max()


def test_decode_bases_and_metric():
    assert set(bench.Decode15B.BASES) == {"q4", "sb6", "sym6", "sym8"}
    assert "4-bit" in bench.Decode15B(rows=1).metric
    wl = bench.Decode15B(rows=1, base="sb6")
    assert wl.rq_kind == "sb6" and wl.rq_bits == 1 and "sb6" in wl.metric
    wl = bench.Decode15B(rows=1, base="sym8")
    assert wl.rq_kind == "sym" and wl.rq_bits == 8
    # every projection of the 24 layers and the head, once
    names = [k for k, _, _ in bench.Decode15B(rows=1)._matrices()]
    assert len(names) == len(set(names)) == 24 * 6 + 1 and names[-1] == "head.weight"


def test_rwkvq_bytes_match_the_runtime_buffers():
    """The algorithmic bytes the bench counts for a .rwkvq matrix are the three
    buffers rwkv_x070_set_param_rwkvq takes for it."""
    OUT, IN = 2048, 8192
    for bits in (0, 1, 2):
        NB = IN // 32
        want = OUT * NB * (16 + 4 * bits) + OUT * NB * 2 + OUT * (IN // 256) * 4
        assert bench.RwkvqGemvSuite.wbytes("sb6", bits, OUT, IN) == want
    for bits in (6, 8):
        code = OUT * IN if bits == 8 else OUT * (IN // 32) * 24
        want = code + OUT * (IN // 16) + OUT * (IN // 256) * 2
        assert bench.RwkvqGemvSuite.wbytes("sym", bits, OUT, IN) == want


class _W:
    def __init__(self, name, rows, rq_kind=None, persistent=False):
        self.name, self.rows, self.rq_kind, self.persistent = name, rows, rq_kind, persistent


def test_traffic_lookup_covers_the_captured_kernels_only():
    assert bench.measured_traffic(_W("decode", 64)) > 0
    assert bench.measured_traffic(_W("decode", 1)) > 0
    assert bench.measured_traffic(_W("gemv", 1)) > 0
    assert bench.measured_traffic(_W("decode", 1, rq_kind="sb6")) is None
    assert bench.measured_traffic(_W("decode", 64, persistent=True)) is None
    assert bench.measured_traffic(_W("decode", 3)) is None
