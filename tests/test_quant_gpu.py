"""GPU parity of the quantised-weight kernels against the oracle, through the
C ABI: bit-exact for codes, scales and unpacked weights; the reference's
2e-5 relative bound (RwkvqSb6GEMVTests.swift:53-77) for GEMVs against the
exact product of the kernel's own dequantised weight."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def host(t):
    return t.detach().cpu().numpy()


def f16(x):
    return x.astype(np.float16)


def make_affine(oracle, rng, OUT, IN, group=64, bits=4):
    W = f16(rng.standard_normal((OUT, IN)) * 0.02)
    wq, sc, bi = oracle.affine_quantize(W.astype(np.float32), group, bits)
    return W, wq, sc, bi


def want_gemm(oracle, x, wq, sc, bi, group=64, bits=4):
    """What rwkv_q_gemm computes for fp16 x: up to 8 rows the exact product of
    the dequantised weight (MLX's quantized matrix-vector numerics); above 8
    rows, on the 4-bit group-64 tensor-core path, the exact product of the
    weight dequantised into fp16 (MLX's quantized matmul dequantises into the
    activation type)."""
    rows = x.shape[0]
    if rows <= 8 or not (bits == 4 and group == 64):
        return oracle.affine_gemv(x.astype(np.float32), wq, sc, bi, group, bits, exact=True)
    w16 = oracle.affine_dequant(wq, sc, bi, group, bits).astype(np.float16).astype(np.float64)
    return x.astype(np.float64) @ w16.T


# BASELINE config 2 matrices (OUT x IN) and a small odd one
MATS = [(2048, 2048), (8192, 2048), (2048, 8192), (65536, 2048), (48, 320)]


@pytest.mark.parametrize("bits,group", [(4, 64), (4, 32), (4, 128), (8, 64), (2, 64)])
def test_quantize_bit_exact(cuda, oracle, rng, bits, group):
    from swiftrwkv_b200 import quant as Q
    W = f16(rng.standard_normal((256, 1024)) * 0.02)
    wq, sc, bi = Q.quantized(dev(W), group, bits)
    owq, osc, obi = oracle.affine_quantize(W.astype(np.float32), group, bits)
    assert np.array_equal(host(wq).view(np.uint32), owq)
    assert np.array_equal(host(sc).view(np.uint16), osc)
    assert np.array_equal(host(bi).view(np.uint16), obi)


@pytest.mark.parametrize("bits", [4, 8, 5, 6, 3])
def test_dequant_bit_exact(cuda, oracle, rng, bits):
    from swiftrwkv_b200 import quant as Q
    OUT, IN, group = 64, 512, 64
    wq = rng.integers(0, 2**32, (OUT, IN * bits // 32), dtype=np.uint64).astype(np.uint32)
    sc = f16(rng.standard_normal((OUT, IN // group)) * 0.01)
    bi = f16(rng.standard_normal((OUT, IN // group)) * 0.05)
    want = oracle.affine_dequant(wq, sc.view(np.uint16), bi.view(np.uint16), group, bits)
    args = (dev(wq.view(np.int32)), dev(sc), dev(bi), group, bits)
    got = Q.dequantized(*args, dtype=torch.float32)
    assert np.array_equal(host(got), want)
    got16 = Q.dequantized(*args, dtype=torch.float16)
    assert np.array_equal(host(got16), f16(want))
    gotbf = Q.dequantized(*args, dtype=torch.bfloat16)
    assert torch.equal(gotbf, torch.from_numpy(want).to(torch.bfloat16).cuda())


@pytest.mark.parametrize("OUT,IN", MATS + [(100, 768), (16, 128), (300, 16384)])
@pytest.mark.parametrize("rows", [1, 2, 8])
def test_gemv_matches_exact_product(cuda, oracle, rng, OUT, IN, rows):
    """fp16 activations, W ~ N(0, 0.02) quantised 4-bit g64.
    1 and 2 rows take the streaming CUDA-core GEMV (row blocks off the grid,
    fewer than 16 units per row, one window), 8 rows the mma.sync GEMV."""
    from swiftrwkv_b200 import quant as Q
    W, wq, sc, bi = make_affine(oracle, rng, OUT, IN)
    x = f16(rng.standard_normal((rows, IN)))
    y = Q.quantizedMM(dev(x), dev(wq.view(np.int32)), dev(sc.view(np.float16)),
                      dev(bi.view(np.float16)), out_dtype=torch.float32)
    want = oracle.affine_gemv(x.astype(np.float32), wq, sc, bi, exact=True)
    assert rel_err(host(y), want) < 2e-5


@pytest.mark.parametrize("rows", [1, 3, 8, 13, 64])
@pytest.mark.parametrize("bits,group", [(4, 64), (8, 32), (5, 32)])
def test_gemm_rows_and_formats(cuda, oracle, rng, rows, bits, group):
    from swiftrwkv_b200 import quant as Q
    OUT, IN = 96, 512
    W, wq, sc, bi = make_affine(oracle, rng, OUT, IN, group, bits)
    x = f16(rng.standard_normal((rows, IN)))
    y = Q.quantizedMM(dev(x), dev(wq.view(np.int32)), dev(sc.view(np.float16)),
                      dev(bi.view(np.float16)), True, group, bits, out_dtype=torch.float32)
    want = want_gemm(oracle, x, wq, sc, bi, group, bits)
    assert rel_err(host(y), want) < 2e-5
    y16 = Q.quantizedMM(dev(x), dev(wq.view(np.int32)), dev(sc.view(np.float16)),
                        dev(bi.view(np.float16)), True, group, bits)
    assert y16.dtype == torch.float16 and rel_err(host(y16).astype(np.float32), want) < 1e-3


def test_quantized_rows(cuda, oracle, rng):
    from swiftrwkv_b200 import quant as Q
    V, C = 1000, 256
    W, wq, sc, bi = make_affine(oracle, rng, V, C)
    dense = oracle.affine_dequant(wq, sc, bi)
    ids = rng.integers(0, V, 37).astype(np.int32)
    qb = Q.QuantBase(dev(wq.view(np.int32)), dev(sc.view(np.float16)), dev(bi.view(np.float16)), 64, 4)
    rows = Q.quantized_rows(dev(ids), qb, dtype=torch.float32)
    assert np.array_equal(host(rows), dense[ids])


# ------------------------------------------------------------------ sb6 / sym

def make_sb6(rng, OUT, IN, xbits):
    NB = IN // 32
    qblk = rng.integers(0, 256, (OUT, NB * (16 + 4 * xbits)), dtype=np.uint8)
    qsqm = np.empty((OUT, NB * 2), np.uint8)
    qsqm[:, 0::2] = rng.integers(0, 64, (OUT, NB))
    qsqm[:, 1::2] = rng.integers(-31, 32, (OUT, NB)).astype(np.int8).view(np.uint8)
    ddm = f16(np.abs(rng.standard_normal((OUT, NB // 8 * 2))) * 1e-3).view(np.uint16)
    ddm[:, 1::2] = f16(np.abs(rng.standard_normal((OUT, NB // 8))) * 1e-3).view(np.uint16)
    return qblk, qsqm, ddm


@pytest.mark.parametrize("xbits", [0, 1, 2])
def test_sb6_dequant_gemv_relayout(cuda, oracle, rng, xbits):
    from swiftrwkv_b200 import quant as Q
    OUT, IN = 256, 2048
    qblk, qsqm, ddm = make_sb6(rng, OUT, IN, xbits)
    want = oracle.sb6_dequant(qblk, qsqm, ddm, OUT, IN, xbits)
    args = (dev(qblk), dev(qsqm), dev(ddm.view(np.float16)))
    got = Q.rwkvqDequantDense(*args, OUT, IN, 8, xbits)
    assert np.array_equal(host(got), want)
    got16 = Q.rwkvqDequantDense(*args, OUT, IN, 8, xbits, dtype=torch.float16)
    assert np.array_equal(host(got16), f16(want))
    for rows in (1, 3):
        x = rng.standard_normal((rows, IN)).astype(np.float32)
        y = Q.rwkvqSb6GEMV(dev(x), *args, OUT, IN, xbits)
        exact = x.astype(np.float64) @ want.astype(np.float64).T
        assert rel_err(host(y), exact) < 2e-5
    wq, sc, bi, ok = oracle.sb6_to_affine(qblk, qsqm, ddm, OUT, IN, xbits)
    nat = Q.nativeAffine(*args, OUT, IN, xbits)
    assert np.array_equal(host(nat.wq).view(np.uint32), wq)
    assert (nat.scales.dtype == torch.float16) == ok
    assert np.array_equal(host(nat.scales.float()), sc if not ok else f16(sc).astype(np.float32))


def test_sb6_kat(cuda, golden):
    from swiftrwkv_b200 import quant as Q
    g = golden("kat_sb6.npz")
    ddm = dev(g["ddm"].view(np.float16))
    live = Q.nativeAffine(dev(g["qblk_live"]), dev(g["qsqm_live"]), ddm, 2, 256, 0)
    assert live.scales.dtype == torch.float32
    assert float(live.scales[0, 3]) == np.float32(1e-8)
    assert float(live.scales[1, 3]) == float(g["scale_row1_blk3"])
    dead = Q.nativeAffine(dev(g["qblk_dead"]), dev(g["qsqm_dead"]), ddm, 2, 256, 0)
    assert dead.scales.dtype == torch.float16 and float(dead.scales[0, 3]) == 0.0


def make_sym(rng, OUT, IN, bits):
    if bits == 8:
        qblk = rng.integers(-127, 128, (OUT, IN)).astype(np.int8).view(np.uint8)
    else:
        qblk = rng.integers(0, 256, (OUT, IN // 32 * 24), dtype=np.uint8)
    qs = rng.integers(-127, 128, (OUT, IN // 16)).astype(np.int8).view(np.uint8)
    d = f16(np.abs(rng.standard_normal((OUT, (IN + 255) // 256))) * 1e-4).view(np.uint16)
    return qblk, qs, d


@pytest.mark.parametrize("bits", [6, 8])
def test_sym_dequant_and_gemv(cuda, oracle, rng, bits):
    from swiftrwkv_b200 import quant as Q
    OUT, IN = 192, 1024
    qblk, qs, d = make_sym(rng, OUT, IN, bits)
    args = (dev(qblk), dev(qs), dev(d.view(np.float16)))
    for odt, tdt in ((oracle.F32, torch.float32), (oracle.F16, torch.float16), (oracle.BF16, torch.bfloat16)):
        want = oracle.sym_dequant(qblk, qs, d, OUT, IN, bits, odt)
        got = Q.rwkvqDequantSym(*args, OUT, IN, bits, dtype=tdt)
        got_bits = host(got) if tdt == torch.float32 else host(got.view(torch.int16)).view(np.uint16)
        assert np.array_equal(got_bits, want), tdt
    dense = oracle.sym_dequant(qblk, qs, d, OUT, IN, bits, oracle.F32)
    x = rng.standard_normal((3, IN)).astype(np.float32)
    y = Q.rwkvqSymGEMV(dev(x), *args, OUT, IN, bits)
    assert rel_err(host(y), x.astype(np.float64) @ dense.astype(np.float64).T) < 2e-5
    assert rel_err(host(y), oracle.sym_gemv(x, qblk, qs, d, OUT, IN, bits)) < 2e-5


def test_sym_fused_equals_separate_bitwise(cuda, rng):
    """RwkvqSymGEMVTests.swift:164-201: fused r/k/v == three separate calls."""
    from swiftrwkv_b200 import quant as Q
    OUT, IN, K = 256, 1024, 3
    mats = [make_sym(rng, OUT, IN, 6) for _ in range(K)]
    xs = rng.standard_normal((K, IN)).astype(np.float32)
    sep = [Q.rwkvqSymGEMV(dev(xs[i:i + 1]), dev(m[0]), dev(m[1]), dev(m[2].view(np.float16)),
                          OUT, IN, 6) for i, m in enumerate(mats)]
    cat = [dev(np.concatenate([m[j] for m in mats])) for j in range(3)]
    fused = Q.symGEMVFused(dev(xs), cat[0], cat[1], cat[2].view(torch.float16), OUT, IN, 6)
    for i in range(K):
        assert torch.equal(fused[i], sep[i][0])


def test_sym_kat_and_rows(cuda, oracle, golden, rng):
    from swiftrwkv_b200 import quant as Q
    g = golden("kat_sym.npz")
    got = Q.rwkvqDequantSym(dev(g["codes"]), dev(g["qs"]), dev(g["d"].view(np.float16)), 2, 48, 8)
    assert np.array_equal(host(got), g["want"])
    V, C = 500, 768
    codes, qs, d = make_sym(rng, V, C, 8)
    table = Q.RwkvqSymRowTable(dev(codes), dev(qs), dev(d.view(np.float16)), V, C)
    ids = rng.integers(0, V, 19).astype(np.int32)
    rows = table.rows(dev(ids))
    assert np.array_equal(host(rows.view(torch.int16)).view(np.uint16),
                          oracle.sym_rows(ids, codes, qs, d, C))
    assert torch.equal(rows, table.dense()[dev(ids).long()])


@pytest.mark.parametrize("OUT,IN", [(96, 64), (2048, 2048), (300, 8192), (8192, 2048)])
@pytest.mark.parametrize("rows", [1, 5, 8, 16, 31, 64, 100, 256])
def test_tensor_core_gemm_shapes(cuda, oracle, rng, OUT, IN, rows):
    """The pipelined tensor-core GEMM behind fp16 rwkv_q_gemm: every tile width
    (8/16/32/64 rows), split-K, OUT off the 64-row tile, a single K group."""
    from swiftrwkv_b200 import quant as Q
    W, wq, sc, bi = make_affine(oracle, rng, OUT, IN)
    x = f16(rng.standard_normal((rows, IN)))
    args = (dev(x), dev(wq.view(np.int32)), dev(sc.view(np.float16)), dev(bi.view(np.float16)))
    y = Q.quantizedMM(*args, out_dtype=torch.float32)
    want = want_gemm(oracle, x, wq, sc, bi)
    assert rel_err(host(y), want) < 2e-5
    y2 = Q.quantizedMM(*args, out_dtype=torch.float32)
    assert torch.equal(y, y2), "split-K reduction must be deterministic"
