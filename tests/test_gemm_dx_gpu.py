"""GPU parity of the projection backward dX = bf16(bf16(dY) W_bf16) (the bf16
VJP of X070Backbone.baseMatmul, X070Backbone.swift:337-356) through the C ABI.

The reference's own test (RwkvqBackwardTests.testBackwardIsTheFormula) asks
the backward to equal matmul(dY.asType(bf16), W(bf16)).asType(x.dtype)
bitwise, within one library.  Across libraries the fp32 sums are grouped
differently, so the bar here is: the kernel's result equals the bf16 rounding
of the exact (float64) sum of the bf16 operands except at near-ties (at most
1 % of the elements), and lies within half a bf16 step of the exact sum plus
fp32 accumulation rounding everywhere; the fused 4-bit kernel equals
dequantise-to-bf16 + the dense kernel bitwise; the dX dtypes and
accumulation are the bf16 result widened, narrowed or added exactly.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def bf16_step(x):
    """Distance to the next bf16 value above |x| (8 significant bits)."""
    e = np.floor(np.log2(np.maximum(np.abs(x), 1e-30)))
    return np.exp2(e - 7)


def check_formula(got, want, exact, abs_sum):
    """got is the bf16 rounding of an fp32-accumulated sum: within half a bf16
    step of the exact sum plus the accumulation's rounding (bounded here by
    2^-20 of the sum of |terms|), and equal to `want` (the bf16 rounding of
    the exact sum) except at near-ties (at most 1 % of the elements)."""
    frac = (got != want).mean()
    assert frac <= 0.01, f"{frac:.4f} of the elements differ from the bf16-rounded exact sum"
    step = bf16_step(np.maximum(np.abs(exact), np.abs(got)))
    bound = 0.5 * step * 1.0001 + abs_sum * 2.0 ** -20
    bad = np.abs(got - exact) > bound
    assert not bad.any(), f"{bad.sum()} elements beyond half a bf16 step of the exact sum"


def abs_terms(oracle, dy, W):
    """sum over o of |bf16(dy)[n, o] * bf16(W)[o, i]|, float64."""
    b = lambda x: oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(x)).astype(np.float64)
    return np.abs(b(dy)) @ np.abs(b(W))


def dense_case(rng, oracle, rows, OUT, IN, scale=1.0):
    dy = (rng.standard_normal((rows, OUT)) * scale).astype(np.float32)
    W = (rng.standard_normal((OUT, IN)) * 0.02).astype(np.float32)
    want, exact = oracle.base_matmul_vjp(dy, W)
    return dy, W, want, exact, abs_terms(oracle, dy, W)


@pytest.mark.parametrize("rows,OUT,IN", [(1, 64, 128), (16, 768, 768), (64, 2048, 2048), (65, 256, 384),
                                         (300, 512, 2048), (257, 2048, 256)])
def test_dense_backward_is_the_formula(cuda, oracle, rng, rows, OUT, IN):
    from swiftrwkv_b200 import quant as Q
    dy, W, want, exact, asum = dense_case(rng, oracle, rows, OUT, IN)
    got = Q.baseMatmulVJP(dev(dy), weight=dev(W).to(torch.bfloat16)).cpu().numpy()
    assert got.dtype == np.float32 and got.shape == (rows, IN)
    check_formula(got, want, exact, asum)


@pytest.mark.parametrize("rows,OUT,IN", [(16, 768, 768), (64, 2048, 2048), (300, 8192, 2048), (100, 2048, 8192)])
def test_q4_backward_matches_oracle_and_the_dense_path(cuda, oracle, rng, rows, OUT, IN):
    from swiftrwkv_b200 import quant as Q
    W = (rng.standard_normal((OUT, IN)) * 0.02).astype(np.float16).astype(np.float32)
    wq, sc, bi = oracle.affine_quantize(W, 64, 4)
    dy = rng.standard_normal((rows, OUT)).astype(np.float32)
    q = Q.QuantBase(dev(wq.view(np.int32)), dev(sc.view(np.float16)), dev(bi.view(np.float16)), 64, 4)
    got = Q.baseMatmulVJP(dev(dy), q=q).cpu().numpy()
    Wd = oracle.affine_dequant(wq, sc.view(np.float16), bi.view(np.float16))
    want, exact = oracle.base_matmul_vjp(dy, Wd)
    check_formula(got, want, exact, abs_terms(oracle, dy, Wd))
    # fused dequant == rwkv_q_dequant to bf16, then the dense kernel (bitwise)
    wb = Q.dequantized(q.wq, q.scales, q.biases, 64, 4, dtype=torch.bfloat16)
    two_step = Q.baseMatmulVJP(dev(dy), weight=wb).cpu().numpy()
    assert np.array_equal(got, two_step)


def test_dx_dtypes_and_accumulation(cuda, oracle, rng):
    from swiftrwkv_b200 import quant as Q
    rows, OUT, IN = 96, 1024, 512
    dy, W, want, exact, asum = dense_case(rng, oracle, rows, OUT, IN)
    wb = dev(W).to(torch.bfloat16)
    f32 = Q.baseMatmulVJP(dev(dy), weight=wb)
    b16 = Q.baseMatmulVJP(dev(dy).to(torch.bfloat16), weight=wb)            # primal bf16
    h16 = Q.baseMatmulVJP(dev(dy), weight=wb, primal_dtype=torch.float16)
    assert b16.dtype == torch.bfloat16 and h16.dtype == torch.float16
    assert torch.equal(b16.float(), f32)                  # the bf16 result, widened losslessly
    assert torch.equal(h16, f32.to(torch.float16))        # narrowed from the bf16 result
    base = dev(rng.standard_normal((rows, IN)).astype(np.float32))
    acc = base.clone()
    Q.baseMatmulVJP(dev(dy), weight=wb, out=acc)
    assert torch.equal(acc, base + f32)                   # one fp32 add per element
    check_formula(f32.cpu().numpy(), want, exact, asum)


def test_small_cotangents_keep_their_digits(cuda, oracle, rng):
    """Why the reference's backward is bf16 rather than fp16: cotangents of a
    loss averaged over many tokens are tiny (here 1e-9 scale, below fp16's
    normal range); the bf16 backward still returns the formula."""
    from swiftrwkv_b200 import quant as Q
    dy, W, want, exact, asum = dense_case(rng, oracle, 32, 512, 256, scale=1e-9)
    got = Q.baseMatmulVJP(dev(dy), weight=dev(W).to(torch.bfloat16)).cpu().numpy()
    assert np.abs(got).max() > 0
    check_formula(got, want, exact, asum)


def test_backward_is_deterministic(cuda, rng):
    from swiftrwkv_b200 import quant as Q
    dy = dev(rng.standard_normal((512, 2048)).astype(np.float32))
    wb = dev((rng.standard_normal((2048, 1024)) * 0.02).astype(np.float32)).to(torch.bfloat16)
    a = Q.baseMatmulVJP(dy, weight=wb)
    b = Q.baseMatmulVJP(dy, weight=wb)
    assert torch.equal(a, b)
