"""CPU tests of the oracle itself: pinned against the golden fixtures (torch
autograd of the reference's unrolled recurrence, and the reference tests'
known-answer cases) before it is trusted as the GPU checker."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err, wkv_inputs


def test_half_conversions_match_numpy_and_torch(oracle, rng):
    x = np.concatenate([rng.standard_normal(4000) * 100, rng.standard_normal(4000) * 1e-6,
                        np.array([0.0, -0.0, 65504.0, 65520.0, 1e-8, 6e-8, 3e-8, np.inf, -np.inf])]
                       ).astype(np.float32)
    assert np.array_equal(oracle.f32_to_f16_bits(x), x.astype(np.float16).view(np.uint16))
    h = np.arange(0, 0x7C00, dtype=np.uint16)
    assert np.array_equal(oracle.f16_bits_to_f32(h), h.view(np.float16).astype(np.float32))
    bf = torch.tensor(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(oracle.f32_to_bf16_bits(x), bf)


def test_wkv7_oracle_matches_autograd_golden(oracle, golden):
    """Forward within 1e-4 and all seven gradients within 1e-3 relative of the
    autograd ground truth (WKV7KernelParityTests.swift:32-62,
    WKV7TrainKernelTests.swift:67-82)."""
    g = golden("wkv7_autograd.npz")
    ins = [g[n] for n in ("r", "w", "k", "v", "a", "b")]
    res = oracle.wkv7_train(*ins, g["h0"], g["dy"], g["dh_out"])
    y, h_out = res[:2]
    assert np.abs(y - g["y"]).max() < 1e-4
    assert np.abs(h_out - g["h_out"]).max() < 1e-4
    for name, got in zip(("dr", "dw", "dk", "dv", "da", "db", "dh0"), res[2:]):
        assert rel_err(got, g[name]) < 1e-3, name
    ex = oracle.wkv7_exact(*ins, g["h0"], g["dy"], g["dh_out"])
    for name, got in zip(("y", "h_out", "dr", "dw", "dk", "dv", "da", "db", "dh0"), ex):
        assert rel_err(got, g[name]) < 1e-5, name


def test_wkv7_split_equals_contiguous_bitwise(oracle, rng):
    """WKV7SequenceTests.swift:50-62 and WKV7StateTests: a pass split through
    the state equals the whole pass bitwise, at aligned and unaligned cuts."""
    r, w, k, v, a, b = wkv_inputs(rng, 2, 53, 3)
    h0 = (rng.standard_normal((2, 3, 64, 64)) * 0.1).astype(np.float32)
    y, h = oracle.wkv7_forward(r, w, k, v, a, b, h0)
    for cut in (16, 17, 1):
        sl1 = [x[:, :cut].copy() for x in (r, w, k, v, a, b)]
        sl2 = [x[:, cut:].copy() for x in (r, w, k, v, a, b)]
        y1, h1 = oracle.wkv7_forward(*sl1, h0)
        y2, h2 = oracle.wkv7_forward(*sl2, h1)
        assert np.array_equal(np.concatenate([y1, y2], 1), y)
        assert np.array_equal(h2, h)


def test_wkv7_step_equals_forward_at_t1(oracle, rng):
    """DecodeKernelTests.swift:27-39: step == forward at T=1, bitwise."""
    for H in (12, 3, 32):
        r, w, k, v, a, b = wkv_inputs(rng, 1, 1, H)
        h0 = (rng.standard_normal((1, H, 64, 64)) * 0.1).astype(np.float32)
        y, h = oracle.wkv7_forward(r, w, k, v, a, b, h0)
        ys, hs = oracle.wkv7_step(*(x[:, 0] for x in (r, w, k, v, a, b)), h0)
        assert np.array_equal(ys, y[:, 0]) and np.array_equal(hs, h)


def test_wkv7_train_forward_agrees_with_frozen(oracle, rng):
    """WKV7TrainKernelTests.swift:117-136: the training forward equals the
    frozen forward; the last checkpoint is the final state."""
    r, w, k, v, a, b = wkv_inputs(rng, 2, 48, 3)
    y, h = oracle.wkv7_forward(r, w, k, v, a, b)
    y2, h2, sa, ck = oracle.wkv7_forward(r, w, k, v, a, b, want_sa=True, ckpt_every=16)
    assert np.array_equal(y, y2) and np.array_equal(h, h2)
    assert np.array_equal(ck[:, :, -1], h)
    assert ck.shape == (2, 3, 3, 64, 64)


def test_padding_steps_leave_state_unchanged(oracle, rng):
    """w=1, k=0, b=0 is the identity on S (WKV7.swift:92-95, RWKVBlock.swift:221-237)."""
    r, w, k, v, a, b = wkv_inputs(rng, 1, 5, 2)
    w[:, 2:] = 1.0
    k[:, 2:] = 0.0
    b[:, 2:] = 0.0
    _, h_all = oracle.wkv7_forward(r, w, k, v, a, b)
    _, h_2 = oracle.wkv7_forward(*(x[:, :2].copy() for x in (r, w, k, v, a, b)))
    assert np.array_equal(h_all, h_2)


def test_tail_matches_formula(oracle, rng):
    """DecodeKernelTests.swift:57-76: tail within 1e-5 of the op-by-op formula."""
    rows, H, S = 3, 4, 64
    D = H * S
    wkv, r, k, v, g = (rng.standard_normal((rows, D)).astype(np.float32) for _ in range(5))
    rk, lnw, lnb = (rng.standard_normal(D).astype(np.float32) for _ in range(3))
    out = oracle.wkv_tail(wkv, r, k, v, rk, lnw, lnb, g, H, S)
    x = wkv.reshape(rows, H, S).astype(np.float64)
    mean = x.mean(-1, keepdims=True)
    var = ((x - mean) ** 2).mean(-1, keepdims=True)
    nrm = ((x - mean) / np.sqrt(var + 64e-5)).reshape(rows, D) * lnw + lnb
    bonus = (r * k * rk).reshape(rows, H, S).sum(-1, keepdims=True) * v.reshape(rows, H, S)
    want = (nrm + bonus.reshape(rows, D)) * g
    assert np.abs(out - want).max() < 1e-5 * max(1.0, np.abs(want).max())


def test_sym_kat_off_superblock(oracle, golden):
    """RwkvqFileTests.swift:237-262, exact."""
    g = golden("kat_sym.npz")
    got = oracle.sym_dequant(g["codes"], g["qs"], g["d"], 2, 48, 8, oracle.F32)
    assert np.array_equal(got, g["want"])


def test_sb6_kat_clamped_scale(oracle, golden):
    """RwkvqModelTests.swift:455-486: the clamp keeps fp32 only where it matters."""
    g = golden("kat_sb6.npz")
    live = oracle.sb6_to_affine(g["qblk_live"], g["qsqm_live"], g["ddm"], 2, 256, 0)
    assert live[3] is False
    assert live[1][0, 3] == np.float32(1e-8)
    assert live[1][1, 3] == g["scale_row1_blk3"]
    dead = oracle.sb6_to_affine(g["qblk_dead"], g["qsqm_dead"], g["ddm"], 2, 256, 0)
    assert dead[3] is True
    assert np.float32(np.float16(dead[1][0, 3])) == 0.0
    # the relayout is lossless except on clamped blocks, where the 1e-8 floor
    # moves a weight by at most code*1e-8 <= 63e-8 (RwkvqNative.swift:119-124)
    wq, sc, bi, _ = oracle.sb6_to_affine(g["qblk_live"], g["qsqm_live"], g["ddm"], 2, 256, 0)
    dense = oracle.sb6_dequant(g["qblk_live"], g["qsqm_live"], g["ddm"], 2, 256, 0)
    aff = oracle.affine_dequant(wq, sc, bi, group=32, bits=4)
    clamped = np.zeros_like(dense, bool)
    clamped[0, 3 * 32:4 * 32] = True
    assert np.array_equal(aff[~clamped], dense[~clamped])
    assert np.abs(aff - dense)[clamped].max() <= 63e-8


@pytest.mark.parametrize("bits,group", [(4, 64), (4, 32), (8, 64), (4, 128)])
def test_affine_quantize_roundtrip(oracle, rng, bits, group):
    """Restated MLX quantiser: every weight within one step of its dequantised
    value (snapping the larger-magnitude edge onto the grid can push the other
    extreme one step past the last code, where it clips), and most within half
    a step."""
    W = (rng.standard_normal((16, 256)) * 0.02).astype(np.float16).astype(np.float32)
    wq, sc, bi = oracle.affine_quantize(W, group, bits)
    deq = oracle.affine_dequant(wq, sc, bi, group, bits)
    step = np.abs(oracle.f16_bits_to_f32(sc)).repeat(group, 1)
    err = np.abs(deq - W)
    # the fp16 rounding of the stored scale adds up to code * 2^-11 steps
    fp16_slack = (1 << bits) * 2.0 ** -11
    assert np.all(err <= step * (1.001 + fp16_slack) + 1e-6)
    assert np.mean(err <= step * (0.5 + fp16_slack) + 1e-6) > 0.98


def test_affine_layout_lsb_first(oracle):
    """Field p of a row starts at bit p*bits (RwkvqNative.swift:28-31)."""
    for bits in (4, 5, 6, 8):
        IN = 64
        codes = (np.arange(IN) * 7 + 3) % (1 << bits)
        words = np.zeros(IN * bits // 32, np.uint64)
        for p, q in enumerate(codes):
            bit = p * bits
            words[bit // 32] |= np.uint64((int(q) << (bit % 32)) & 0xFFFFFFFF)
            if bit % 32 + bits > 32:
                words[bit // 32 + 1] |= np.uint64(int(q) >> (32 - bit % 32))
        wq = words.astype(np.uint32).reshape(1, -1)
        sc = np.ones((1, 1), np.float32)
        bi = np.zeros((1, 1), np.float32)
        got = oracle.affine_dequant(wq, sc, bi, group=64, bits=bits)
        assert np.array_equal(got[0], codes.astype(np.float32))


def test_affine_gemv_oracle_vs_exact(oracle, rng):
    W = (rng.standard_normal((64, 512)) * 0.02).astype(np.float16).astype(np.float32)
    wq, sc, bi = oracle.affine_quantize(W, 64, 4)
    x = rng.standard_normal((3, 512)).astype(np.float16).astype(np.float32)
    y = oracle.affine_gemv(x, wq, sc, bi)
    ye = oracle.affine_gemv(x, wq, sc, bi, exact=True)
    assert rel_err(y, ye) < 2e-5
    ref = x.astype(np.float64) @ oracle.affine_dequant(wq, sc, bi).astype(np.float64).T
    assert rel_err(ye, ref) < 1e-6
