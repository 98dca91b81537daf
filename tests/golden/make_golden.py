"""Generate the golden fixtures under tests/golden/ (run from the repo root):

    python tests/golden/make_golden.py

wkv7_autograd.npz
    WKV-7 forward and all seven gradients from torch-CPU autograd (float64)
    over the unrolled recurrence of the reference's ground truth,
    wkv7ReferenceWithState (Sources/RWKVKernel/WKV7Reference.swift:31-76),
    differentiated like WKV7KernelParityTests / WKV7TrainKernelTests: loss =
    sum(out * g) + sum(h_out * gh), with a non-symmetric h0.  Inputs follow
    the reference test recipe (WKV7KernelParityTests.swift:15-30) drawn from
    numpy's PCG64 seeded 0x5EED2026 (MLXRandom streams cannot be reproduced).

kat_sym.npz
    The reference's hand-computed sym case (RwkvqFileTests.swift:237-262):
    OUT=2, IN=48, codes i*37-90 (int8 wrap), qs [3,-5,7,11,-2,1],
    d [0.0123, 0.25] (fp16); expected w = code * float(half(qs * d)).

kat_sb6.npz
    The reference's synthetic degenerate-block case
    (RwkvqModelTests.swift:455-486): OUT=2, IN=256, xbits 0, all code bytes
    0x21 except row 0 block 3, qs 20 / qm -3 everywhere except qs=0 at row 0
    block 3, d = dm = 0.01 (fp16).  Expected relayout scales: row 0 block 3
    is clamped to 1e-8 and must stay fp32 when that block's codes are
    non-zero, fp16 (scale 0) when they are zero; row 1 block 3 scale is
    half(20 * half(0.01)).
"""
from __future__ import annotations

import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
SEED = 0x5EED2026


def wkv7_reference(r, w, k, v, a, b, h0):
    """Unrolled recurrence, S[b,h,dv,dk] (WKV7Reference.swift:47-74)."""
    s = h0
    outs = []
    for t in range(r.shape[1]):
        rt, wt, kt, vt, at, bt = (x[:, t] for x in (r, w, k, v, a, b))
        sa = (s * at.unsqueeze(-2)).sum(-1)
        s = s * wt.unsqueeze(-2) + vt.unsqueeze(-1) * kt.unsqueeze(-2) + sa.unsqueeze(-1) * bt.unsqueeze(-2)
        outs.append((s * rt.unsqueeze(-2)).sum(-1).unsqueeze(1))
    return torch.cat(outs, 1), s


def make_wkv7():
    rng = np.random.default_rng(SEED)
    B, T, H, N = 1, 32, 2, 64

    def rnd(s):
        return rng.standard_normal((B, T, H, N)) * s

    r, v, k = rnd(0.5), rnd(0.5), rnd(0.5)
    kk = k / np.sqrt((k * k).sum(-1, keepdims=True) + 1e-12)
    iclr = 1 / (1 + np.exp(-rnd(1.0)))
    a = -kk
    b = kk * iclr
    w = np.exp(-0.606531 / (1 + np.exp(-rnd(1.0))))
    g = rnd(1.0)
    h0 = rng.standard_normal((B, H, N, N)) * 0.2          # non-symmetric
    gh = rng.standard_normal((B, H, N, N)) * 0.1
    ins = [x.astype(np.float32) for x in (r, w, k, v, a, b, h0)]
    g, gh = g.astype(np.float32), gh.astype(np.float32)
    ts = [torch.tensor(x, dtype=torch.float64, requires_grad=True) for x in ins]
    out, h_out = wkv7_reference(*ts)
    loss = (out * torch.tensor(g, dtype=torch.float64)).sum() + \
           (h_out * torch.tensor(gh, dtype=torch.float64)).sum()
    loss.backward()
    names = ["r", "w", "k", "v", "a", "b", "h0"]
    data = {n: x for n, x in zip(names, ins)}
    data.update(dy=g, dh_out=gh, y=out.detach().numpy().astype(np.float32),
                h_out=h_out.detach().numpy().astype(np.float32))
    for n, t in zip(names, ts):
        data["d" + n] = t.grad.numpy().astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "wkv7_autograd.npz"), **data)


def make_sym():
    OUT, IN = 2, 48
    codes = ((np.arange(OUT * IN) * 37 - 90) % 256).astype(np.uint8)  # Int8(truncatingIfNeeded:)
    qs = np.array([3, -5, 7, 11, -2, 1], np.int8)
    d = np.array([0.0123, 0.25], np.float32).astype(np.float16)
    dh = d.astype(np.float32)
    want = np.empty((OUT, IN), np.float32)
    for rr in range(OUT):
        for c in range(IN):
            scale = np.float32(np.float16(np.float32(qs[rr * 3 + c // 16]) * dh[rr]))
            want[rr, c] = np.float32(codes.view(np.int8)[rr * IN + c]) * scale
    np.savez_compressed(os.path.join(HERE, "kat_sym.npz"), codes=codes.reshape(OUT, IN),
                        qs=qs.view(np.uint8).reshape(OUT, 3), d=d.view(np.uint16).reshape(OUT, 1),
                        want=want)


def make_sb6():
    OUT, IN, NB = 2, 256, 8
    out = {}
    for name, dead in (("live", 0x21), ("dead", 0x00)):
        qblk = np.full(OUT * NB * 16, 0x21, np.uint8)
        qblk[3 * 16:4 * 16] = dead
        qsqm = np.zeros(OUT * NB * 2, np.uint8)
        qsqm[0::2] = 20
        qsqm[1::2] = np.uint8(256 - 3)
        qsqm[2 * 3] = 0
        out["qblk_" + name] = qblk.reshape(OUT, NB * 16)
        out["qsqm_" + name] = qsqm.reshape(OUT, NB * 2)
    ddm = np.full((OUT, 2), 0.01, np.float32).astype(np.float16)
    out["ddm"] = ddm.view(np.uint16)
    out["scale_row1_blk3"] = np.float32(np.float16(20 * np.float32(np.float16(0.01))))
    np.savez_compressed(os.path.join(HERE, "kat_sb6.npz"), **out)


if __name__ == "__main__":
    make_wkv7()
    make_sym()
    make_sb6()
    for f in sorted(os.listdir(HERE)):
        print(f, os.path.getsize(os.path.join(HERE, f)))
