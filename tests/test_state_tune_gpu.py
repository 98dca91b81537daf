"""State tuning on the GPU: the three state-tuning entry points and the
tuner's step through the C ABI, against the oracle.

  rwkv_state_broadcast / rwkv_state_grad_sum   bit-exact (copies, ordered adds)
  rwkv_adamw_clip_step                         oracle step to 2e-6 relative
                                               (only the norm's summation order
                                               differs, in double)
  WKVStateTuner.step                           state gradients within the WKV
                                               backward tolerance, 1e-3 relative
  NCCL, two ranks (when two GPUs are present)  ranks identical, and equal to one
                                               process over the whole batch
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from conftest import rel_err, wkv_inputs
from test_state_tune import OracleOps

import oracle.oracle as orc
from swiftrwkv_b200 import _lib
from swiftrwkv_b200.state_tune import StateTuneConfig, WKVStateTuner

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-3


def _p(t):
    return None if t is None else _lib.P(t.data_ptr())


def _st():
    return _lib.P(torch.cuda.current_stream().cuda_stream)


def test_broadcast_and_grad_sum_are_exact():
    rng = np.random.default_rng(5)
    B, H = 3, 5
    s = torch.from_numpy(rng.standard_normal((H, 64, 64)).astype(np.float32)).cuda()
    h = torch.full((B, H, 64, 64), float("nan"), device="cuda")
    _lib.call("rwkv_state_broadcast", _p(s), _p(h), B, H, 64, _st())
    assert torch.equal(h, s.expand(B, H, 64, 64))
    dh = rng.standard_normal((B, H, 64, 64)).astype(np.float32)
    g = torch.full((H, 64, 64), float("nan"), device="cuda")
    _lib.call("rwkv_state_grad_sum", _p(torch.from_numpy(dh).cuda()), _p(g), B, H, 64, 0, _st())
    want = np.zeros((H, 64, 64), np.float32)
    for b in range(B):
        want = (want + dh[b]).astype(np.float32)
    np.testing.assert_array_equal(g.cpu().numpy(), want)
    # accumulate adds onto what is there
    _lib.call("rwkv_state_grad_sum", _p(torch.from_numpy(dh).cuda()), _p(g), B, H, 64, 1, _st())
    want2 = want.copy()
    for b in range(B):
        want2 = (want2 + dh[b]).astype(np.float32)
    np.testing.assert_array_equal(g.cpu().numpy(), want2)


@pytest.mark.parametrize("n,clip,wd", [(1000, 1.0, 0.0), (32 * 40 * 4096, 1.0, 0.01), (4096 * 3 + 7, 0.0, 0.0)])
def test_adamw_clip_step_matches_the_oracle(n, clip, wd):
    rng = np.random.default_rng(n)
    p = rng.standard_normal(n).astype(np.float32)
    m = (rng.standard_normal(n) * 0.01).astype(np.float32)
    v = (np.abs(rng.standard_normal(n)) * 1e-4).astype(np.float32)
    g = (rng.standard_normal(n) * 0.05).astype(np.float32)
    cfg = StateTuneConfig()
    c1, c2 = cfg.bias_corrections(4)
    kw = dict(grad_scale=0.125, clip=clip, lr=3e-4, beta1=0.9, beta2=0.99, eps=1e-8,
              weight_decay=wd, c1=c1, c2=c2)
    wp, wm, wv, wn = orc.adamw_clip_step(p, m, v, g, **kw)
    dp, dm, dv, dg = (torch.from_numpy(x).cuda() for x in (p, m, v, g))
    norm = torch.zeros((), device="cuda")
    ws_bytes = int(_lib.lib().rwkv_adamw_workspace_size(n))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    _lib.call("rwkv_adamw_clip_step", _p(dp), _p(dm), _p(dv), _p(dg), n, kw["grad_scale"], clip,
              kw["lr"], kw["beta1"], kw["beta2"], kw["eps"], wd, c1, c2, _p(norm), _p(ws), ws_bytes,
              _st())
    torch.cuda.synchronize()
    assert abs(float(norm) - float(wn)) <= 2e-6 * float(wn)
    np.testing.assert_allclose(dm.cpu().numpy(), wm, rtol=2e-6, atol=1e-12)
    np.testing.assert_allclose(dv.cpu().numpy(), wv, rtol=2e-6, atol=1e-15)
    np.testing.assert_allclose(dp.cpu().numpy(), wp, rtol=2e-6, atol=1e-9)


def test_adamw_clip_step_rejects_bad_arguments():
    lib = _lib.lib()
    t = torch.zeros(64, device="cuda")
    p = _p(t)
    ws_bytes = int(lib.rwkv_adamw_workspace_size(64))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    args = lambda **o: [o.get("param", p), p, p, p, o.get("n", 64), 1.0, 1.0, 1e-3, 0.9, 0.99, 1e-8,
                        0.0, o.get("c1", 0.1), 0.01, None, o.get("ws", _p(ws)), o.get("wsb", ws_bytes),
                        None]
    assert lib.rwkv_adamw_clip_step(*args(param=None)) == _lib.E_NULL
    assert lib.rwkv_adamw_clip_step(*args(n=0)) == _lib.E_SHAPE
    assert lib.rwkv_adamw_clip_step(*args(c1=0.0)) == _lib.E_SHAPE
    assert lib.rwkv_adamw_clip_step(*args(wsb=ws_bytes - 8)) == _lib.E_WORKSPACE
    assert lib.rwkv_adamw_clip_step(*args(ws=None)) == _lib.E_WORKSPACE


def _layers(rng, L, B, T, H):
    out = []
    for _ in range(L):
        r, w, k, v, a, b = wkv_inputs(rng, B, T, H)
        dy = rng.standard_normal((B, T, H, 64)).astype(np.float32)
        out.append([torch.from_numpy(np.ascontiguousarray(x)) for x in (r, w, k, v, a, b, dy)])
    return out


def test_tuner_step_on_the_gpu_matches_the_oracle():
    rng = np.random.default_rng(8)
    L, B, T, H = 3, 2, 48, 4
    layers = _layers(rng, L, B, T, H)
    init = torch.from_numpy((rng.standard_normal((L, H, 64, 64)) * 0.1).astype(np.float32))
    cfg = StateTuneConfig(lr=1e-2, warmupSteps=0, maxSteps=4)
    gpu = WKVStateTuner(L, H, config=cfg, initial=init.cuda())
    cpu = WKVStateTuner(L, H, config=cfg, initial=init, device="cpu", ops=OracleOps())
    n_gpu = float(gpu.step([[x.cuda() for x in t] for t in layers]))
    n_cpu = float(cpu.step(layers))
    for l in range(L):
        assert rel_err(gpu.grads[l].cpu().numpy(), cpu.grads[l].numpy()) < GRAD_TOL, l
    assert abs(n_gpu - n_cpu) <= GRAD_TOL * n_cpu
    # the update moves every entry by about lr (first Adam step), the same way
    d_gpu = (gpu.params.cpu() - init).numpy()
    d_cpu = (cpu.params - init).numpy()
    big = np.abs(cpu.grads.numpy()) > 1e-3 * np.abs(cpu.grads.numpy()).max()
    assert (np.sign(d_gpu[big]) == np.sign(d_cpu[big])).mean() > 0.999


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_problem():
    rng = np.random.default_rng(21)
    L, BG, T, H = 2, 4, 32, 4
    layers = _layers(rng, L, BG, T, H)
    init = torch.from_numpy((rng.standard_normal((L, H, 64, 64)) * 0.1).astype(np.float32))
    return L, BG, H, layers, init


def _nccl_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=60),
                                         device_id=torch.device("cuda", rank))
    try:
        L, BG, H, layers, init = _nccl_problem()
        sl = WKVStateTuner.local_slice(BG, rank, world)
        local = [[x[sl].contiguous().cuda() for x in t] for t in layers]
        tu = WKVStateTuner(L, H, config=StateTuneConfig(lr=1e-2, warmupSteps=0, maxSteps=4),
                           initial=init.cuda())
        for _ in range(2):
            tu.step(local)
        torch.cuda.synchronize()
        torch.save({"params": tu.params.cpu()}, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_two_ranks_equal_one_process(tmp_path):
    world = 2
    torch.multiprocessing.start_processes(_nccl_worker, args=(world, _free_port(), str(tmp_path)),
                                          nprocs=world, join=True, start_method="spawn")
    r0, r1 = (torch.load(tmp_path / f"rank{r}.pt")["params"] for r in range(world))
    # the same two steps in this process (no process group: no allreduce) over
    # the whole batch, gradients averaged over the ranks' count
    L, BG, H, layers, init = _nccl_problem()
    single = WKVStateTuner(L, H, config=StateTuneConfig(lr=1e-2, warmupSteps=0, maxSteps=4),
                           initial=init.cuda(), grad_scale=1.0 / world)
    full = [[x.cuda() for x in t] for t in layers]
    for _ in range(2):
        single.step(full)
    one = single.params.cpu()
    assert torch.equal(r0, r1)
    np.testing.assert_allclose(r0.numpy(), one.numpy(), rtol=0, atol=1e-5)
