"""GPU parity of the x070 decode runtime against the CPU decode oracle on the
reference's TinyBackbone-style fixture (L=2, D=128, vocab 64)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def tiny(act, rows=4, n_layer=2, n_embd=128, vocab=64, seed=42):
    from oracle import x070_oracle as XO
    from swiftrwkv_b200.x070 import X070Backbone, X070Config
    cfg = X070Config(n_layer, n_embd, vocab)
    w = XO.tiny_weights(XO.Cfg(n_layer, n_embd, vocab), seed)
    m = X070Backbone(cfg, max_rows=rows, act=act).load(w)
    ref = XO.X070Oracle(XO.Cfg(n_layer, n_embd, vocab), w, act=act)
    return m, ref


@pytest.mark.parametrize("act,tol", [("f32", 1e-4), ("f16", 2e-3)])
@pytest.mark.parametrize("rows", [1, 2, 4])
def test_step_logits_match_oracle(cuda, act, tol, rows):
    """1 and 2 rows of fp16 activations run the 4-bit projections on the
    streaming CUDA-core GEMV, 4 rows on the mma.sync GEMV."""
    from oracle import x070_oracle as XO
    m, ref = tiny(act, rows=rows)
    ids = XO.splitmix_ids(rows, 6)
    m.reset(rows)
    st = ref.new_state(rows)
    for t in range(ids.shape[1]):
        got = m.step(torch.from_numpy(ids[:, t]).cuda()).cpu().numpy()
        want = ref.step(ids[:, t], st)
        assert rel_err(got, want) < tol, (t, rel_err(got, want))


def test_wide_batch_tensor_core_path_matches_oracle(cuda):
    """More than 8 rows at D=256: every 4-bit projection, the fp16 low-rank
    projections and the head run on the tcgen05 GEMM (TMA + TMEM), whose
    weights are dequantised into fp16 as MLX's quantized matmul does."""
    from oracle import x070_oracle as XO
    rows = 20
    m, ref = tiny("f16", rows=rows, n_embd=256, vocab=200, seed=7)
    ids = XO.splitmix_ids(rows, 4, vocab=200)
    m.reset(rows)
    st = ref.new_state(rows)
    for t in range(ids.shape[1]):
        got = m.step(torch.from_numpy(ids[:, t]).cuda()).cpu().numpy()
        want = ref.step(ids[:, t], st)
        assert rel_err(got, want) < 2e-3, (t, rel_err(got, want))


def test_greedy_tokens_identical_fp32(cuda):
    """north_star: greedy decode token ids identical for the fp32 path."""
    from oracle import x070_oracle as XO
    m, ref = tiny("f32", rows=1)
    prompt = XO.splitmix_ids(1, 5)[0]
    got = m.generate(prompt, 12)
    st = ref.new_state(1)
    for t in prompt:
        logits = ref.step(np.array([t]), st)
    want = []
    for _ in range(12):
        nxt = int(np.argmax(logits[0]))
        want.append(nxt)
        logits = ref.step(np.array([nxt]), st)
    assert list(got) == want


def test_batch_rows_equal_single_runs(cuda):
    """BatchGenerateTests.swift:40-94: a batch row equals the single-row run
    (1e-5) and greedy batch tokens equal single generate."""
    from oracle import x070_oracle as XO
    m, _ = tiny("f32", rows=3)
    prompts = XO.splitmix_ids(3, 4, seed=7)
    batch = m.generateBatch(prompts, 8)
    for i in range(3):
        assert list(m.generate(prompts[i], 8)) == list(batch[i])
    m.reset(3)
    lb = [m.step(torch.from_numpy(prompts[:, t]).cuda()) for t in range(4)][-1].cpu().numpy()
    for i in range(3):
        m.reset(1)
        ls = [m.step(torch.from_numpy(prompts[i:i + 1, t]).cuda()) for t in range(4)][-1]
        assert rel_err(ls.cpu().numpy()[0], lb[i]) < 1e-5


def test_graph_replay_equals_eager_bitwise(cuda):
    from oracle import x070_oracle as XO
    m, _ = tiny("f16", rows=2)
    ids = XO.splitmix_ids(2, 5, seed=3)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        m.reset(2)
        eager = [m.step(torch.from_numpy(ids[:, t]).cuda(), use_graph=False) for t in range(5)]
        m.reset(2)
        graph = [m.step(torch.from_numpy(ids[:, t]).cuda(), use_graph=True) for t in range(5)]
    s.synchronize()
    for a, b in zip(eager, graph):
        assert torch.equal(a, b)


def test_random_init_runs(cuda):
    """Device-side x070 init on a small config: finite logits, deterministic."""
    from swiftrwkv_b200.x070 import X070Backbone, X070Config
    cfg = X070Config(2, 256, 512)
    outs = []
    for _ in range(2):
        m = X070Backbone(cfg, max_rows=2).init_random(seed=5)
        m.reset(2)
        outs.append(m.step(torch.tensor([1, 2], dtype=torch.int32).cuda()))
        m.close()
    assert torch.isfinite(outs[0]).all()
    assert torch.equal(outs[0], outs[1])


def adapters(cfg_tuple, rank=16, seed=3, alpha=32.0):
    """LoRA adapters (LoRA.swift:118-127 keys and scale alpha / rank) on every
    target the runtime takes: r/k/v/o, cmix key/value, head; B non-zero so that
    they change the result (the reference starts B at zero)."""
    n_layer, D, V = cfg_tuple
    F = 4 * D
    rng = np.random.default_rng(seed)
    w = {}
    tg = [("tmix.r_proj", D, D), ("tmix.k_proj", D, D), ("tmix.v_proj", D, D), ("tmix.o_proj", D, D),
          ("cmix.key", D, F), ("cmix.value", F, D)]
    for L in range(n_layer):
        for t, IN, OUT in tg:
            p = f"blocks.{L}.{t}."
            w[p + "lora_a"] = (rng.standard_normal((rank, IN)) / np.sqrt(IN)).astype(np.float32)
            w[p + "lora_b"] = (rng.standard_normal((OUT, rank)) * 0.05).astype(np.float32)
            w[p + "lora_scale"] = np.array([alpha / rank], np.float32)
    w["head.lora_a"] = (rng.standard_normal((rank, D)) / np.sqrt(D)).astype(np.float32)
    w["head.lora_b"] = (rng.standard_normal((V, rank)) * 0.05).astype(np.float32)
    w["head.lora_scale"] = np.array([alpha / rank], np.float32)
    return w


def tiny_lora(act, rows=4, n_layer=2, n_embd=128, vocab=64, seed=42):
    from oracle import x070_oracle as XO
    from swiftrwkv_b200.x070 import X070Backbone, X070Config
    w = XO.tiny_weights(XO.Cfg(n_layer, n_embd, vocab), seed)
    w.update(adapters((n_layer, n_embd, vocab)))
    m = X070Backbone(X070Config(n_layer, n_embd, vocab), max_rows=rows, act=act).load(w)
    ref = XO.X070Oracle(XO.Cfg(n_layer, n_embd, vocab), w, act=act)
    return m, ref


@pytest.mark.parametrize("act,tol", [("f32", 1e-4), ("f16", 2e-3)])
def test_lora_adapters_match_oracle(cuda, act, tol):
    """proj = base + scale (x A^T) B^T on every adapted projection
    (X070Backbone.swift:746-752), the key adapter before relu^2."""
    from oracle import x070_oracle as XO
    m, ref = tiny_lora(act)
    rows = 4
    ids = XO.splitmix_ids(rows, 5)
    m.reset(rows)
    st = ref.new_state(rows)
    for t in range(ids.shape[1]):
        got = m.step(torch.from_numpy(ids[:, t]).cuda()).cpu().numpy()
        want = ref.step(ids[:, t], st)
        assert rel_err(got, want) < tol, (t, rel_err(got, want))
    # 10 launches per layer + 4, plus per layer r/k/v (2) + o (2) + key (3) + value (2), head (2)
    assert m.launches_per_step == 1 + 2 * 10 + 4 + 2 * 9 + 2


def test_lora_adapters_wide_batch_tensor_core_path(cuda):
    from oracle import x070_oracle as XO
    rows = 20
    m, ref = tiny_lora("f16", rows=rows, n_embd=256, vocab=200, seed=7)
    ids = XO.splitmix_ids(rows, 3, vocab=200)
    m.reset(rows)
    st = ref.new_state(rows)
    for t in range(ids.shape[1]):
        got = m.step(torch.from_numpy(ids[:, t]).cuda()).cpu().numpy()
        want = ref.step(ids[:, t], st)
        assert rel_err(got, want) < 2e-3, (t, rel_err(got, want))


def test_lora_adapter_set_after_capture_drops_the_graph(cuda):
    """Setting an adapter changes the launch sequence: a step graph captured
    before must not replay; graph replay equals eager with the adapters."""
    from oracle import x070_oracle as XO
    from swiftrwkv_b200.x070 import X070Backbone, X070Config
    w = XO.tiny_weights(XO.Cfg(2, 128, 64), 42)
    m = X070Backbone(X070Config(2, 128, 64), max_rows=2, act="f16").load(w)
    ids = XO.splitmix_ids(2, 4, seed=3)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        m.reset(2)
        m.step(torch.from_numpy(ids[:, 0]).cuda(), use_graph=True)    # captures a graph without adapters
        m.load(adapters((2, 128, 64)))
        m.reset(2)
        eager = [m.step(torch.from_numpy(ids[:, t]).cuda(), use_graph=False) for t in range(4)]
        m.reset(2)
        graph = [m.step(torch.from_numpy(ids[:, t]).cuda(), use_graph=True) for t in range(4)]
    s.synchronize()
    for a, b in zip(eager, graph):
        assert torch.equal(a, b)


def test_lora_adapter_shape_errors(cuda):
    from swiftrwkv_b200 import _lib
    from swiftrwkv_b200.x070 import X070Backbone, X070Config
    m = X070Backbone(X070Config(1, 128, 64), max_rows=1)
    bad = {"blocks.0.tmix.r_proj.lora_a": np.zeros((12, 128), np.float32)}     # rank 12: not a multiple of 16
    with pytest.raises(_lib.RWKVError):
        m.load(bad)
    with pytest.raises(_lib.RWKVError):
        m.load({"blocks.0.tmix.r_proj.lora_a": np.zeros(100, np.float32)})       # not rank x IN
    with pytest.raises(_lib.RWKVError):
        m.load({"head.lora_scale": np.zeros(2, np.float32)})
