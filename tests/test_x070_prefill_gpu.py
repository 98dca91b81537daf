"""GPU parity of the runtime's parallel prefill (rwkv_x070_prefill) and of
generateBatch over it, against the decode oracle run token by token.

The reference prefills with its parallel pass (bodyWithState,
X070Backbone.swift:1011-1048) and keeps the recurrent pass as the reference
it is checked against (X070Generation.swift:330-343); its batch prefill
right-pads ragged prompts and masks the padding (w = 1, k = 0, b = 0) so a
row's state stops at its last real token (RWKVBlock.swift:221-237), taking
the token-shift state there (RWKVBatchState.swift:159-175).  Checked here:

  * logits of each row's last real token equal the oracle's after feeding the
    row's own tokens one by one (fp16: 2e-3, the prefill's projections are
    products with the fp16-dequantised weight, as the oracle takes them for
    more than 8 rows; fp32: 1e-4);
  * the state left behind (WKV and both token shifts) continues decoding like
    the oracle's;
  * equal and ragged lengths, and prompts longer than one prefill block;
  * generateBatch: greedy ids of ragged prompts identical to the oracle's in
    fp32, stop tokens end a row (the stop id kept) and the row leaves the
    batch while the others continue unchanged.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def model(act, rows, n_layer=2, n_embd=128, vocab=64, seed=42):
    from oracle import x070_oracle as XO
    from swiftrwkv_b200.x070 import X070Backbone, X070Config
    cfg = XO.Cfg(n_layer, n_embd, vocab)
    w = XO.tiny_weights(cfg, seed)
    m = X070Backbone(X070Config(n_layer, n_embd, vocab), max_rows=rows, act=act).load(w)
    return m, XO.X070Oracle(cfg, w, act=act)


def oracle_rows(ref, prompts, wide):
    """Each row's own tokens through the oracle one at a time (all rows of a
    step together, a finished row's state kept aside); wide: the projections
    as the prefill GEMMs take them (fp16-dequantised weight)."""
    rows = len(prompts)
    ref.GEMV_MAX_ROWS = -1 if wide else 8
    states, last = [], []
    for i in range(rows):
        st = ref.new_state(1)
        lg = None
        for t in prompts[i]:
            lg = ref.step(np.array([t], np.int32), st)
        states.append(st)
        last.append(lg[0])
    ref.GEMV_MAX_ROWS = 8
    return np.stack(last), states


def merge(states):
    return {k: np.concatenate([s[k] for s in states], axis=1) for k in states[0]}


@pytest.mark.parametrize("act,tol", [("f16", 2e-3), ("f32", 1e-4)])
@pytest.mark.parametrize("lengths", [[20, 20, 20], [20, 7, 13], [1, 5, 16]])
def test_prefill_matches_recurrent_oracle(cuda, act, tol, lengths):
    from oracle import x070_oracle as XO
    rows, T = len(lengths), max(lengths)
    m, ref = model(act, rows)
    ids = XO.splitmix_ids(rows, T, seed=5)
    prompts = [list(ids[i, :lengths[i]]) for i in range(rows)]
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        m.reset(rows)
        got = m.prefill(torch.from_numpy(ids).cuda(), lengths)
        # continue: two decode steps from the prefilled state
        nxt = [XO.splitmix_ids(rows, 2, seed=9)[:, j] for j in range(2)]
        cont = [m.step(torch.from_numpy(n).cuda()) for n in nxt]
    s.synchronize()
    want, states = oracle_rows(ref, prompts, wide=(act == "f16"))
    assert rel_err(got.cpu().numpy(), want) < tol, rel_err(got.cpu().numpy(), want)
    st = merge(states)
    for j in range(2):
        w = ref.step(nxt[j], st)
        assert rel_err(cont[j].cpu().numpy(), w) < tol, (j, rel_err(cont[j].cpu().numpy(), w))


def test_prefill_over_several_blocks(cuda):
    """rows * T above the prefill block (8192 token rows): the prompt runs in
    blocks of 192 positions, rows ending in the first block and in the
    second; fp32 so that only the block split can differ."""
    from oracle import x070_oracle as XO
    rows, T = 40, 256
    m, ref = model("f32", rows)
    ids = XO.splitmix_ids(rows, T, seed=17)
    lengths = [T if i % 3 == 0 else (150 if i % 3 == 1 else 200) for i in range(rows)]
    prompts = [list(ids[i, :lengths[i]]) for i in range(rows)]
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        m.reset(rows)
        got = m.prefill(torch.from_numpy(ids).cuda(), lengths)
        nxt = XO.splitmix_ids(rows, 1, seed=3)[:, 0]
        cont = m.step(torch.from_numpy(nxt).cuda())
    s.synchronize()
    # the oracle in one pass over all rows, padding kept out by per-row steps
    want, states = oracle_rows(ref, prompts, wide=False)
    assert rel_err(got.cpu().numpy(), want) < 1e-4
    w = ref.step(nxt, merge(states))
    assert rel_err(cont.cpu().numpy(), w) < 1e-4


def test_prefill_continues_an_existing_state(cuda):
    """bodyWithState(state:): a prompt split in two prefills equals one."""
    from oracle import x070_oracle as XO
    rows, T = 2, 24
    m, _ = model("f32", rows)
    ids = XO.splitmix_ids(rows, T, seed=23)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        m.reset(rows)
        one = m.prefill(torch.from_numpy(ids).cuda())
        m.reset(rows)
        m.prefill(torch.from_numpy(ids[:, :10].copy()).cuda(), logits=False)
        two = m.prefill(torch.from_numpy(ids[:, 10:].copy()).cuda())
    s.synchronize()
    assert rel_err(two.cpu().numpy(), one.cpu().numpy()) < 1e-5


def test_generate_batch_ragged_greedy_identical_fp32(cuda):
    from oracle import x070_oracle as XO
    rows = 3
    m, ref = model("f32", rows)
    ids = XO.splitmix_ids(rows, 12, seed=31)
    lengths = [12, 4, 9]
    prompts = [list(ids[i, :lengths[i]]) for i in range(rows)]
    n_new = 8
    got = m.generateBatch(prompts, n_new)
    for i in range(rows):
        st = ref.new_state(1)
        for t in prompts[i]:
            lg = ref.step(np.array([t], np.int32), st)
        want = []
        for _ in range(n_new):
            nxt = int(np.argmax(lg[0]))
            want.append(nxt)
            lg = ref.step(np.array([nxt], np.int32), st)
        assert [int(x) for x in got[i]] == want, i


def test_generate_batch_stop_tokens_drop_rows(cuda):
    """A row that emits a stop id ends there (the id kept) and leaves the
    batch; the rows that continue produce what they produce without stops."""
    from oracle import x070_oracle as XO
    rows = 4
    m, _ = model("f32", rows)
    ids = XO.splitmix_ids(rows, 6, seed=41)
    prompts = [list(ids[i, :6 - i]) for i in range(rows)]
    n_new = 10
    free = m.generateBatch(prompts, n_new, stopTokens=[])
    assert all(len(r) == n_new for r in free)
    # a stop id that row 1 emits at step 3 (and that ends any other row that emits it)
    stop = int(free[1][3])
    got = m.generateBatch(prompts, n_new, stopTokens=[stop])
    for i in range(rows):
        want = free[i]
        if stop in want:
            want = want[:want.index(stop) + 1]
        assert [int(x) for x in got[i]] == [int(x) for x in want], i
    assert len(got[1]) <= 4
