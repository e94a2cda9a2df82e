"""Batched decode (several sequences per step, sequence i on KV slot i, through the
tensor-core layer pass) against the oracle run one sequence at a time.

Each sequence starts from its own prompt (different lengths, so the sequences sit
at different positions and cross KV pages at different steps). Bars as for the
single-sequence path: greedy tokens identical to the oracle's; one step's logits
within 2e-2 max-abs and 1e-3 relative RMS.
"""
from __future__ import annotations

import numpy as np
import pytest

import fiber_b200 as fb
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

MAX_ABS, REL_RMS = 2e-2, 1e-3


def _rel_rms(a, b):
    return float(np.sqrt(np.mean((a.astype(np.float64) - b) ** 2)) / np.sqrt(np.mean(b.astype(np.float64) ** 2)))


def _prompt(vocab, n, seed):
    return np.random.default_rng(seed).integers(1, vocab, n).astype(np.int32)


def _start(ctx, kv, vocab, n_seq, seed):
    prompts = [_prompt(vocab, 3 + 17 * i, seed + i) for i in range(n_seq)]
    firsts = [ctx.prefill(kv, pr, slot=i) for i, pr in enumerate(prompts)]
    return prompts, firsts


@pytest.mark.parametrize("name", ["q4km", "q5km", "f16", "gqa8", "hd128"])
def test_batched_greedy_matches_oracle(tiny_model, name):
    path = tiny_model(name)
    hm = fb.HostModel(path)
    ctx = fb.Context(hm, max_seq=256, max_batch=8)
    kv = ctx.kv(256, max_batch=8)
    prompts, firsts = _start(ctx, kv, hm.params.vocab_size, 5, 40)
    n = 24
    dev, _ = ctx.decode_greedy_batch(kv, firsts, [len(p) for p in prompts], n)
    om = orc.Model(path)
    for i, pr in enumerate(prompts):
        want = om.state(256, kv_fp16=True).generate(pr, n)
        assert firsts[i] == want[0], (name, i)
        assert dev[:, i].tolist() == want[1:].tolist(), (name, i)


@pytest.mark.parametrize("name", ["q4km", "q5km", "gqa8"])
def test_batched_step_logits_match_oracle(tiny_model, name):
    path = tiny_model(name)
    hm = fb.HostModel(path)
    ctx = fb.Context(hm, max_seq=256, max_batch=4)
    kv = ctx.kv(256, max_batch=4)
    prompts, firsts = _start(ctx, kv, hm.params.vocab_size, 3, 60)
    am, lg = ctx.forward_batch(kv, firsts, [len(p) for p in prompts])
    om = orc.Model(path)
    for i, pr in enumerate(prompts):
        st = om.state(256, kv_fp16=True)
        for pos, t in enumerate(pr):
            st.forward(int(t), pos)
        want = st.forward(firsts[i], len(pr))
        assert np.abs(lg[i] - want).max() < MAX_ABS, (name, i)
        assert _rel_rms(lg[i], want) < REL_RMS, (name, i)
        assert am[i] == int(np.argmax(lg[i]))


def test_batch_of_one_and_host_steps_agree(tiny_model):
    """The device loop over a batch equals host-driven batched steps."""
    path = tiny_model("q4km")
    hm = fb.HostModel(path)
    ctx = fb.Context(hm, max_seq=256, max_batch=4)
    kv = ctx.kv(256, max_batch=4)
    prompts, firsts = _start(ctx, kv, hm.params.vocab_size, 3, 80)
    pos = np.array([len(p) for p in prompts], np.int32)
    dev, _ = ctx.decode_greedy_batch(kv, firsts, pos, 10)
    kv2 = ctx.kv(256, max_batch=4)
    for i, pr in enumerate(prompts):
        ctx.prefill(kv2, pr, slot=i)
    tok = np.array(firsts, np.int32)
    for s in range(10):
        am, _ = ctx.forward_batch(kv2, tok, pos + s, want_logits=False)
        assert am.tolist() == dev[s].tolist(), s
        tok = am


def test_batch_errors_are_reported(tiny_model):
    path = tiny_model("q4km")
    hm = fb.HostModel(path)
    with pytest.raises(fb.FiberError):
        fb.Context(hm, max_seq=128, max_batch=65)
    ctx = fb.Context(hm, max_seq=128, max_batch=4)
    kv = ctx.kv(128, max_batch=2)
    with pytest.raises(fb.FiberError):
        ctx.forward_batch(kv, [1, 2, 3], [0, 0, 0])  # more sequences than KV slots
    with pytest.raises(fb.FiberError):
        ctx.forward_batch(kv, [1, 2], [0, 128])  # position outside the cache
    with pytest.raises(fb.FiberError):
        ctx.forward_batch(kv, [1, hm.params.vocab_size], [0, 0])  # token out of range
    with pytest.raises(fb.FiberError):
        ctx.decode_greedy_batch(kv, [1, 2], [100, 0], 40)  # runs past max_seq
    with pytest.raises(fb.FiberError):
        ctx.prefill(kv, _prompt(hm.params.vocab_size, 5, 1), slot=2)  # no such slot
    am, _ = ctx.forward_batch(kv, [1, 2], [0, 0])  # still usable
    assert len(am) == 2
