"""Batched prefill (tensor-core dequant-GEMMs + causal attention over the cache)
against the oracle and against the token-by-token path: the first generated token
and the following greedy tokens equal the oracle's, and the KV cache it fills
matches the step-by-step cache to fp16 rounding. Prompts cross the 128-token chunk
and the 64-position page boundaries; a prompt split over two calls (start > 0)
gives the same cache."""
from __future__ import annotations

import numpy as np
import pytest

import fiber_b200 as fb
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _prompt(vocab, n, seed):
    return np.random.default_rng(seed).integers(1, vocab, n).astype(np.int32)


@pytest.mark.parametrize("name", ["q4km", "q5km", "f16", "q6k", "gqa8", "hd128"])
def test_batched_prefill_matches_oracle(tiny_model, name):
    path = tiny_model(name)
    hm = fb.HostModel(path)
    ctx = fb.Context(hm, max_seq=512)
    kv = ctx.kv(512)
    prompt = _prompt(hm.params.vocab_size, 150, 21)
    first = ctx.prefill(kv, prompt)
    dev, _ = ctx.decode_greedy(kv, first, len(prompt), 40)
    st = orc.Model(path).state(512, kv_fp16=True)
    want = st.generate(prompt, 40)
    assert first == want[0]
    assert dev.tolist() == want[1:].tolist()


@pytest.mark.parametrize("name", ["q4km", "gqa8"])
def test_batched_and_stepwise_prefill_fill_the_same_cache(tiny_model, name):
    path = tiny_model(name)
    hm = fb.HostModel(path)
    p = hm.params
    ctx = fb.Context(hm, max_seq=512)
    prompt = _prompt(p.vocab_size, 200, 22)
    kv_b = ctx.kv(512)
    first_b = ctx.prefill(kv_b, prompt)
    ctx.set_prefill_mode(1)
    kv_s = ctx.kv(512)
    first_s = ctx.prefill(kv_s, prompt)
    ctx.set_prefill_mode(0)
    assert first_b == first_s
    for layer in range(p.n_layers):
        kb, vb = kv_b.read(layer, 0, len(prompt))
        ks, vs = kv_s.read(layer, 0, len(prompt))
        for a, b in ((kb, ks), (vb, vs)):
            assert np.abs(a - b).max() <= 2e-3 * (np.abs(b).max() + 1e-3)
    # split over two calls (the second starts at position 70)
    kv_2 = ctx.kv(512)
    ctx.prefill(kv_2, prompt[:70])
    first_2 = ctx.prefill(kv_2, prompt[70:], start_pos=70)
    assert first_2 == first_b
    k2, _ = kv_2.read(0, 0, len(prompt))
    kb0, _ = kv_b.read(0, 0, len(prompt))
    assert np.abs(k2 - kb0).max() <= 2e-3 * (np.abs(kb0).max() + 1e-3)


def test_prefill_rejects_out_of_range(tiny_model):
    path = tiny_model("q4km")
    hm = fb.HostModel(path)
    ctx = fb.Context(hm, max_seq=64)
    kv = ctx.kv(64)
    with pytest.raises(fb.FiberError):
        ctx.prefill(kv, _prompt(hm.params.vocab_size, 70, 1))
    bad = _prompt(hm.params.vocab_size, 10, 2)
    bad[3] = hm.params.vocab_size
    with pytest.raises(fb.FiberError):
        ctx.prefill(kv, bad)
    assert ctx.prefill(kv, _prompt(hm.params.vocab_size, 10, 3)) >= 0  # still usable
