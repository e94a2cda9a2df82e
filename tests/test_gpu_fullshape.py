"""Greedy-token and logit parity at the benchmark workloads' real shapes.

The fixtures (tests/golden/fullshape_*.json / .npz) hold the oracle's greedy token
sequence, its per-step top-2 margins and teacher-forced logits for each workload, and
the SHA-256 of the seeded GGUF they were computed on; tests/golden/make_fullshape.py
writes them. Here the same seeded model is rebuilt (the hash must match), decoded on the
GPU through the C-ABI and compared: tokens bit-exact, logits within 2e-2 max-abs and
1e-3 relative RMS. Workloads:

* 1.1B Q4_K_M (TinyLlama shape): 128-token prompt (batched prefill, and token by
  token), then 512 greedy steps, in every decode mode that covers the model;
* stories fp16 (dim 768, 12 layers): 32-token prompt, 256 steps;
* 1.1B Q5_K_M with the KV cache pre-filled to 2048 positions: 64 steps at batch 1,
  and the same from 8 KV slots at once (batched decode);
* 7B Q4_K_M: 512-token prompt, 32 steps.
"""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np
import pytest

import fiber_b200 as fb

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
MAX_ABS, REL_RMS = 2e-2, 1e-3
SEED = 1234


def _fixture(name):
    path = os.path.join(HERE, "golden", f"fullshape_{name}.json")
    if not os.path.exists(path):
        pytest.skip(f"fixture {path} not generated")
    with open(path) as f:
        fx = json.load(f)
    arrays = np.load(os.path.join(HERE, "golden", f"fullshape_{name}.npz"))
    return fx, {int(k.split("_")[1]): arrays[k].astype(np.float32) for k in arrays.files}


def _model(tmp_path_factory, fx):
    path = str(tmp_path_factory.getbasetemp() / f"fullshape_{fx['workload']}.gguf")
    if not os.path.exists(path):
        fb.write_model(path, fb.synth_cfg(fx["preset"], seed=fx["seed"]))
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    assert h.hexdigest() == fx["sha256"], "the seeded model differs from the one the fixture was computed on"
    return path


def _prompt(vocab, n):
    return np.random.default_rng(SEED).integers(1, vocab, n).astype(np.int32)


def _rel_rms(a, b):
    return float(np.sqrt(np.mean((a.astype(np.float64) - b) ** 2)) / np.sqrt(np.mean(b.astype(np.float64) ** 2)))


def _check_logits(ctx, kv, fx, logits, prompt):
    """Teacher-forced logits at the fixture's steps (the cache already holds every row)."""
    P, toks = fx["prompt_len"], fx["tokens"]
    for s, want in logits.items():
        tok = int(prompt[P - 1]) if s == 0 else toks[s - 1]
        am, lg = ctx.forward(kv, tok, P - 1 + s)
        assert np.abs(lg - want).max() < MAX_ABS, (fx["workload"], s)
        assert _rel_rms(lg, want) < REL_RMS, (fx["workload"], s)
        assert am == toks[s]


def _modes(ctx):
    out = []
    for m in (2, 0, 1):
        try:
            ctx.set_mode(m)
            out.append(m)
        except fb.FiberError:
            pass
    return out


@pytest.mark.parametrize("name", ["tinyllama", "stories"])
def test_prompted_decode_matches_oracle(tmp_path_factory, name):
    fx, logits = _fixture(name)
    path = _model(tmp_path_factory, fx)
    hm = fb.HostModel(path)
    P, D = fx["prompt_len"], fx["decode_steps"]
    prompt = _prompt(hm.params.vocab_size, P)
    ctx = fb.Context(hm, max_seq=P + D + 1)
    kv = ctx.kv(P + D + 1)
    modes = _modes(ctx)
    assert 2 in modes or 0 in modes, "no one-kernel decode mode covers the workload"
    for mode in modes:
        ctx.set_mode(mode)
        first = ctx.prefill(kv, prompt)  # batched (tensor-core) prefill
        assert first == fx["tokens"][0], mode
        toks, _ = ctx.decode_greedy(kv, first, P, D)
        assert toks.tolist() == fx["tokens"][1:], (mode, next(i for i, (a, b) in enumerate(
            zip(toks.tolist(), fx["tokens"][1:])) if a != b))
    _check_logits(ctx, kv, fx, logits, prompt)
    # token-by-token prefill (the reference's own prefill loop) gives the same tokens
    ctx.set_prefill_mode(1)
    first = ctx.prefill(kv, prompt)
    assert first == fx["tokens"][0]
    toks, _ = ctx.decode_greedy(kv, first, P, min(D, 64))
    assert toks.tolist() == fx["tokens"][1:len(toks) + 1]
    ctx.close()


def _fill_q5(kv, hm, P, slots):
    p = hm.params
    kvd = p.n_kv_heads * p.head_dim
    for layer in range(p.n_layers):
        k = fb.randn(P * kvd, seed=100 + layer).reshape(P, kvd)
        v = fb.randn(P * kvd, seed=200 + layer).reshape(P, kvd)
        for s in range(slots):
            kv.write(layer, 0, k, v, slot=s)


def test_long_context_q5km_batch1(tmp_path_factory):
    fx, logits = _fixture("q5long")
    path = _model(tmp_path_factory, fx)
    hm = fb.HostModel(path)
    P, D = fx["context"], fx["decode_steps"]
    ctx = fb.Context(hm, max_seq=P + D + 1)
    kv = ctx.kv(P + D + 1)
    _fill_q5(kv, hm, P, 1)
    slot0 = fx["slots"][0]
    for mode in _modes(ctx):
        ctx.set_mode(mode)
        toks, _ = ctx.decode_greedy(kv, slot0["first"], P, D)
        assert toks.tolist() == slot0["tokens"], mode
    for s, want in logits.items():
        tok = slot0["first"] if s == 0 else slot0["tokens"][s - 1]
        am, lg = ctx.forward(kv, tok, P + s)
        assert np.abs(lg - want).max() < MAX_ABS, s
        assert _rel_rms(lg, want) < REL_RMS, s
    ctx.close()


def test_long_context_q5km_eight_slots(tmp_path_factory):
    fx, _ = _fixture("q5long")
    path = _model(tmp_path_factory, fx)
    hm = fb.HostModel(path)
    P, D = fx["context"], fx["decode_steps"]
    B = len(fx["slots"])
    ctx = fb.Context(hm, max_seq=P + D + 1, max_batch=B)
    kv = ctx.kv(P + D + 1, max_batch=B)
    _fill_q5(kv, hm, P, B)
    firsts = [s["first"] for s in fx["slots"]]
    toks, _ = ctx.decode_greedy_batch(kv, firsts, [P] * B, D)
    for s in range(B):
        assert toks[:, s].tolist() == fx["slots"][s]["tokens"], s
    ctx.close()


def test_llama7b_prompted_decode(tmp_path_factory):
    fx, logits = _fixture("llama7b")
    path = _model(tmp_path_factory, fx)
    hm = fb.HostModel(path)
    P, D = fx["prompt_len"], fx["decode_steps"]
    prompt = _prompt(hm.params.vocab_size, P)
    ctx = fb.Context(hm, max_seq=P + D + 1)
    kv = ctx.kv(P + D + 1)
    for mode in _modes(ctx):
        ctx.set_mode(mode)
        first = ctx.prefill(kv, prompt)
        assert first == fx["tokens"][0], mode
        toks, _ = ctx.decode_greedy(kv, first, P, D)
        assert toks.tolist() == fx["tokens"][1:], mode
    _check_logits(ctx, kv, fx, logits, prompt)
    ctx.close()
