"""End-to-end decode parity on the GPU against the CPU oracle.

The oracle runs with fp16 K/V storage (oracle.h: kv_fp16) so both sides keep
the same cache precision. Bars (from the north star): greedy token sequences
identical; logits within 2e-2 max-abs and 1e-3 relative RMS (fp32 accumulation).
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


def _ctx(hm, max_seq, mode):
    """Context in decode mode `mode` (0 grid-barrier persistent kernel, 1 one kernel per
    phase, 2 dataflow kernel); skips when that kernel does not cover the model."""
    ctx = fb.Context(hm, max_seq=max_seq)
    try:
        ctx.set_mode(mode)
    except fb.FiberError:
        pytest.skip(f"decode mode {mode} does not cover this model")
    return ctx


def _prompt(vocab, n, seed):
    rng = np.random.default_rng(seed)
    return rng.integers(1, vocab, n).astype(np.int32)


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("name", ["q4km", "q5km", "f16", "q6k", "gqa8", "hd128"])
def test_teacher_forced_logits(tiny_model, name, mode):
    path = tiny_model(name)
    hm = fb.HostModel(path)
    ctx = _ctx(hm, 256, mode)
    kv = ctx.kv(256)
    om = orc.Model(path)
    st = om.state(256, kv_fp16=True)
    toks = _prompt(hm.params.vocab_size, 80, 1)  # crosses a 64-position page
    for pos, t in enumerate(toks):
        am, lg = ctx.forward(kv, int(t), pos)
        want = st.forward(int(t), pos)
        assert np.abs(lg - want).max() < MAX_ABS, (name, pos)
        assert _rel_rms(lg, want) < REL_RMS, (name, pos)
        assert am == int(np.argmax(lg))


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("name", ["q4km", "q5km", "f16", "gqa8"])
def test_greedy_tokens_match_oracle(tiny_model, name, mode):
    path = tiny_model(name)
    hm = fb.HostModel(path)
    ctx = _ctx(hm, 512, mode)
    kv = ctx.kv(512)
    prompt = _prompt(hm.params.vocab_size, 16, 2)
    n_gen = 150
    first = ctx.prefill(kv, prompt)
    dev, _ = ctx.decode_greedy(kv, first, len(prompt), n_gen)
    om = orc.Model(path)
    st = om.state(512, kv_fp16=True)
    want = st.generate(prompt, n_gen)
    assert first == want[0]
    assert dev.tolist() == want[1:].tolist()


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_device_loop_equals_host_loop(tiny_model, mode):
    path = tiny_model("gqa8")
    hm = fb.HostModel(path)
    ctx = _ctx(hm, 512, mode)
    prompt = _prompt(hm.params.vocab_size, 10, 3)
    kv1 = ctx.kv(512)
    first = ctx.prefill(kv1, prompt)
    dev, _ = ctx.decode_greedy(kv1, first, len(prompt), 70)
    kv2 = ctx.kv(512)
    assert ctx.prefill(kv2, prompt) == first
    tok, host_seq = first, []
    for i in range(70):
        tok, _ = ctx.forward(kv2, tok, len(prompt) + i, want_logits=False)
        host_seq.append(tok)
    assert dev.tolist() == host_seq
    k1, v1 = kv1.read(1, 0, 80)
    k2, v2 = kv2.read(1, 0, 80)
    assert np.array_equal(k1, k2) and np.array_equal(v1, v2)


def test_kv_cache_contents_match_oracle(tiny_model):
    path = tiny_model("q4km")
    hm = fb.HostModel(path)
    ctx = fb.Context(hm, max_seq=256)
    kv = ctx.kv(256)
    om = orc.Model(path)
    st = om.state(256, kv_fp16=True)
    toks = _prompt(hm.params.vocab_size, 70, 4)
    for pos, t in enumerate(toks):
        ctx.forward(kv, int(t), pos, want_logits=False)
        st.forward(int(t), pos)
    kvd = hm.params.n_kv_heads * hm.params.head_dim
    for layer in range(hm.params.n_layers):
        k, v = kv.read(layer, 0, len(toks))
        ok = np.empty(kvd, np.float32)
        ov = np.empty(kvd, np.float32)
        for pos in [0, 1, 63, 64, 69]:
            orc.lib().orc_state_get_kv(st.h, layer, pos, ok, ov)
            assert np.abs(k[pos] - ok).max() <= 2e-3 * (np.abs(ok).max() + 1e-3)
            assert np.abs(v[pos] - ov).max() <= 2e-3 * (np.abs(ov).max() + 1e-3)


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_prefilled_long_context(tiny_model, mode):
    """Long context over many KV pages: cache pre-filled with seeded N(0,1)
    keys/values (as in the long-context workload), then greedy decode."""
    path = tiny_model("gqa8")
    hm = fb.HostModel(path)
    p = hm.params
    ctx = _ctx(hm, 1024, mode)
    kv = ctx.kv(1024)
    om = orc.Model(path)
    st = om.state(1024, kv_fp16=True)
    n_fill = 700
    kvd = p.n_kv_heads * p.head_dim
    for layer in range(p.n_layers):
        k = fb.randn(n_fill * kvd, seed=100 + layer).reshape(n_fill, kvd)
        v = fb.randn(n_fill * kvd, seed=200 + layer).reshape(n_fill, kvd)
        kv.write(layer, 0, k, v)
        for pos in range(n_fill):
            st.set_kv(layer, pos, k[pos], v[pos])
    first = 5
    dev, _ = ctx.decode_greedy(kv, first, n_fill, 40)
    want = st.generate(np.array([first], np.int32), 39, start=n_fill)
    assert dev.tolist() == want.tolist()


def test_reference_named_api(tiny_model):
    """gpu_init / gpu_embed / gpu_forward_token / gpu_get_logits as the
    reference's main.m drives them (src/main.m:60-64, 568-586)."""
    import ctypes as C

    path = tiny_model("q4km")
    hm = fb.HostModel(path)
    L = fb.cuda_lib()
    ctx = L.gpu_init(hm.h)
    assert ctx
    p = hm.params
    kvp = L.kv_cache_init(L.gpu_get_device(ctx), p.n_layers, p.n_kv_heads, p.head_dim, 128)
    kv = C.cast(kvp, C.c_void_p).value
    om = orc.Model(path)
    st = om.state(128, kv_fp16=True)
    try:
        tok = 1
        for pos in range(20):
            L.gpu_embed(ctx, hm.h, tok)
            ms = L.gpu_forward_token(ctx, hm.h, kv, pos)
            assert ms >= 0
            lg = np.ctypeslib.as_array(L.gpu_get_logits(ctx), shape=(p.vocab_size,)).copy()
            want = st.forward(tok, pos)
            assert np.abs(lg - want).max() < MAX_ABS
            tok = int(np.argmax(lg))
        assert L.gpu_forward_token(ctx, hm.h, kv, 128) < 0  # past the cache: error, no fault
    finally:
        L.kv_cache_free(kv)
        L.gpu_free(ctx)


def test_errors_are_reported_not_faulted(tiny_model):
    path = tiny_model("q4km")
    hm = fb.HostModel(path)
    ctx = fb.Context(hm, max_seq=64)
    kv = ctx.kv(64)
    with pytest.raises(fb.FiberError):
        ctx.forward(kv, 1, 64)
    with pytest.raises(fb.FiberError):
        ctx.forward(kv, hm.params.vocab_size, 0)
    with pytest.raises(fb.FiberError):
        ctx.decode_greedy(kv, 1, 60, 10)
    am, _ = ctx.forward(kv, 1, 0)  # context still usable
    assert 0 <= am < hm.params.vocab_size


@pytest.mark.parametrize("mode", [0, 2])
@pytest.mark.parametrize("name", ["q4km", "f16", "gqa8", "hd128", "q6k"])
def test_persistent_and_per_phase_kernels_agree(tiny_model, name, mode):
    """The one-kernel steps and the per-phase kernels compute the same arithmetic per
    row; the token sequences must match and the logits agree to fp32 reordering noise."""
    path = tiny_model(name)
    hm = fb.HostModel(path)
    a = _ctx(hm, 256, mode)
    b = _ctx(hm, 256, 1)
    ka, kb = a.kv(256), b.kv(256)
    toks = _prompt(hm.params.vocab_size, 70, 9)
    for pos, t in enumerate(toks):
        ia, la = a.forward(ka, int(t), pos)
        ib, lb = b.forward(kb, int(t), pos)
        assert np.abs(la - lb).max() <= 1e-4 * (np.abs(lb).max() + 1), pos
        assert ia == ib, pos
    ga, _ = a.decode_greedy(ka, 3, len(toks), 60)
    gb, _ = b.decode_greedy(kb, 3, len(toks), 60)
    assert ga.tolist() == gb.tolist()


@pytest.mark.parametrize("mode", [0, 2])
@pytest.mark.parametrize("ring_kb", [64, 96])
def test_ring_filled_exactly_by_attention_pages(tiny_model, monkeypatch, ring_kb, mode):
    """A weight/KV ring whose size is a multiple of the attention page pair (head_dim
    128: 32 KB of K and V per page), so a tile can end exactly at the ring's end and
    the next one must start again at the front. Positions up to 199 need up to four
    pages per head, more than such a ring holds at once."""
    monkeypatch.setenv("FIBER_PK_RING_KB", str(ring_kb))
    monkeypatch.setenv("FIBER_FL_RING_KB", str(ring_kb))
    path = tiny_model("q6k")
    hm = fb.HostModel(path)
    a = _ctx(hm, 256, mode)
    assert a.ring_bytes == ring_kb * 1024, "the requested ring is not the one in use"
    b = _ctx(hm, 256, 1)
    ka, kb = a.kv(256), b.kv(256)
    toks = _prompt(hm.params.vocab_size, 200, 11)
    for pos, t in enumerate(toks):
        ia, la = a.forward(ka, int(t), pos)
        ib, lb = b.forward(kb, int(t), pos)
        assert np.abs(la - lb).max() <= 1e-4 * (np.abs(lb).max() + 1), pos
        assert ia == ib, pos
