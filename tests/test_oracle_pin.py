"""Pin the restated oracle (oracle/oracle.c) to the reference's own C.

The reference ships no golden vectors or known-answer tests for this path, so
the pin is the reference itself, compiled from its sources into oracle/_ref
(oracle/Makefile): its dequant.h, gguf.c, sampler.c, tokenizer.c and the
cpu_forward_token of src/fiber_proof.m. The same checks also pin the product's
host C (GGUF reader, tokenizer, sampler) against the reference.
The committed fixtures in tests/golden/ (made by tests/golden/make_golden.py from
the reference build) cover the case where oracle/_ref is absent.
"""
from __future__ import annotations

import ctypes as C
import json
import os

import numpy as np
import pytest

import fiber_b200 as fb
from oracle import oracle as orc

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
need_ref = pytest.mark.skipif(not orc.ref_available(), reason="oracle/_ref not built (reference tree absent)")


@need_ref
@pytest.mark.parametrize("t", [fb.GGML_Q4_K, fb.GGML_Q6_K])
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_dequant_matches_reference_dequant_h(t, seed):
    rows, cols = 16, 1024
    blocks = fb.random_blocks(t, rows, cols, seed)
    a = orc.dequant_f16(t, blocks, rows, cols).view(np.uint16)
    b = orc.ref_dequant_f16(t, blocks, rows, cols).view(np.uint16)
    assert np.array_equal(a, b)


@need_ref
@pytest.mark.parametrize("t", [fb.GGML_Q4_K, fb.GGML_Q6_K])
def test_dequant_of_quantized_weights_matches_reference(t):
    x = fb.randn(8 * 512, 5, 0.02).reshape(8, 512)
    blocks = fb.quantize_rows(t, x)
    a = orc.dequant_f16(t, blocks, 8, 512).view(np.uint16)
    b = orc.ref_dequant_f16(t, blocks, 8, 512).view(np.uint16)
    assert np.array_equal(a, b)


def test_dequant_golden_vectors():
    with open(os.path.join(GOLDEN, "dequant.json")) as f:
        g = json.load(f)
    for case in g["cases"]:
        blocks = np.frombuffer(bytes.fromhex(case["blocks"]), np.uint8).copy()
        got = orc.dequant_f16(case["type"], blocks, case["rows"], case["cols"]).view(np.uint16)
        assert got.reshape(-1).tolist() == case["f16_bits"], case["type"]


def test_q5k_decode_follows_metal_layout():
    """Q5_K has no CPU dequant in the reference; check the oracle's decode of
    hand-built blocks against the Metal kernel's formula written out here."""
    rng = np.random.default_rng(0)
    blk = rng.integers(0, 256, 176, dtype=np.uint8)
    blk[0:2] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
    blk[2:4] = np.frombuffer(np.float16(0.003).tobytes(), np.uint8)
    got = orc.dequant_f32(fb.GGML_Q5_K, blk, 1, 256)[0]
    sc = blk[4:16]
    d, dm = np.float32(np.float16(0.01)), np.float32(np.float16(0.003))

    def smk(j):
        if j < 4:
            return sc[j] & 63, sc[j + 4] & 63
        return (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4), (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4)

    for e in range(256):
        g_, s, w = e // 64, (e // 32) & 1, e % 32
        q = blk[48 + 32 * g_ + w]
        nib = (q >> 4) if s else (q & 0xF)
        hi = (blk[16 + w] >> (2 * g_ + s)) & 1
        sv, mv = smk(2 * g_ + s)
        want = np.float32(np.float32(d * np.float32(sv)) * np.float32(nib + 16 * hi)) - np.float32(dm * np.float32(mv))
        assert got[e] == np.float32(want), e


@need_ref
@pytest.mark.parametrize("name", ["q4km", "f16", "q6k", "gqa8", "hd128"])
def test_forward_matches_reference_cpu_forward_token(tiny_model, name):
    path = tiny_model(name)
    m = orc.Model(path)
    r = orc.RefModel(path)
    st, rk = m.state(64), r.kv(64)
    toks = [1, 17, 300, 42, 7, 99, 5, 250]
    for pos, t in enumerate(toks):
        a, b = st.forward(t, pos), rk.forward(t, pos)
        assert np.array_equal(a, b), (name, pos, float(np.abs(a - b).max()))


def test_forward_golden_logits(tiny_model):
    """Logits of the reference's cpu_forward_token on the committed tiny model
    (fixture written by tests/golden/make_golden.py)."""
    with open(os.path.join(GOLDEN, "forward.json")) as f:
        g = json.load(f)
    path = tiny_model(g["model"])
    m = orc.Model(path)
    st = m.state(64)
    for step in g["steps"]:
        lg = st.forward(step["token"], step["pos"])
        idx = np.array(step["idx"])
        assert np.array_equal(lg[idx].view(np.uint32), np.array(step["bits"], np.uint32)), step["pos"]
        assert int(np.argmax(lg)) == step["argmax"]


@need_ref
def test_gguf_reader_matches_reference(tiny_model):
    path = tiny_model("q4km").encode()
    R = orc.ref()
    H = fb.host()
    a, b = H.gguf_open(path), R.gguf_open(path)
    try:
        for key in [b"llama.block_count", b"llama.embedding_length", b"llama.attention.head_count_kv",
                    b"llama.feed_forward_length", b"general.alignment", b"tokenizer.ggml.bos_token_id"]:
            assert H.gguf_get_u32(a, key, 7) == R.gguf_get_u32(b, key, 7)
        for key in [b"llama.rope.freq_base", b"llama.attention.layer_norm_rms_epsilon"]:
            assert H.gguf_get_f32(a, key, 0.0) == R.gguf_get_f32(b, key, 0.0)
        assert H.gguf_get_str(a, b"general.architecture") == R.gguf_get_str(b, b"general.architecture")
        for name in [b"token_embd.weight", b"blk.0.attn_q.weight", b"blk.1.ffn_down.weight", b"output.weight",
                     b"output_norm.weight"]:
            ta, tb = H.gguf_find_tensor(a, name), R.gguf_find_tensor(b, name)
            assert ta and tb
            da, db = H.gguf_tensor_data(a, ta), R.gguf_tensor_data(b, tb)
            assert C.string_at(da, 256) == C.string_at(db, 256)
        assert H.gguf_find_tensor(a, b"nope") is None and R.gguf_find_tensor(b, b"nope") is None
    finally:
        H.gguf_close(a)
        R.gguf_close(b)


@need_ref
def test_tokenizer_matches_reference(tiny_model):
    path = tiny_model("q4km")
    hm = fb.HostModel(path)
    tok = fb.Tokenizer(hm)
    R = orc.ref()
    g = R.gguf_open(path.encode())
    rt = R.tokenizer_init(g)
    rng = np.random.default_rng(3)
    alphabet = list("abcdefghijklmnopqrstuvwxyz   ,.!?0123456789") + ["é", "ß", "日本", "\n", "\t"]
    texts = ["Hello world", "the quick brown fox", " leading space", "", "a", "zz zz zz"]
    texts += ["".join(rng.choice(alphabet, size=rng.integers(1, 60))) for _ in range(200)]
    try:
        for t in texts:
            mine = tok.encode(t, 512)
            out = np.zeros(512, np.int32)
            n = R.tokenizer_encode(rt, t.encode(), out, 512)
            assert mine.tolist() == out[:n].tolist(), repr(t)
            for i in mine.tolist():
                assert tok.decode(i) == R.tokenizer_decode(rt, i)
    finally:
        R.tokenizer_free(rt)
        R.gguf_close(g)


@need_ref
@pytest.mark.parametrize("temp,top_k,top_p", [(0.0, 40, 0.9), (0.7, 40, 0.9), (1.0, 0, 1.0), (0.5, 5, 0.5),
                                              (1.3, 100, 0.95)])
def test_sampler_matches_reference(temp, top_k, top_p):
    rng = np.random.default_rng(9)
    R = orc.ref()
    st = fb.Sampler()
    fb.host().sampler_init(C.byref(st), 1000, temp, top_k, top_p)
    rs = fb.Sampler()
    R.sampler_init(C.byref(rs), 1000, temp, top_k, top_p)
    for _ in range(50):
        lg = (rng.standard_normal(1000) * 3).astype(np.float32)
        lg[rng.integers(0, 1000)] = lg.max()  # planted tie
        a = fb.host().sampler_sample(C.byref(st), lg)
        b = R.sampler_sample(C.byref(rs), lg)
        assert a == b
