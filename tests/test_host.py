"""Host-side C: GGUF reader robustness, model validation, synthetic models and
quantizers (no GPU)."""
from __future__ import annotations

import os
import struct

import numpy as np
import pytest

import fiber_b200 as fb
from oracle import oracle as orc


def test_model_open_reads_params(tiny_model):
    m = fb.HostModel(tiny_model("gqa8"))
    p = m.params
    assert (p.dim, p.n_layers, p.n_heads, p.n_kv_heads, p.head_dim, p.ffn_dim, p.vocab_size) == (
        512, 3, 8, 1, 64, 1024, 1200)
    assert abs(p.rope_freq_base - 10000.0) < 1e-3 and abs(p.rms_norm_eps - 1e-5) < 1e-12
    assert p.arch == b"llama"


def _corrupt(src, dst, fn):
    data = bytearray(open(src, "rb").read())
    data = fn(data)
    open(dst, "wb").write(bytes(data))
    return dst


@pytest.mark.parametrize("case", ["truncated_header", "truncated_data", "bad_magic", "bad_version",
                                  "huge_kv_count", "huge_string", "bad_alignment", "tiny"])
def test_gguf_rejects_corrupt_files(tiny_model, tmp_path, case):
    src = tiny_model("q4km")
    size = os.path.getsize(src)

    def f(d):
        if case == "truncated_header":
            return d[:200]
        if case == "truncated_data":
            return d[: size - 1000]
        if case == "bad_magic":
            d[0:4] = b"GGUX"
        elif case == "bad_version":
            d[4:8] = struct.pack("<I", 9)
        elif case == "huge_kv_count":
            d[16:24] = struct.pack("<Q", 1 << 40)
        elif case == "huge_string":
            d[24:32] = struct.pack("<Q", 1 << 50)  # first key length
        elif case == "bad_alignment":
            i = d.find(b"general.alignment")
            d[i + 17 + 4:i + 17 + 8] = struct.pack("<I", 24)
        elif case == "tiny":
            return d[:10]
        return d

    path = _corrupt(src, str(tmp_path / f"{case}.gguf"), f)
    assert fb.host().gguf_open(path.encode()) is None
    with pytest.raises(RuntimeError):
        fb.HostModel(path)


def test_model_open_rejects_missing_tensor(tmp_path):
    cfg = fb.synth_cfg(dim=256, n_layers=1, n_heads=4, n_kv_heads=2, ffn_dim=256, vocab=400, recipe="Q4_K")
    path = str(tmp_path / "m.gguf")
    fb.write_model(path, cfg)
    data = bytearray(open(path, "rb").read())
    i = data.find(b"blk.0.ffn_up.weight")
    data[i:i + 4] = b"XXX."
    bad = str(tmp_path / "bad.gguf")
    open(bad, "wb").write(bytes(data))
    with pytest.raises(RuntimeError):
        fb.HostModel(bad)


@pytest.mark.parametrize("t,tol", [(fb.GGML_Q4_K, 0.12), (fb.GGML_Q5_K, 0.06), (fb.GGML_Q6_K, 0.03),
                                   (fb.GGML_F16, 1e-3)])
def test_quantizer_roundtrip_error(t, tol):
    x = fb.randn(64 * 1024, 21, 0.02).reshape(64, 1024)
    blocks = fb.quantize_rows(t, x)
    if t == fb.GGML_F16:
        back = blocks.view(np.float16).astype(np.float32).reshape(64, 1024)
    else:
        back = orc.dequant_f32(t, blocks, 64, 1024)
    rel = np.sqrt(np.mean((back - x) ** 2)) / np.sqrt(np.mean(x ** 2))
    assert rel < tol, rel


def test_synthetic_model_is_deterministic(tmp_path):
    cfg = fb.synth_cfg(dim=256, n_layers=1, n_heads=4, n_kv_heads=4, ffn_dim=256, vocab=400, recipe="Q4_K_M",
                       seed=5, n_threads=1)
    a = fb.write_model(str(tmp_path / "a.gguf"), cfg)
    cfg.n_threads = 4
    b = fb.write_model(str(tmp_path / "b.gguf"), cfg)
    assert open(a, "rb").read() == open(b, "rb").read()


def test_recipe_q4km_types(tiny_model):
    m = fb.HostModel(tiny_model("gqa8"))
    H = fb.host()
    g = m.gguf
    import ctypes as C

    class TI(C.Structure):
        _fields_ = [("name_len", C.c_uint64), ("name", C.c_char_p), ("n_dims", C.c_uint32),
                    ("dims", C.c_uint64 * 4), ("type", C.c_int)]

    def ttype(name):
        t = H.gguf_find_tensor(g, name.encode())
        return C.cast(t, C.POINTER(TI)).contents.type

    assert ttype("output.weight") == fb.GGML_Q6_K
    assert ttype("token_embd.weight") == fb.GGML_Q4_K
    assert ttype("blk.0.attn_v.weight") == fb.GGML_Q6_K and ttype("blk.0.ffn_down.weight") == fb.GGML_Q6_K
    assert ttype("blk.1.attn_v.weight") == fb.GGML_Q4_K and ttype("blk.1.ffn_down.weight") == fb.GGML_Q4_K
    assert ttype("blk.2.attn_q.weight") == fb.GGML_Q4_K
    assert ttype("blk.0.attn_norm.weight") == fb.GGML_F32


def test_random_blocks_fields():
    b = fb.random_blocks(fb.GGML_Q4_K, 4, 512, 3).reshape(-1, 144)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    assert (d >= 0).all() and d.max() < 0.01
    q = b[:, 16:]
    assert q.min() == 0 and q.max() == 255
