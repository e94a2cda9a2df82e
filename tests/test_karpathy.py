"""karpathy / llama2.c checkpoint loader (include/fiber_ckpt.h): the converted GGUF holds
every array of the .bin at the offsets of the llama2.c layout (the reference's
fiber_model_load_karpathy, src/fiber_ckpt.m:125-259), matrices and embedding rounded to
fp16, norms in fp32; the header gives the model parameters; separate classifiers sit
after the freq_cis tables; bad files are rejected."""
from __future__ import annotations

import ctypes as C
import struct

import numpy as np
import pytest

import fiber_b200 as fb


def write_bin(path, dim=256, hidden=512, n_layers=2, n_heads=4, n_kv_heads=2, vocab=400, seq=64, shared=True,
              seed=3, truncate=0):
    """A llama2.c checkpoint with seeded N(0, 0.05) arrays; returns the arrays by name."""
    rng = np.random.default_rng(seed)
    hd = dim // n_heads
    kv = n_kv_heads * hd
    shapes = [("embd", (vocab, dim)), ("rms_att", (n_layers, dim)), ("wq", (n_layers, dim, dim)),
              ("wk", (n_layers, kv, dim)), ("wv", (n_layers, kv, dim)), ("wo", (n_layers, dim, dim)),
              ("rms_ffn", (n_layers, dim)), ("w1", (n_layers, hidden, dim)), ("w2", (n_layers, dim, hidden)),
              ("w3", (n_layers, hidden, dim)), ("rms_final", (dim,)), ("freq_real", (seq, hd // 2)),
              ("freq_imag", (seq, hd // 2))]
    if not shared:
        shapes.append(("wcls", (vocab, dim)))
    arrs = {n: (rng.standard_normal(sh) * 0.05).astype(np.float32) for n, sh in shapes}
    for n in ("rms_att", "rms_ffn", "rms_final"):
        arrs[n] = (1 + 0.1 * rng.standard_normal(arrs[n].shape)).astype(np.float32)
    blob = struct.pack("7i", dim, hidden, n_layers, n_heads, n_kv_heads, vocab if shared else -vocab, seq)
    blob += b"".join(arrs[n].tobytes() for n, _ in shapes)
    with open(path, "wb") as f:
        f.write(blob[: len(blob) - truncate] if truncate else blob)
    return arrs


class _TI(C.Structure):
    _fields_ = [("name_len", C.c_uint64), ("name", C.c_char_p), ("n_dims", C.c_uint32), ("dims", C.c_uint64 * 4),
                ("type", C.c_int), ("offset", C.c_uint64), ("size_bytes", C.c_size_t), ("n_elements", C.c_uint64)]


def _tensor(hm, name):
    H = fb.host()
    t = H.gguf_find_tensor(hm.gguf, name.encode())
    assert t, name
    ti = C.cast(t, C.POINTER(_TI)).contents
    data = H.gguf_tensor_data(hm.gguf, t)
    n = int(ti.n_elements)
    if ti.type == fb.GGML_F16:
        return np.ctypeslib.as_array(C.cast(data, C.POINTER(C.c_uint16)), (n,)).view(np.float16).astype(np.float32), ti
    assert ti.type == fb.GGML_F32
    return np.ctypeslib.as_array(C.cast(data, C.POINTER(C.c_float)), (n,)).copy(), ti


@pytest.mark.parametrize("shared", [True, False])
def test_converted_tensors_match_the_checkpoint(tmp_path, shared):
    b = str(tmp_path / "m.bin")
    g = str(tmp_path / "m.gguf")
    arrs = write_bin(b, shared=shared)
    cfg = fb.karpathy_config(b)
    assert (cfg.dim, cfg.hidden_dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.vocab_size, cfg.seq_len) == \
        (256, 512, 2, 4, 2, 400, 64)
    assert cfg.shared_classifier == int(shared)
    fb.karpathy_to_gguf(b, g)
    hm = fb.HostModel(g)
    p = hm.params
    assert (p.dim, p.ffn_dim, p.n_layers, p.n_heads, p.n_kv_heads, p.vocab_size, p.context_length) == \
        (256, 512, 2, 4, 2, 400, 64)
    f16 = lambda a: a.astype(np.float16).astype(np.float32).reshape(-1)  # noqa: E731
    got, ti = _tensor(hm, "token_embd.weight")
    assert ti.type == fb.GGML_F16 and np.array_equal(got, f16(arrs["embd"]))
    got, _ = _tensor(hm, "output_norm.weight")
    assert np.array_equal(got, arrs["rms_final"])
    H = fb.host()
    if shared:
        assert not H.gguf_find_tensor(hm.gguf, b"output.weight")  # tied: the embedding classifies
    else:
        got, _ = _tensor(hm, "output.weight")
        assert np.array_equal(got, f16(arrs["wcls"]))
    names = {"attn_q": "wq", "attn_k": "wk", "attn_v": "wv", "attn_output": "wo", "ffn_gate": "w1",
             "ffn_down": "w2", "ffn_up": "w3"}
    for l in range(2):
        for gname, bname in names.items():
            got, ti = _tensor(hm, f"blk.{l}.{gname}.weight")
            want = arrs[bname][l]
            assert (ti.dims[0], ti.dims[1]) == (want.shape[1], want.shape[0]), gname  # [in, out]
            assert np.array_equal(got, f16(want)), (l, gname)
        for gname, bname in (("attn_norm", "rms_att"), ("ffn_norm", "rms_ffn")):
            got, _ = _tensor(hm, f"blk.{l}.{gname}.weight")
            assert np.array_equal(got, arrs[bname][l]), (l, gname)


def test_bad_checkpoints_are_rejected(tmp_path):
    b = str(tmp_path / "t.bin")
    write_bin(b, truncate=100)  # shorter than its header says
    with pytest.raises(ValueError):
        fb.karpathy_to_gguf(b, str(tmp_path / "t.gguf"))
    write_bin(b, dim=288, n_heads=6, n_kv_heads=6)  # stories15M shape: not a multiple of 256
    with pytest.raises(ValueError):
        fb.karpathy_to_gguf(b, str(tmp_path / "t.gguf"))
    with open(b, "wb") as f:
        f.write(struct.pack("7i", 256, 512, 2, 3, 2, 400, 64))  # heads do not divide dim
    with pytest.raises(ValueError):
        fb.karpathy_config(b)
    with pytest.raises(ValueError):
        fb.karpathy_to_gguf(str(tmp_path / "missing.bin"), str(tmp_path / "t.gguf"))
