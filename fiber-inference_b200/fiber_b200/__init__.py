"""fiber_b200 -- Python bindings (ctypes) over the two product libraries.

* ``lib/libfiber_host.so``: GGUF reader, model loader, tokenizer, sampler and
  synthetic-model writer (C).
* ``lib/libfiber_cuda.so``: the sm_100a decode path behind the ``extern "C"``
  API of include/gpu_ffn.h, include/kv_cache.h and include/fiber_cuda.h.

Nothing here computes: every call goes to the C/CUDA libraries. There is no CPU
fallback -- when ``libfiber_cuda.so`` is missing or cannot reach a GPU, the calls
raise.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_DIR = os.path.join(PKG_DIR, "lib")
HOST_SO = os.path.join(LIB_DIR, "libfiber_host.so")
CUDA_SO = os.path.join(LIB_DIR, "libfiber_cuda.so")

GGML_F32, GGML_F16, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K = 0, 1, 12, 13, 14
BLOCK_BYTES = {GGML_Q4_K: 144, GGML_Q5_K: 176, GGML_Q6_K: 210}
RECIPES = {"F16": 0, "Q4_K_M": 1, "Q5_K_M": 2, "Q4_K": 3, "Q6_K": 4, "Q5_K": 5}

F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
I32P = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


class SynthCfg(C.Structure):
    _fields_ = [
        ("dim", C.c_uint32), ("n_layers", C.c_uint32), ("n_heads", C.c_uint32),
        ("n_kv_heads", C.c_uint32), ("ffn_dim", C.c_uint32), ("vocab", C.c_uint32),
        ("context_length", C.c_uint32), ("rope_base", C.c_float), ("eps", C.c_float),
        ("recipe", C.c_int), ("weight_std", C.c_float), ("norm_value", C.c_float),
        ("seed", C.c_uint64), ("tied", C.c_int), ("n_threads", C.c_int), ("ffn_norm_value", C.c_float),
    ]


class ModelParams(C.Structure):
    _fields_ = [
        ("n_layers", C.c_uint32), ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32),
        ("dim", C.c_uint32), ("head_dim", C.c_uint32), ("ffn_dim", C.c_uint32),
        ("vocab_size", C.c_uint32), ("context_length", C.c_uint32),
        ("rope_freq_base", C.c_float), ("rms_norm_eps", C.c_float), ("arch", C.c_char_p),
    ]


class Sampler(C.Structure):
    _fields_ = [("vocab_size", C.c_int), ("temperature", C.c_float), ("top_k", C.c_int),
                ("top_p", C.c_float), ("rng_state", C.c_ulonglong)]


_host = None


def host() -> C.CDLL:
    global _host
    if _host is None:
        if not os.path.exists(HOST_SO):
            raise RuntimeError(f"{HOST_SO} missing: run `make -C fiber-inference_b200 host`")
        H = C.CDLL(HOST_SO)
        H.fiber_synth_preset.argtypes = [C.c_char_p, C.POINTER(SynthCfg)]
        H.fiber_synth_write_gguf.argtypes = [C.c_char_p, C.POINTER(SynthCfg)]
        H.fiber_synth_recipe_type.argtypes = [C.c_int, C.c_int, C.c_uint32, C.c_uint32]
        H.fiber_quantize_rows.argtypes = [C.c_int, F32P, C.c_void_p, C.c_size_t, C.c_size_t]
        H.fiber_random_blocks.argtypes = [C.c_int, C.c_void_p, C.c_size_t, C.c_size_t, C.c_uint64,
                                          C.c_float, C.c_float]
        H.fiber_randn.argtypes = [F32P, C.c_size_t, C.c_uint64, C.c_float]
        H.model_open.restype = C.c_void_p
        H.model_open.argtypes = [C.c_char_p]
        H.model_close.argtypes = [C.c_void_p]
        H.model_get_params.argtypes = [C.c_void_p, C.POINTER(ModelParams)]
        H.model_gguf.restype = C.c_void_p
        H.model_gguf.argtypes = [C.c_void_p]
        H.gguf_open.restype = C.c_void_p
        H.gguf_open.argtypes = [C.c_char_p]
        H.gguf_close.argtypes = [C.c_void_p]
        H.gguf_get_u32.restype = C.c_uint32
        H.gguf_get_u32.argtypes = [C.c_void_p, C.c_char_p, C.c_uint32]
        H.gguf_get_f32.restype = C.c_float
        H.gguf_get_f32.argtypes = [C.c_void_p, C.c_char_p, C.c_float]
        H.gguf_get_str.restype = C.c_char_p
        H.gguf_get_str.argtypes = [C.c_void_p, C.c_char_p]
        H.gguf_find_tensor.restype = C.c_void_p
        H.gguf_find_tensor.argtypes = [C.c_void_p, C.c_char_p]
        H.gguf_tensor_data.restype = C.c_void_p
        H.gguf_tensor_data.argtypes = [C.c_void_p, C.c_void_p]
        H.ggml_type_size.restype = C.c_size_t
        H.ggml_type_size.argtypes = [C.c_int]
        H.ggml_block_size.restype = C.c_size_t
        H.ggml_block_size.argtypes = [C.c_int]
        H.tokenizer_init.restype = C.c_void_p
        H.tokenizer_init.argtypes = [C.c_void_p]
        H.tokenizer_free.argtypes = [C.c_void_p]
        H.tokenizer_encode.argtypes = [C.c_void_p, C.c_char_p, I32P, C.c_int]
        H.tokenizer_decode.restype = C.c_char_p
        H.tokenizer_decode.argtypes = [C.c_void_p, C.c_int]
        H.tokenizer_eos.argtypes = [C.c_void_p]
        H.tokenizer_bos.argtypes = [C.c_void_p]
        H.sampler_init.argtypes = [C.POINTER(Sampler), C.c_int, C.c_float, C.c_int, C.c_float]
        H.sampler_sample.argtypes = [C.POINTER(Sampler), F32P]
        H.fiber_karpathy_config.argtypes = [C.c_char_p, C.POINTER(KarpathyConfig)]
        H.fiber_karpathy_to_gguf.argtypes = [C.c_char_p, C.c_char_p]
        H.model_open_karpathy.restype = C.c_void_p
        H.model_open_karpathy.argtypes = [C.c_char_p, C.c_char_p]
        _host = H
    return _host


# ---- synthetic models and blocks ------------------------------------------------

class KarpathyConfig(C.Structure):
    """fiber_karpathy_config_t (include/fiber_ckpt.h)."""
    _fields_ = [(n, C.c_int32) for n in ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size",
                                         "seq_len", "shared_classifier")]


def karpathy_config(bin_path: str) -> KarpathyConfig:
    """Header of a karpathy / llama2.c checkpoint (fiber_karpathy_config)."""
    out = KarpathyConfig()
    if host().fiber_karpathy_config(bin_path.encode(), C.byref(out)) != 0:
        raise ValueError(f"not a karpathy checkpoint: {bin_path}")
    return out


def karpathy_to_gguf(bin_path: str, gguf_path: str) -> str:
    """Rewrite a karpathy / llama2.c checkpoint as a Llama GGUF (fiber_karpathy_to_gguf)."""
    if host().fiber_karpathy_to_gguf(bin_path.encode(), gguf_path.encode()) != 0:
        raise ValueError(f"cannot convert {bin_path}")
    return gguf_path


def synth_cfg(preset: str | None = None, **over) -> SynthCfg:
    cfg = SynthCfg()
    if preset is not None:
        if host().fiber_synth_preset(preset.encode(), C.byref(cfg)) != 0:
            raise ValueError(f"unknown preset {preset}")
    else:
        cfg.rope_base, cfg.eps, cfg.weight_std, cfg.norm_value = 10000.0, 1e-5, 0.02, 1.0
        cfg.seed, cfg.vocab, cfg.context_length = 1234, 32000, 2048
    for k, v in over.items():
        if k == "recipe" and isinstance(v, str):
            v = RECIPES[v]
        setattr(cfg, k, v)
    return cfg


def write_model(path: str, cfg: SynthCfg) -> str:
    if host().fiber_synth_write_gguf(path.encode(), C.byref(cfg)) != 0:
        raise RuntimeError(f"failed to write {path}")
    return path


def quantize_rows(ggml_type: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.shape
    nbytes = rows * cols // int(host().ggml_block_size(ggml_type)) * int(host().ggml_type_size(ggml_type))
    out = np.empty(nbytes, np.uint8)
    if host().fiber_quantize_rows(ggml_type, x, out.ctypes.data, rows, cols) != 0:
        raise ValueError("quantize failed")
    return out


def random_blocks(ggml_type: int, rows: int, cols: int, seed: int, d_scale: float = 1e-3,
                  dmin_scale: float = 5e-4) -> np.ndarray:
    out = np.empty(rows * cols // 256 * BLOCK_BYTES[ggml_type], np.uint8)
    if host().fiber_random_blocks(ggml_type, out.ctypes.data, rows, cols, seed, d_scale, dmin_scale) != 0:
        raise ValueError("random_blocks failed")
    return out


def randn(n: int, seed: int, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    host().fiber_randn(out, n, seed, std)
    return out


# ---- host model / tokenizer / sampler ----------------------------------------------

class HostModel:
    """model_open() handle (include/model.h)."""

    def __init__(self, path: str):
        self.path = path
        self.h = host().model_open(path.encode())
        if not self.h:
            raise RuntimeError(f"model_open failed for {path}")
        p = ModelParams()
        host().model_get_params(self.h, C.byref(p))
        self.params = p

    def close(self):
        if self.h:
            host().model_close(self.h)
            self.h = None

    __del__ = close

    @property
    def gguf(self) -> int:
        return host().model_gguf(self.h)


class Tokenizer:
    def __init__(self, model: HostModel):
        self.model = model
        self.h = host().tokenizer_init(model.gguf)
        if not self.h:
            raise RuntimeError("tokenizer_init failed")

    def close(self):
        if self.h:
            host().tokenizer_free(self.h)
            self.h = None

    __del__ = close

    def encode(self, text: str, max_tokens: int = 8192) -> np.ndarray:
        out = np.zeros(max_tokens, np.int32)
        n = host().tokenizer_encode(self.h, text.encode(), out, max_tokens)
        return out[:n].copy()

    def decode(self, tok: int) -> bytes:
        return host().tokenizer_decode(self.h, int(tok))

    @property
    def eos(self) -> int:
        return host().tokenizer_eos(self.h)


def sample(logits: np.ndarray, temperature: float, top_k: int, top_p: float, state: Sampler | None = None):
    logits = np.ascontiguousarray(logits, np.float32)
    if state is None:
        state = Sampler()
        host().sampler_init(C.byref(state), len(logits), temperature, top_k, top_p)
    return host().sampler_sample(C.byref(state), logits), state


from .cuda import *  # noqa: E402,F401,F403  (device API; loads lazily)
