"""ctypes wrappers for the CPU checker libraries. TEST INFRASTRUCTURE.

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of bench.py may
import this module. It loads

* ``oracle/liboracle.so`` -- the restated reference decode path (oracle.c),
* ``oracle/_ref/libref.so`` -- the reference's own C (gguf.c, sampler.c,
  tokenizer.c, dequant.h and cpu_forward_token from src/fiber_proof.m) built by
  oracle/Makefile from the reference sources; optional, absent when the
  reference tree was not available at build time.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_ORACLE = os.path.join(HERE, "liboracle.so")
_REF = os.path.join(HERE, "_ref", "libref.so")

F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
U16P = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
I32P = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")

_lib = None
_ref = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_ORACLE):
            raise RuntimeError(f"{_ORACLE} missing: run `make -C oracle`")
        L = C.CDLL(_ORACLE)
        L.orc_dequant_q4k_row_f16.argtypes = [C.c_void_p, C.c_int, U16P, C.c_int]
        L.orc_dequant_q6k_row_f16.argtypes = [C.c_void_p, C.c_int, U16P, C.c_int]
        L.orc_dequant_q5k_row_f32.argtypes = [C.c_void_p, C.c_int, F32P, C.c_int]
        L.orc_dequant_row_f32.argtypes = [C.c_int, C.c_void_p, C.c_int, F32P, C.c_int]
        L.orc_embed_row.argtypes = [C.c_int, C.c_void_p, C.c_int, F32P, C.c_int]
        L.orc_gemv.argtypes = [C.c_int, C.c_void_p, F32P, F32P, C.c_int, C.c_int, C.c_int]
        L.orc_model_load.restype = C.c_void_p
        L.orc_model_load.argtypes = [C.c_char_p, C.c_int]
        L.orc_model_free.argtypes = [C.c_void_p]
        L.orc_model_dims.argtypes = [C.c_void_p, I32P]
        L.orc_state_new.restype = C.c_void_p
        L.orc_state_new.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int]
        L.orc_state_free.argtypes = [C.c_void_p]
        L.orc_state_set_kv.argtypes = [C.c_void_p, C.c_int, C.c_int, F32P, F32P]
        L.orc_state_get_kv.argtypes = [C.c_void_p, C.c_int, C.c_int, F32P, F32P]
        L.orc_forward_token.argtypes = [C.c_void_p, C.c_int, C.c_int, F32P]
        L.orc_argmax.argtypes = [F32P, C.c_int]
        L.orc_generate.argtypes = [C.c_void_p, I32P, C.c_int, C.c_int, C.c_int, I32P, C.c_void_p]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(_REF)


def ref() -> C.CDLL:
    """The reference's own C, compiled from its sources (oracle/_ref)."""
    global _ref
    if _ref is None:
        if not ref_available():
            raise RuntimeError(f"{_REF} missing: the reference tree was not present at build time")
        R = C.CDLL(_REF)
        R.ref_dequant_q4k_row_f16.argtypes = [C.c_void_p, C.c_int, U16P, C.c_int]
        R.ref_dequant_q6k_row_f16.argtypes = [C.c_void_p, C.c_int, U16P, C.c_int]
        R.ref_argmax.argtypes = [F32P, C.c_int]
        R.ref_model_load.restype = C.c_void_p
        R.ref_model_load.argtypes = [C.c_char_p]
        R.ref_model_free.argtypes = [C.c_void_p]
        R.ref_model_dims.argtypes = [C.c_void_p, I32P]
        R.ref_kv_new.restype = C.c_void_p
        R.ref_kv_new.argtypes = [C.c_void_p, C.c_int]
        R.ref_kv_free.argtypes = [C.c_void_p]
        R.ref_forward_token.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, F32P]
        R.gguf_open.restype = C.c_void_p
        R.gguf_open.argtypes = [C.c_char_p]
        R.gguf_close.argtypes = [C.c_void_p]
        R.gguf_get_u32.restype = C.c_uint32
        R.gguf_get_u32.argtypes = [C.c_void_p, C.c_char_p, C.c_uint32]
        R.gguf_get_f32.restype = C.c_float
        R.gguf_get_f32.argtypes = [C.c_void_p, C.c_char_p, C.c_float]
        R.gguf_get_str.restype = C.c_char_p
        R.gguf_get_str.argtypes = [C.c_void_p, C.c_char_p]
        R.gguf_find_tensor.restype = C.c_void_p
        R.gguf_find_tensor.argtypes = [C.c_void_p, C.c_char_p]
        R.gguf_tensor_data.restype = C.c_void_p
        R.gguf_tensor_data.argtypes = [C.c_void_p, C.c_void_p]
        R.tokenizer_init.restype = C.c_void_p
        R.tokenizer_init.argtypes = [C.c_void_p]
        R.tokenizer_free.argtypes = [C.c_void_p]
        R.tokenizer_encode.argtypes = [C.c_void_p, C.c_char_p, I32P, C.c_int]
        R.tokenizer_decode.restype = C.c_char_p
        R.tokenizer_decode.argtypes = [C.c_void_p, C.c_int]
        R.sampler_init.argtypes = [C.c_void_p, C.c_int, C.c_float, C.c_int, C.c_float]
        R.sampler_sample.argtypes = [C.c_void_p, F32P]
        _ref = R
    return _ref


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def dequant_f16(ggml_type: int, blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """fp16 dequant of Q4_K/Q6_K rows (src/dequant.h restated)."""
    out = np.empty((rows, cols), np.uint16)
    fn = {12: lib().orc_dequant_q4k_row_f16, 14: lib().orc_dequant_q6k_row_f16}[ggml_type]
    for r in range(rows):
        fn(_ptr(blocks), r, out[r], cols)
    return out.view(np.float16)


def dequant_f32(ggml_type: int, blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
    out = np.empty((rows, cols), np.float32)
    for r in range(rows):
        if lib().orc_dequant_row_f32(ggml_type, _ptr(blocks), r, out[r], cols) != 0:
            raise ValueError(f"unsupported type {ggml_type}")
    return out


def ref_dequant_f16(ggml_type: int, blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
    out = np.empty((rows, cols), np.uint16)
    fn = {12: ref().ref_dequant_q4k_row_f16, 14: ref().ref_dequant_q6k_row_f16}[ggml_type]
    for r in range(rows):
        fn(_ptr(blocks), r, out[r], cols)
    return out.view(np.float16)


def gemv(ggml_type: int, blocks: np.ndarray, x: np.ndarray, rows: int, cols: int, threads: int = 0) -> np.ndarray:
    y = np.empty(rows, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    if lib().orc_gemv(ggml_type, _ptr(blocks), x, y, rows, cols, threads) != 0:
        raise ValueError("orc_gemv failed")
    return y


class Model:
    """Restated forward over a GGUF file (weights dequantized to fp32 at load)."""

    def __init__(self, path: str, threads: int = 0):
        self.h = lib().orc_model_load(path.encode(), threads)
        if not self.h:
            raise RuntimeError(f"oracle could not load {path}")
        d = np.zeros(8, np.int32)
        lib().orc_model_dims(self.h, d)
        (self.dim, self.n_layers, self.n_heads, self.n_kv_heads, self.head_dim, self.ffn_dim,
         self.vocab, self.context_length) = (int(v) for v in d)
        self.threads = threads

    def close(self):
        if self.h:
            lib().orc_model_free(self.h)
            self.h = None

    __del__ = close

    def state(self, max_seq: int, kv_fp16: bool = False) -> "State":
        return State(self, max_seq, kv_fp16)


class State:
    def __init__(self, model: Model, max_seq: int, kv_fp16: bool):
        self.model = model
        self.h = lib().orc_state_new(model.h, max_seq, int(kv_fp16), model.threads)
        if not self.h:
            raise MemoryError("orc_state_new failed")

    def close(self):
        if self.h:
            lib().orc_state_free(self.h)
            self.h = None

    __del__ = close

    def forward(self, token: int, pos: int) -> np.ndarray:
        lg = np.empty(self.model.vocab, np.float32)
        if lib().orc_forward_token(self.h, int(token), int(pos), lg) != 0:
            raise ValueError("orc_forward_token failed")
        return lg

    def set_kv(self, layer: int, pos: int, k: np.ndarray, v: np.ndarray):
        lib().orc_state_set_kv(self.h, layer, pos, np.ascontiguousarray(k, np.float32),
                               np.ascontiguousarray(v, np.float32))

    def generate(self, prompt, n_gen: int, start: int = 0, want_logits: bool = False):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(n_gen + 1, np.int32)
        lg = np.empty(self.model.vocab, np.float32) if want_logits else None
        rc = lib().orc_generate(self.h, p, len(p), start, n_gen, out,
                                lg.ctypes.data if lg is not None else None)
        if rc != 0:
            raise ValueError("orc_generate failed")
        return (out, lg) if want_logits else out


class RefModel:
    """The reference's cpu_forward_token over a fiber_model_t built by gguf.c + dequant.h."""

    def __init__(self, path: str):
        self.h = ref().ref_model_load(path.encode())
        if not self.h:
            raise RuntimeError(f"reference loader could not load {path}")
        d = np.zeros(7, np.int32)
        ref().ref_model_dims(self.h, d)
        self.dim, self.n_layers, self.n_heads, self.n_kv_heads, self.head_dim, self.ffn_dim, self.vocab = (
            int(v) for v in d)

    def close(self):
        if self.h:
            ref().ref_model_free(self.h)
            self.h = None

    __del__ = close

    def kv(self, max_seq: int):
        return RefKV(self, max_seq)


class RefKV:
    def __init__(self, model: RefModel, max_seq: int):
        self.model = model
        self.h = ref().ref_kv_new(model.h, max_seq)

    def close(self):
        if self.h:
            ref().ref_kv_free(self.h)
            self.h = None

    __del__ = close

    def forward(self, token: int, pos: int) -> np.ndarray:
        lg = np.empty(self.model.vocab, np.float32)
        if ref().ref_forward_token(self.model.h, self.h, int(token), int(pos), lg) != 0:
            raise ValueError("ref_forward_token failed")
        return lg
