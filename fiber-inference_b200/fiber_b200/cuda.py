"""ctypes bindings of libfiber_cuda.so (include/fiber_cuda.h, gpu_ffn.h, kv_cache.h).

Device buffers handed to the kernel-level calls are plain device addresses
(e.g. ``torch.Tensor.data_ptr()``); the model-level calls own their memory.
Every call raises ``FiberError`` with ``fiber_last_error()`` on a non-zero status.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import CUDA_SO, ModelParams  # noqa: F401

__all__ = ["FiberError", "cuda_lib", "cuda_available", "gemv", "gemv_host", "gemv_argmax_noalloc", "dequant", "Context", "KVCache",
           "device_count", "TPPlan", "TP_ID_BYTES", "tp_plan", "tp_unique_id", "gemm", "PREFILL_CHUNK",
           "sample_device"]

PREFILL_CHUNK = 512  # FIBER_PREFILL_CHUNK: tokens per pass of the batched prefill

F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
I32P = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")

EXPORTED = [
    "fiber_last_error", "fiber_device_count", "fiber_cuda_init", "fiber_cuda_free", "fiber_forward_token",
    "fiber_prefill", "fiber_decode_greedy", "fiber_step_launches", "fiber_set_decode_mode",
    "fiber_get_decode_mode", "fiber_trace_step", "fiber_time_kernel", "fiber_gemv", "fiber_tp_plan",
    "fiber_tp_unique_id", "fiber_cuda_init_tp", "fiber_tp_info", "fiber_gemm", "fiber_set_prefill_mode",
    "fiber_dequant", "fiber_gemv_host", "gpu_init", "gpu_free", "gpu_embed", "gpu_forward_token",
    "gpu_get_logits", "gpu_forward_classifier", "gpu_get_device", "kv_cache_init", "kv_cache_init_paged",
    "kv_cache_free", "kv_cache_write", "kv_cache_read", "fiber_gemv_argmax_noalloc", "fiber_prefill_slot",
    "fiber_decode_greedy_batch", "fiber_sample", "fiber_decode_sample", "fiber_tp_collective", "fiber_set_max_batch",
    "fiber_step_ring_bytes",
]


class FiberError(RuntimeError):
    pass


class TPPlan(C.Structure):
    _fields_ = [("rank", C.c_int), ("world", C.c_int), ("heads", C.c_int), ("head0", C.c_int),
                ("kv_heads", C.c_int), ("kv_head0", C.c_int), ("ffn_block0", C.c_int), ("ffn_blocks", C.c_int)]


TP_ID_BYTES = 128


class KVCacheT(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("max_seq", C.c_int),
                ("device", C.c_int), ("max_batch", C.c_int), ("page_size", C.c_int),
                ("max_pages_per_seq", C.c_int), ("n_pages", C.c_int), ("k_pool", C.c_void_p),
                ("v_pool", C.c_void_p), ("page_table", C.c_void_p)]


_cuda = None


def cuda_lib() -> C.CDLL:
    """Load libfiber_cuda.so (no GPU needed to load it)."""
    global _cuda
    if _cuda is None:
        if not os.path.exists(CUDA_SO):
            raise FiberError(f"{CUDA_SO} missing: run `make -C fiber-inference_b200 cuda`")
        L = C.CDLL(CUDA_SO)
        L.fiber_last_error.restype = C.c_char_p
        L.fiber_cuda_init.restype = C.c_void_p
        L.fiber_cuda_init.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int]
        L.fiber_cuda_free.argtypes = [C.c_void_p]
        L.fiber_forward_token.argtypes = [C.c_void_p, C.c_void_p, I32P, I32P, C.c_int, C.c_void_p, C.c_void_p]
        L.fiber_prefill.argtypes = [C.c_void_p, C.c_void_p, I32P, C.c_int, C.c_int, C.c_void_p]
        L.fiber_prefill_slot.argtypes = [C.c_void_p, C.c_void_p, C.c_int, I32P, C.c_int, C.c_int, C.c_void_p]
        L.fiber_decode_greedy_batch.argtypes = [C.c_void_p, C.c_void_p, I32P, I32P, C.c_int, C.c_int, C.c_void_p,
                                                C.c_void_p]
        L.fiber_sample.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int, C.c_float, C.c_void_p,
                                   C.c_void_p, C.c_void_p]
        L.fiber_decode_sample.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_int, C.c_int, C.c_float, C.c_int,
                                          C.c_float, C.POINTER(C.c_ulonglong), C.c_void_p, C.c_void_p]
        L.fiber_decode_greedy.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_int, C.c_int, C.c_void_p,
                                          C.c_void_p]
        L.fiber_step_launches.argtypes = [C.c_void_p]
        L.fiber_step_ring_bytes.argtypes = [C.c_void_p]
        L.fiber_set_decode_mode.argtypes = [C.c_void_p, C.c_int]
        L.fiber_get_decode_mode.argtypes = [C.c_void_p]
        L.fiber_tp_plan.argtypes = [C.c_void_p, C.c_int, C.c_int, C.POINTER(TPPlan)]
        L.fiber_tp_unique_id.argtypes = [C.c_void_p]
        L.fiber_cuda_init_tp.restype = C.c_void_p
        L.fiber_cuda_init_tp.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int]
        L.fiber_tp_info.argtypes = [C.c_void_p, C.POINTER(TPPlan)]
        L.fiber_tp_collective.argtypes = [C.c_void_p]
        L.fiber_set_max_batch.argtypes = [C.c_void_p, C.c_int]
        L.fiber_set_prefill_mode.argtypes = [C.c_void_p, C.c_int]
        L.fiber_gemm.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                 C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]
        L.fiber_trace_step.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t,
                                       C.POINTER(C.c_int), C.POINTER(C.c_int)]
        L.fiber_time_kernel.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_double),
                                        C.POINTER(C.c_double)]
        L.fiber_gemv.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.fiber_gemv_host.argtypes = [C.c_int, C.c_void_p, F32P, F32P, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                      C.c_void_p]
        L.fiber_dequant.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.fiber_gemv_argmax_noalloc.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                                C.c_int, C.c_void_p]
        L.kv_cache_init.restype = C.POINTER(KVCacheT)
        L.kv_cache_init.argtypes = [C.c_int] * 5
        L.kv_cache_init_paged.restype = C.POINTER(KVCacheT)
        L.kv_cache_init_paged.argtypes = [C.c_int] * 7
        L.kv_cache_free.argtypes = [C.c_void_p]
        L.kv_cache_write.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, F32P, F32P]
        L.kv_cache_read.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, F32P, F32P]
        L.gpu_init.restype = C.c_void_p
        L.gpu_init.argtypes = [C.c_void_p]
        L.gpu_free.argtypes = [C.c_void_p]
        L.gpu_embed.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
        L.gpu_forward_token.restype = C.c_double
        L.gpu_forward_token.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
        L.gpu_get_logits.restype = C.POINTER(C.c_float)
        L.gpu_get_logits.argtypes = [C.c_void_p]
        L.gpu_forward_classifier.argtypes = [C.c_void_p, C.c_void_p]
        L.gpu_get_device.argtypes = [C.c_void_p]
        _cuda = L
    return _cuda


def _check(rc: int, what: str):
    if rc != 0:
        raise FiberError(f"{what}: {cuda_lib().fiber_last_error().decode()} (status {rc})")


def device_count() -> int:
    return int(cuda_lib().fiber_device_count())


def cuda_available() -> bool:
    try:
        return device_count() > 0
    except (OSError, FiberError):
        return False


def _stream_ptr(stream) -> int | None:
    if stream is None:
        return None
    return int(getattr(stream, "cuda_stream", stream))


def gemv(ggml_type: int, d_w: int, d_x: int, d_y: int, rows: int, cols: int, stream=None):
    _check(cuda_lib().fiber_gemv(ggml_type, d_w, d_x, d_y, rows, cols, _stream_ptr(stream)), "fiber_gemv")


def gemv_host(ggml_type: int, d_w: int, x: np.ndarray, y: np.ndarray, rows: int, cols: int, d_x: int, d_y: int,
              stream=None):
    _check(cuda_lib().fiber_gemv_host(ggml_type, d_w, x, y, rows, cols, d_x, d_y, _stream_ptr(stream)),
           "fiber_gemv_host")


def gemv_argmax_noalloc(ggml_type: int, d_w: int, d_x: int, d_y: int, d_argmax: int, rows: int, cols: int,
                        stream=None):
    """Greedy lm_head step whose scratch is a static device array (no allocation)."""
    _check(cuda_lib().fiber_gemv_argmax_noalloc(ggml_type, d_w, d_x, d_y, d_argmax, rows, cols, _stream_ptr(stream)),
           "fiber_gemv_argmax_noalloc")


def gemm(ggml_type: int, d_w: int, rows: int, cols: int, d_x: int, ntok: int, d_y: int, ldy: int,
         out_off: int = 0, d_rrms: int | None = None, d_nw: int | None = None, accumulate: bool = False,
         ldx: int | None = None, stream=None):
    """fiber_gemm: y[t][out_off + r] (+)= sum_k W[r,k] * xn[t][k] on the tensor cores."""
    _check(cuda_lib().fiber_gemm(ggml_type, d_w, rows, cols, d_x, ntok, ldx or cols, d_rrms, d_nw, d_y, ldy, out_off,
                                 1 if accumulate else 0, _stream_ptr(stream)), "fiber_gemm")


def sample_device(d_logits: int, rows: int, vocab: int, ld: int, temperature: float, top_k: int, top_p: float,
                  d_rng: int, d_out: int, stream=None):
    """fiber_sample: one token per logits row on the device (the reference sampler's procedure)."""
    _check(cuda_lib().fiber_sample(d_logits, rows, vocab, ld, temperature, top_k, top_p, d_rng, d_out,
                                   _stream_ptr(stream)), "fiber_sample")


def dequant(ggml_type: int, d_w: int, d_out: int, rows: int, cols: int, stream=None):
    _check(cuda_lib().fiber_dequant(ggml_type, d_w, d_out, rows, cols, _stream_ptr(stream)), "fiber_dequant")


class KVCache:
    def __init__(self, device: int, n_layers: int, n_kv_heads: int, head_dim: int, max_seq: int, max_batch: int = 1):
        if max_batch == 1:
            self.ptr = cuda_lib().kv_cache_init(device, n_layers, n_kv_heads, head_dim, max_seq)
        else:
            self.ptr = cuda_lib().kv_cache_init_paged(device, n_layers, n_kv_heads, head_dim, max_seq, max_batch, 64)
        if not self.ptr:
            raise FiberError(f"kv_cache_init: {cuda_lib().fiber_last_error().decode()}")
        self.s = self.ptr.contents

    @property
    def addr(self) -> int:
        return C.cast(self.ptr, C.c_void_p).value

    def close(self):
        if self.ptr:
            cuda_lib().kv_cache_free(self.addr)
            self.ptr = None

    __del__ = close

    def write(self, layer: int, pos: int, k: np.ndarray, v: np.ndarray, slot: int = 0):
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        n = k.shape[0] if k.ndim == 2 else 1
        _check(cuda_lib().kv_cache_write(self.addr, slot, layer, pos, n, k, v), "kv_cache_write")

    def read(self, layer: int, pos: int, n: int, slot: int = 0):
        kvd = self.s.n_kv_heads * self.s.head_dim
        k = np.empty((n, kvd), np.float32)
        v = np.empty((n, kvd), np.float32)
        _check(cuda_lib().kv_cache_read(self.addr, slot, layer, pos, n, k, v), "kv_cache_read")
        return k, v


def tp_plan(params, rank: int, world: int) -> TPPlan:
    """fiber_tp_plan: this rank's heads / KV heads / FFN blocks (host only, no GPU)."""
    out = TPPlan()
    _check(cuda_lib().fiber_tp_plan(C.byref(params), rank, world, C.byref(out)), "fiber_tp_plan")
    return out


def tp_unique_id() -> bytes:
    buf = (C.c_uint8 * TP_ID_BYTES)()
    _check(cuda_lib().fiber_tp_unique_id(buf), "fiber_tp_unique_id")
    return bytes(buf)


class Context:
    """fiber_cuda_init over a host model (fiber_b200.HostModel); with tp=(rank, world,
    id bytes) a tensor-parallel context (fiber_cuda_init_tp)."""

    def __init__(self, host_model, device: int = 0, max_seq: int = 0, tp=None, max_batch: int = 1):
        self.model = host_model
        self.p = host_model.params
        self.max_batch = max_batch
        if tp is None:
            self.h = cuda_lib().fiber_cuda_init(host_model.h, device, max_batch, max_seq)
        else:
            rank, world, nid = tp
            idbuf = (C.c_uint8 * TP_ID_BYTES).from_buffer_copy(nid)
            self.h = cuda_lib().fiber_cuda_init_tp(host_model.h, device, rank, world, idbuf, max_seq)
        if not self.h:
            raise FiberError(f"fiber_cuda_init: {cuda_lib().fiber_last_error().decode()}")
        if tp is not None and max_batch > 1:
            _check(cuda_lib().fiber_set_max_batch(self.h, int(max_batch)), "fiber_set_max_batch")
        self.device = device
        self.max_seq = max_seq or self.p.context_length
        self.plan = TPPlan()
        _check(cuda_lib().fiber_tp_info(self.h, C.byref(self.plan)), "fiber_tp_info")

    def close(self):
        if self.h:
            cuda_lib().fiber_cuda_free(self.h)
            self.h = None

    __del__ = close

    def kv(self, max_seq: int | None = None, max_batch: int = 1) -> KVCache:
        return KVCache(self.device, self.p.n_layers, self.plan.kv_heads, self.p.head_dim, max_seq or self.max_seq,
                       max_batch)

    def forward(self, kv: KVCache, token: int, pos: int, want_logits: bool = True):
        lg = np.empty(self.p.vocab_size, np.float32) if want_logits else None
        am = np.zeros(1, np.int32)
        _check(cuda_lib().fiber_forward_token(self.h, kv.addr, np.array([token], np.int32),
                                              np.array([pos], np.int32), 1,
                                              lg.ctypes.data if lg is not None else None, am.ctypes.data),
               "fiber_forward_token")
        return int(am[0]), lg

    def prefill(self, kv: KVCache, tokens, start_pos: int = 0, slot: int | None = None) -> int:
        """fiber_prefill (slot None: KV slot 0) or fiber_prefill_slot; returns the next greedy token."""
        t = np.ascontiguousarray(tokens, np.int32)
        am = np.zeros(1, np.int32)
        if slot is None:
            _check(cuda_lib().fiber_prefill(self.h, kv.addr, t, len(t), start_pos, am.ctypes.data), "fiber_prefill")
        else:
            _check(cuda_lib().fiber_prefill_slot(self.h, kv.addr, int(slot), t, len(t), start_pos, am.ctypes.data),
                   "fiber_prefill_slot")
        return int(am[0])

    def forward_batch(self, kv: KVCache, tokens, pos, want_logits: bool = True):
        """One decode step of len(tokens) sequences (sequence i on KV slot i):
        (argmax [batch], logits [batch][vocab] or None)."""
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(pos, np.int32)
        lg = np.empty((len(t), self.p.vocab_size), np.float32) if want_logits else None
        am = np.zeros(len(t), np.int32)
        _check(cuda_lib().fiber_forward_token(self.h, kv.addr, t, p, len(t),
                                              lg.ctypes.data if lg is not None else None, am.ctypes.data),
               "fiber_forward_token")
        return am, lg

    def decode_greedy_batch(self, kv: KVCache, first_tokens, start_pos, n_steps: int):
        """fiber_decode_greedy_batch: (tokens [n_steps][batch], device ms)."""
        t = np.ascontiguousarray(first_tokens, np.int32)
        p = np.ascontiguousarray(start_pos, np.int32)
        out = np.zeros((n_steps, len(t)), np.int32)
        ms = C.c_float(0.0)
        _check(cuda_lib().fiber_decode_greedy_batch(self.h, kv.addr, t, p, len(t), int(n_steps), out.ctypes.data,
                                                    C.addressof(ms)), "fiber_decode_greedy_batch")
        return out, float(ms.value)

    def decode_greedy(self, kv: KVCache, first_token: int, start_pos: int, n_steps: int):
        out = np.zeros(n_steps, np.int32)
        ms = C.c_float(0.0)
        _check(cuda_lib().fiber_decode_greedy(self.h, kv.addr, int(first_token), int(start_pos), int(n_steps),
                                              out.ctypes.data, C.addressof(ms)), "fiber_decode_greedy")
        return out, float(ms.value)

    def decode_sample(self, kv: KVCache, first_token: int, start_pos: int, n_steps: int, temperature: float,
                      top_k: int, top_p: float, rng_state: int = 42):
        """fiber_decode_sample: (tokens, device ms, advanced random state)."""
        out = np.zeros(n_steps, np.int32)
        ms = C.c_float(0.0)
        st = C.c_ulonglong(rng_state)
        _check(cuda_lib().fiber_decode_sample(self.h, kv.addr, int(first_token), int(start_pos), int(n_steps),
                                              float(temperature), int(top_k), float(top_p), C.byref(st),
                                              out.ctypes.data, C.addressof(ms)), "fiber_decode_sample")
        return out, float(ms.value), int(st.value)

    def set_mode(self, mode: int):
        """0: grid-barrier persistent one-kernel step; 1: one kernel per phase;
        2: dataflow one-kernel step (tagged-word hand-off between phases)."""
        _check(cuda_lib().fiber_set_decode_mode(self.h, int(mode)), "fiber_set_decode_mode")

    def set_prefill_mode(self, mode: int):
        """0: batched tensor-core prefill when supported (default); 1: one decode step per token."""
        _check(cuda_lib().fiber_set_prefill_mode(self.h, int(mode)), "fiber_set_prefill_mode")

    @property
    def tp_collective(self) -> int:
        """fiber_tp_collective: 0 none, 1 NCCL, 2 one-shot peer all-reduce, 3 fused into the
        dataflow step (peer stores in the residual phases)."""
        return int(cuda_lib().fiber_tp_collective(self.h))

    @property
    def mode(self) -> int:
        return int(cuda_lib().fiber_get_decode_mode(self.h))

    @property
    def ring_bytes(self) -> int:
        """Bytes of the shared-memory ring of the current one-kernel decode mode (0 in mode 1)."""
        return int(cuda_lib().fiber_step_ring_bytes(self.h))

    def step_launches(self) -> int:
        n = cuda_lib().fiber_step_launches(self.h)
        if n < 0:
            _check(n, "fiber_step_launches")
        return int(n)

    TRACE_FIELDS = ["t_release_ns", "cyc_barrier", "cyc_stage", "cyc_tiles", "cyc_wait_tiles", "cyc_arrive",
                    "t_producer_done_ns", "cyc_producer_wait", "cyc_attn_qkv", "cyc_attn_pages"]

    FLOW_TRACE_FIELDS = ["t_start_ns", "cyc_poll", "cyc_stage", "cyc_phase", "cyc_wait_ring", "t_end_ns",
                         "t_producer_done_ns", "cyc_producer_wait", "cyc_attn_pages", "cyc_attn_merge",
                         "t_inputs_staged_ns", "t_last_epilogue_ns", "cyc_attn_acquire_or_dots",
                         "cyc_attn_qk_or_publish", "cyc_attn_softmax_or_n_epilogues", "cyc_attn_pv_or_n_tiles"]

    def trace_step(self, kv: KVCache, token: int, pos: int, max_phases: int = 4096, max_ctas: int = 1024):
        """Per-phase, per-CTA timeline of one one-kernel step: uint64 array
        [n_phases, n_ctas, n_fields] with the fields of TRACE_FIELDS (mode 0) or
        FLOW_TRACE_FIELDS (mode 2)."""
        nf = len(self.FLOW_TRACE_FIELDS if self.mode == 2 else self.TRACE_FIELDS)
        buf = np.zeros(max_phases * max_ctas * nf, np.uint64)
        nph, nct = C.c_int(), C.c_int()
        _check(cuda_lib().fiber_trace_step(self.h, kv.addr, int(token), int(pos), buf.ctypes.data, buf.size,
                                           C.byref(nph), C.byref(nct)), "fiber_trace_step")
        return buf[: nph.value * nct.value * nf].reshape(nph.value, nct.value, nf)

    KINDS = ["qkv", "attention", "wo", "gate_up", "down", "lm_head", "embed"]

    def time_kernel(self, kv: KVCache, kind: int, pos: int, reps: int = 20):
        """(microseconds per launch, algorithmic bytes per launch) of one kernel kind."""
        us, b = C.c_double(), C.c_double()
        _check(cuda_lib().fiber_time_kernel(self.h, kv.addr, kind, pos, reps, C.byref(us), C.byref(b)),
               "fiber_time_kernel")
        return us.value, b.value
