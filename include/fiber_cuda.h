/* fiber_cuda.h — extern "C" API of libfiber_cuda.so beyond the reference's names.
 *
 * Conventions: plain pointers and sizes; `stream` is a cudaStream_t passed as
 * void* (NULL = the default stream); "d_" pointers are device memory, "h_"
 * pointers host memory. Every function returns FIBER_OK (0) or a negative
 * FIBER_E* code and never exits; fiber_last_error() describes the last failure
 * on the calling thread. One host thread per context; all device work of a
 * context runs on its own stream.
 *
 * Numerics (identical on every path): K-quant weights are decoded exactly as
 * the reference's CPU dequantizer does it (src/dequant.h:9-58: fp32 products,
 * one rounding to fp16) -- Q5_K as the reference's Metal kernel does
 * (metal/kernels.metal:141-169, fp32) -- activations and accumulation are fp32,
 * the KV cache is fp16.
 */
#ifndef FIBER_CUDA_H
#define FIBER_CUDA_H

#include <stddef.h>
#include <stdint.h>

#include "gpu_ffn.h"
#include "kv_cache.h"
#include "model.h"

#ifdef __cplusplus
extern "C" {
#endif

#define FIBER_OK 0
#define FIBER_EARG (-1)         /* bad argument / unsupported shape or type */
#define FIBER_ECUDA (-2)        /* CUDA runtime error */
#define FIBER_ENOMEM (-3)       /* device or pinned allocation failed */
#define FIBER_EUNSUPPORTED (-4) /* model feature the kernels do not cover */
#define FIBER_ETIMEOUT (-5)     /* a bounded device-side wait gave up */

const char *fiber_last_error(void);
int fiber_device_count(void);

/* ---- model-level decode (greedy loop of src/main.m:553-586) --------------------- */

/* Sequences one batched decode step can carry. */
#define FIBER_MAX_BATCH 64

typedef struct gpu_context fiber_ctx_t;

/* Upload the GGUF data section unchanged to `device`, resolve per-layer device
 * pointers once, allocate activations and scratch for up to max_seq positions.
 * (gpu_init equivalent, src/gpu_ffn.m:141-204.) max_batch (1 .. FIBER_MAX_BATCH)
 * bounds the sequences of one batched step; above 1 the model must suit the
 * tensor-core layer pass (Q4_K/Q5_K/Q6_K/F16 matrices, GQA group <= 8), else NULL
 * with FIBER_EUNSUPPORTED. */
fiber_ctx_t *fiber_cuda_init(const model_t *m, int device, int max_batch, int max_seq);
void fiber_cuda_free(fiber_ctx_t *ctx);

/* One decode step for `batch` sequences (1 .. max_batch): embeds tokens[i] at
 * position pos[i] (host arrays), runs all layers and the classifier, then, if
 * non-NULL, copies the fp32 logits [batch][vocab] and the greedy argmax
 * (lowest index on ties, src/sampler.c:38-46) to host memory. Blocks until done.
 * batch 1 runs the GEMV step on KV slot 0; batch > 1 runs sequence i on KV slot i
 * through the tensor-core layer pass (the reference decodes one sequence only). */
int fiber_forward_token(fiber_ctx_t *ctx, kv_cache_t *kv, const int32_t *tokens,
                        const int32_t *pos, int batch, float *logits_or_null,
                        int32_t *argmax_or_null);

/* Prompt of n tokens at positions start_pos.. of KV slot 0 (src/main.m:561-563
 * steps it token by token; here batched, see fiber_set_prefill_mode);
 * *argmax_out (optional) gets the greedy token after the last one. */
int fiber_prefill(fiber_ctx_t *ctx, kv_cache_t *kv, const int32_t *tokens, int n, int start_pos,
                  int32_t *argmax_out);
/* The same for KV slot `slot` (batched layer pass only), to start a batch of
 * sequences. No counterpart in the reference (one sequence only). */
int fiber_prefill_slot(fiber_ctx_t *ctx, kv_cache_t *kv, int slot, const int32_t *tokens, int n,
                       int start_pos, int32_t *argmax_out);

/* Device-resident greedy loop: n_steps decode steps starting with first_token at
 * start_pos; each step's argmax feeds the next on the device (one graph replay
 * per step, no host round trip). h_tokens_out[i] = argmax of step i. If ms_out
 * is non-NULL it receives the device time of the n_steps replays (CUDA events
 * on the context stream). */
int fiber_decode_greedy(fiber_ctx_t *ctx, kv_cache_t *kv, int32_t first_token, int start_pos,
                        int n_steps, int32_t *h_tokens_out, float *ms_out);
/* The device-resident greedy loop for `batch` sequences (1 .. max_batch): sequence
 * i starts with first_tokens[i] at start_pos[i] in KV slot i; one captured graph
 * of the batched step per step. h_tokens_out[step * batch + i] = sequence i's
 * argmax at that step. ms_out as for fiber_decode_greedy. No counterpart in the
 * reference (one sequence only). */
int fiber_decode_greedy_batch(fiber_ctx_t *ctx, kv_cache_t *kv, const int32_t *first_tokens,
                              const int32_t *start_pos, int batch, int n_steps, int32_t *h_tokens_out,
                              float *ms_out);

/* Sampling on the device with the reference sampler's procedure (src/sampler.c:48-112):
 * temperature <= 0 (or < 1e-6) is the greedy argmax; otherwise logits * (1/T), the
 * top_k (top_k <= 0: all) largest sorted descending (equal values in index order; with
 * k = vocab the candidates stay in index order, as the reference leaves them unsorted),
 * softmax, nucleus cut at top_p, one xorshift64* draw. Sums are taken in the reference's
 * order; exp is CUDA's expf, so a draw within an ulp of a boundary can differ from the
 * host sampler. Limits: top_k <= 1024 when below the vocabulary; vocab <= 49152 when
 * top_k covers it (else FIBER_EUNSUPPORTED; the host sampler has no limit).
 *
 * Kernel level: one token per row of d_logits ([rows][ld] fp32) into d_out; d_rng holds
 * one xorshift64* state per row (the reference starts at 42), advanced by the draw.
 * Enqueued on `stream`, no synchronization. No counterpart in the reference (host only). */
int fiber_sample(const float *d_logits, int rows, int vocab, int ld, float temperature, int top_k,
                 float top_p, unsigned long long *d_rng, int32_t *d_out, void *stream);

/* Device-resident sampling decode loop: as fiber_decode_greedy, with each step's token
 * drawn by the device sampler above; *rng_state (the reference sampler's state, 42 at
 * sampler_init) is used and advanced. temperature <= 0 is fiber_decode_greedy. */
int fiber_decode_sample(fiber_ctx_t *ctx, kv_cache_t *kv, int32_t first_token, int start_pos,
                        int n_steps, float temperature, int top_k, float top_p,
                        unsigned long long *rng_state, int32_t *h_tokens_out, float *ms_out);

/* How a decode step runs. mode 2 (default when the model fits): one cooperative
 * dataflow kernel per step -- every SM streams its weight tiles of all phases through
 * a shared-memory ring, and each phase waits only for the words of its input (tagged
 * with the launch), not for a grid barrier. mode 0: the same kernel shape with a grid
 * barrier between phases (persistent kernel). mode 1: one kernel per phase
 * (2 + 5 * n_layers launches, PDL-chained). All give the same tokens; mode 1 also
 * serves models the one-kernel steps do not cover (Q5_K weights). Returns
 * FIBER_EUNSUPPORTED for mode 0 or 2 then. */
int fiber_set_decode_mode(fiber_ctx_t *ctx, int mode);

/* Tokens per pass of the batched prefill through the layer stack. */
#define FIBER_PREFILL_CHUNK 512

/* Prefill path of fiber_prefill: 0 (default) = batched, the prompt in chunks of
 * FIBER_PREFILL_CHUNK tokens through tensor-core dequant-GEMMs (tcgen05) with causal attention over the
 * cache, when every matrix is Q4_K / Q5_K / Q6_K / F16 and the context is not sharded;
 * 1 = one decode step per token. Both fill the same KV cache and return the first
 * generated token. */
int fiber_set_prefill_mode(fiber_ctx_t *ctx, int mode);
int fiber_get_decode_mode(fiber_ctx_t *ctx);

/* Number of kernels one decode step launches (all of them this library's own). */
int fiber_step_launches(fiber_ctx_t *ctx);

/* Bytes of the shared-memory weight / KV ring the current one-kernel decode mode
 * streams through (0 in mode 1). No counterpart in the reference: the ring is how
 * the one-kernel steps stage weights; tests use it to check a requested ring size
 * (FIBER_PK_RING_KB / FIBER_FL_RING_KB) is the one in use. */
int fiber_step_ring_bytes(fiber_ctx_t *ctx);

/* ---- tensor parallelism (one process per GPU) ------------------------------------ */

#define FIBER_TP_ID_BYTES 128

/* This rank's share of the model: query heads [head0, head0 + heads), KV heads
 * [kv_head0, kv_head0 + kv_heads), FFN blocks of 256 [ffn_block0, + ffn_blocks). */
typedef struct {
    int rank, world;
    int heads, head0;
    int kv_heads, kv_head0;
    int ffn_block0, ffn_blocks;
} fiber_tp_plan_t;

/* Pure host computation of the split (no GPU): heads and KV heads evenly, FFN
 * super-blocks as evenly as whole blocks allow; FIBER_EUNSUPPORTED when the model
 * does not split over `world` (Wo shards must be whole super-blocks). */
int fiber_tp_plan(const model_params_t *p, int rank, int world, fiber_tp_plan_t *out);

/* Communicator id for fiber_cuda_init_tp, made on rank 0 and passed to every rank
 * by the caller (FIBER_TP_ID_BYTES bytes). */
int fiber_tp_unique_id(uint8_t out[FIBER_TP_ID_BYTES]);

/* Tensor-parallel context for rank `rank` of `world` on CUDA device `device`
 * (replaces the reference's single-device gpu_init for the sharded 7B/13B
 * decode): Wq/Wk/Wv and W_gate/W_up split by rows (heads, FFN blocks), Wo and
 * W_down split along their input dimension at super-block granularity; the
 * embedding, norms and lm_head are replicated. Every decode step all-reduces
 * (NCCL, sum) the dim-vector after Wo and after W_down inside the step graph, so
 * every rank holds the same residual stream and the same greedy token. Must be
 * called by all ranks together. The KV cache holds this rank's KV heads
 * (fiber_tp_info). Steps run the dataflow kernel with the exchange fused into it
 * (decode mode 2) where the model fits it, else the per-phase kernels (mode 1). */
fiber_ctx_t *fiber_cuda_init_tp(const model_t *m, int device, int rank, int world,
                                const uint8_t nccl_id[FIBER_TP_ID_BYTES], int max_seq);
int fiber_tp_info(fiber_ctx_t *ctx, fiber_tp_plan_t *out);

/* The all-reduce a sharded step uses after Wo and after W_down: 0 none (world 1),
 * 1 NCCL (ncclAllReduce), 2 the one-shot peer-memory all-reduce (each rank stores its
 * partial into every rank's slot over NVLink, each 8-byte word holding a value and the
 * call's epoch; readers poll the words with a bounded wait, and every rank sums the
 * partials in rank order: identical results on all ranks).
 * 2 is the default for up to 8 ranks; FIBER_TP_ALLREDUCE=nccl in the environment at
 * fiber_cuda_init_tp selects NCCL. 3: the exchange is fused into the dataflow step
 * (decode mode 2, the default where the model fits it): the Wo and W_down epilogues
 * store each rank's partial sums into every rank's exchange buffer over NVLink (tagged
 * words, CUDA IPC mappings), and the next phase's staging adds the ranks' partials to the
 * residual in rank order, so no separate collective runs in the step; modes 1 and 0 use
 * the collective above. In mode 2, calls that want only the token (fiber_decode_greedy,
 * fiber_forward_token without a logits buffer) also split the lm_head tiles across the
 * ranks, which exchange their best (logit, row) keys: every rank must make the same call
 * with the same logits choice (a rank left waiting reports error 4 after 2 s). */
int fiber_tp_collective(fiber_ctx_t *ctx);

/* Raise the sequences one batched step can carry (as fiber_cuda_init's max_batch; the
 * tensor-parallel constructor starts at 1). Only before the first batched call. */
int fiber_set_max_batch(fiber_ctx_t *ctx, int max_batch);

/* Timeline of one persistent decode step (mode 0): runs the step for `token` at
 * `pos` and fills out[n_phases][n_ctas][10] (uint64) with, per phase and CTA:
 * 0 globaltimer ns when the phase's grid barrier released the CTA, 1 SM cycles
 * at that barrier, 2 cycles staging the input vector, 3 cycles in the tile loop
 * (attention: the units), 4 of those waiting for weight tiles to land, 5 cycles
 * to the arrive, 6 globaltimer ns when the producer issued the phase's last
 * tile, 7 producer cycles spent waiting for ring space in the phase; attention
 * phases: 8 cycles until q/k/v are staged, 9 cycles of the page loop.
 * `cap` is the number of uint64 values `out` holds. */
int fiber_trace_step(fiber_ctx_t *ctx, kv_cache_t *kv, int token, int pos, uint64_t *out, size_t cap,
                     int *n_phases, int *n_ctas);

/* Device time of one kernel kind of the decode step, measured the way it runs in
 * the step: a CUDA graph of its n_layers per-layer launches (lm_head and embed:
 * n_layers repeats) is replayed `reps` times between CUDA events on the context
 * stream, with the position set to `pos` (attention reads pos+1 KV rows and
 * rewrites row pos). kind: 0 QKV, 1 attention, 2 Wo, 3 gate/up+SwiGLU, 4 down,
 * 5 lm_head+argmax, 6 embedding. Outputs: average microseconds per launch and
 * algorithmic bytes per launch (weights + KV + vectors). Overwrites the hidden
 * state: call it between decode calls. */
int fiber_time_kernel(fiber_ctx_t *ctx, kv_cache_t *kv, int kind, int pos, int reps,
                      double *us_per_launch, double *bytes_per_launch);

/* ---- kernel-level entry points (device pointers) -------------------------------- */

/* y[r] = sum_k W[r,k] * x[k] for rows x cols weights in GGUF layout
 * (ggml_type Q4_K / Q5_K / Q6_K / F16; cols % 256 == 0), fp32 x and y. */
int fiber_gemv(int ggml_type, const void *d_w, const float *d_x, float *d_y, int rows, int cols,
               void *stream);
/* Tensor-core dequant-GEMM (the prefill building block; tcgen05, fp32 accumulation):
 * y[t][out_off + r] = (accumulate ? y[t][out_off + r] : 0) + sum_k W[r,k] * xn[t][k]
 * for t < ntok, with xn = x * rrms[t] * nw[k] when d_nw is given (RMSNorm folded
 * in; rrms taken as 1 when d_rrms is null) and xn = x otherwise. W: Q4_K / Q5_K /
 * Q6_K / F16 super-blocks, cols % 256 == 0; x: [ntok][ldx] fp32; y: [ntok][ldy] fp32.
 * The weights are decoded exactly as the GEMV does (Q5_K's fp32 values as fp16 hi +
 * lo parts); xn is split into fp16 hi + lo parts
 * and must stay below 65504 in magnitude (else FIBER_EARG). d_w, d_x and d_nw must
 * be 16-byte aligned and ldx a multiple of 4; Q6_K rows are read through
 * 16-byte-aligned spans, so 14 bytes after the last block must be readable.
 * Allocates a packed copy of x for the call and synchronizes the stream. */
int fiber_gemm(int ggml_type, const void *d_w, int rows, int cols, const float *d_x, int ntok, int ldx,
               const float *d_rrms, const float *d_nw, float *d_y, int ldy, int out_off, int accumulate,
               void *stream);
/* Decoded weights: fp16 bits for Q4_K/Q6_K/F16, fp32 for Q5_K, [rows][cols]. */
int fiber_dequant(int ggml_type, const void *d_w, void *d_out, int rows, int cols, void *stream);
/* Same GEMV with host buffers: copies x in and y out around the launch on the
 * given stream and synchronizes (d_w stays resident). */
int fiber_gemv_host(int ggml_type, const void *d_w, const float *h_x, float *h_y, int rows,
                    int cols, float *d_x_scratch, float *d_y_scratch, void *stream);

/* ---- allocation-free greedy lm_head step ----------------------------------------
 * No counterpart in the reference. Same result as fiber_gemv followed by a greedy
 * argmax (the first index of the maximum; index 0 when every value is NaN): d_y = W.x and
 * *d_argmax, both device memory, enqueued on `stream`. It exists for callers that
 * cannot allocate device memory where they run the step: a host application
 * whose own pool owns all device memory and forbids further cudaMalloc, or a
 * latency-critical loop that cannot accept cudaMalloc's implicit device
 * synchronization. The kernel's cross-CTA scratch (one value/index pair per CTA
 * and a merge ticket, about 128 KB) is a fixed static device array that every GPU
 * loading this library holds until the process exits; the call makes no
 * cudaMalloc, cudaFree or other allocating call. The first call on a device looks
 * up the array's device address with that device current, so make that first
 * call before any stream capture. Every call shares the array and it keeps the
 * last call's contents; the ticket is cleared at the start of each call. Calls
 * that overlap on the GPU (e.g. on two streams of one device) race on it.
 * rows > FIBER_NOALLOC_MAX_ROWS returns FIBER_EARG. */
#define FIBER_NOALLOC_MAX_ROWS 262144
int fiber_gemv_argmax_noalloc(int ggml_type, const void *d_w, const float *d_x, float *d_y,
                              int32_t *d_argmax, int rows, int cols, void *stream);

#ifdef __cplusplus
}
#endif
#endif
