/* oracle.h — CPU restatement of the reference's decode path. TEST INFRASTRUCTURE.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load
 * this library, and only as the checker / the timed CPU reference. The product
 * (libfiber_cuda.so) never calls it and has no CPU fallback.
 *
 * What it restates (file:line in the Fiber-Inference reference):
 *  - dequant_q4k_row_f16, dequant_q6k_row_f16          src/dequant.h:9-58
 *  - Q5_K element decode                               metal/kernels.metal:141-169
 *  - cpu_rmsnorm, cpu_rope, cpu_forward_token, argmax  src/fiber_proof.m:23-154, 245-249
 *  - embedding row lookup                              src/gpu_ffn.m:466-482
 *  - hyperparameters, tensor names, tied classifier    src/model.m:41-136, 144-177
 *  - greedy sampling (first maximum wins)              src/sampler.c:38-46
 * Pinning: dequant, the GGUF reader, sampler and tokenizer are checked against
 * the reference's own C compiled from its sources (oracle/_ref), and the forward
 * against the reference's cpu_forward_token compiled from src/fiber_proof.m with
 * a portable cblas_sgemv stand-in (oracle/ref_shim.c); see tests/test_oracle_pin.py.
 *
 * Numerics: weights are the dequantizer's fp16 values widened to fp32 (Q5_K:
 * the fp32 value the Metal kernel computes); activations, KV and accumulation
 * are fp32 as in cpu_forward_token. Option kv_fp16 rounds K and V to fp16 when
 * they are stored, mirroring the device's fp16 KV cache (disclosed deviation
 * from the reference, off by default). Every dot product uses the same fixed
 * 8-lane accumulation order (orc_dot) as the cblas stand-in of the reference
 * build, so both give bit-identical results.
 */
#ifndef FIBER_ORACLE_H
#define FIBER_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids used here (fixed by the GGUF format) */
#define ORC_F32 0
#define ORC_F16 1
#define ORC_Q4_K 12
#define ORC_Q5_K 13
#define ORC_Q6_K 14

void orc_dequant_q4k_row_f16(const void *data, int row, uint16_t *out, int dim);
void orc_dequant_q6k_row_f16(const void *data, int row, uint16_t *out, int dim);
void orc_dequant_q5k_row_f32(const void *data, int row, float *out, int dim);
/* the fp32 weights the forward multiplies with; returns 0 or -1 (bad type) */
int orc_dequant_row_f32(int type, const void *data, int row, float *out, int dim);
/* embedding row as cpu_forward_token sees it: fp16 values widened to fp32 */
int orc_embed_row(int type, const void *data, int row, float *out, int dim);

/* fixed-order dot product used by every matrix-vector product here */
float orc_dot(const float *a, const float *x, int n);
/* y[r] = W[r,:] . x over dequantized rows; n_threads <= 0 uses all */
int orc_gemv(int type, const void *w, const float *x, float *y, int rows, int dim, int n_threads);

typedef struct orc_model orc_model_t;
typedef struct orc_state orc_state_t;

/* Load a GGUF model and dequantize every matrix to fp32 (like the reference's
 * *_f32 arrays). Returns NULL on error. */
orc_model_t *orc_model_load(const char *path, int n_threads);
void orc_model_free(orc_model_t *m);
/* out: dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, context_length */
void orc_model_dims(const orc_model_t *m, int out[8]);

orc_state_t *orc_state_new(const orc_model_t *m, int max_seq, int kv_fp16, int n_threads);
void orc_state_free(orc_state_t *s);
/* Write K/V of one layer/position directly (pre-filled long-context cache). */
int orc_state_set_kv(orc_state_t *s, int layer, int pos, const float *k, const float *v);
int orc_state_get_kv(const orc_state_t *s, int layer, int pos, float *k, float *v);

/* One token: embed, all layers, classifier -> logits[vocab]. Returns 0 or -1. */
int orc_forward_token(orc_state_t *s, int token, int pos, float *logits);
int orc_argmax(const float *v, int n);
/* Prefill n_prompt tokens at positions start..start+n_prompt-1 (token by token),
 * then n_gen greedy steps; out[0..n_gen) gets the generated ids (out[0] is the
 * argmax after the prompt). last_logits (optional) gets the final step's logits. */
int orc_generate(orc_state_t *s, const int *prompt, int n_prompt, int start, int n_gen, int *out,
                 float *last_logits);

#ifdef __cplusplus
}
#endif
#endif
