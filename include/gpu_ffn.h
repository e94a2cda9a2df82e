/* gpu_ffn.h — the reference's decode entry points, served by libfiber_cuda.so.
 *
 * Drop-in for src/gpu_ffn.h:9-33 of the reference (Metal): same names, argument
 * meaning and error behaviour (NULL / no-op on failure, message on stderr and
 * in fiber_last_error()). The Metal command buffer becomes one CUDA graph per
 * decode step on the context's stream; weights are the GGUF data section copied
 * unchanged into HBM at gpu_init.
 *
 *   gpu_init             src/gpu_ffn.h:11   device 0, max_seq = model context length
 *   gpu_free             src/gpu_ffn.h:12
 *   gpu_embed            src/gpu_ffn.h:15   records the token; the embedding row is
 *                                           dequantized on the device in the next forward
 *   gpu_forward_token    src/gpu_ffn.h:18   all layers + classifier; blocks; returns ms
 *   gpu_get_logits       src/gpu_ffn.h:22   copies the fp32 logits to a host buffer owned
 *                                           by ctx (valid until the next call)
 *   gpu_forward_classifier src/gpu_ffn.h:33 final RMSNorm + lm_head on the current state
 *   gpu_get_device       src/gpu_ffn.h:44   CUDA ordinal instead of id<MTLDevice>
 * The ANE-prefill helpers (gpu_forward_ffn_layer, gpu_init_ffn_batch,
 * gpu_forward_ffn_batch, gpu_get_buf_x) have no counterpart: that prefill path
 * is Apple-only and is replaced by fiber_prefill (fiber_cuda.h).
 */
#ifndef FIBER_GPU_FFN_H
#define FIBER_GPU_FFN_H

#include "kv_cache.h"
#include "model.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct gpu_context gpu_context_t;

gpu_context_t *gpu_init(const model_t *m);
void gpu_free(gpu_context_t *ctx);
void gpu_embed(gpu_context_t *ctx, const model_t *m, int token_id);
double gpu_forward_token(gpu_context_t *ctx, const model_t *m, kv_cache_t *kv, int pos);
const float *gpu_get_logits(gpu_context_t *ctx);
void gpu_forward_classifier(gpu_context_t *ctx, const model_t *m);
int gpu_get_device(gpu_context_t *ctx);

#ifdef __cplusplus
}
#endif
#endif
