/* model.h — Llama-family GGUF model handle (host side).
 *
 * Mirrors the reference's model API (src/model.h:11-105): model_params_t with the
 * same fields and GGUF keys, layer_weights_t with the same per-tensor pointers /
 * types / sizes, model_open / model_close / model_layer_weights /
 * model_print_info. Pointers point into the mmapped GGUF file.
 *
 * Differences, all additive:
 *  - model_open resolves every layer's tensors ONCE (model_t.layers); the
 *    reference re-ran 9 linear name scans per layer per token
 *    (src/model.m:17-29, 144-177). model_layer_weights copies from that table.
 *  - tensor byte offsets relative to the GGUF data section (data_off fields) are
 *    kept, because the CUDA side uploads the data section unchanged and
 *    addresses weights by offset.
 *  - the ANE-only FP16 attention copies (src/model.h:51-56, 70-76) and the
 *    madvise prefetch/evict helpers are not part of this build: weights live in
 *    HBM.
 */
#ifndef FIBER_MODEL_H
#define FIBER_MODEL_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#include "gguf.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    uint32_t n_layers;
    uint32_t n_heads;
    uint32_t n_kv_heads;
    uint32_t dim;      /* embedding dimension */
    uint32_t head_dim; /* dim / n_heads */
    uint32_t ffn_dim;
    uint32_t vocab_size;
    uint32_t context_length;
    float rope_freq_base;
    float rms_norm_eps;
    const char *arch; /* general.architecture, valid until model_close */
} model_params_t;

typedef struct {
    const void *attn_norm;
    const void *wq;
    const void *wk;
    const void *wv;
    const void *wo;
    const void *ffn_norm;
    const void *w1; /* ffn_gate */
    const void *w2; /* ffn_down */
    const void *w3; /* ffn_up */
    ggml_type_t attn_norm_type;
    ggml_type_t wq_type;
    ggml_type_t wk_type;
    ggml_type_t wv_type;
    ggml_type_t wo_type;
    ggml_type_t ffn_norm_type;
    ggml_type_t w1_type;
    ggml_type_t w2_type;
    ggml_type_t w3_type;
    size_t wq_size, wk_size, wv_size, wo_size;
    size_t w1_size, w2_size, w3_size;
} layer_weights_t;

/* Offsets of a layer's tensors relative to the GGUF data section. */
typedef struct {
    uint64_t attn_norm, wq, wk, wv, wo, ffn_norm, w1, w2, w3;
} layer_offsets_t;

typedef struct {
    gguf_file_t *gf;
    model_params_t params;
    const void *token_embd;
    const void *output_norm;
    const void *output; /* classifier; falls back to token_embd (tied) */
    ggml_type_t token_embd_type;
    ggml_type_t output_norm_type;
    ggml_type_t output_type;
    /* resolved once by model_open */
    layer_weights_t *layers;    /* [n_layers] */
    layer_offsets_t *layer_off; /* [n_layers] */
    uint64_t token_embd_off, output_norm_off, output_off;
} model_t;

/* Returns NULL (and prints why) if the file is not a usable Llama-family GGUF. */
model_t *model_open(const char *path);
void model_close(model_t *m);
bool model_layer_weights(const model_t *m, uint32_t layer_idx, layer_weights_t *lw);
void model_print_info(const model_t *m);
size_t model_get_rss(void);

/* Accessors for FFI callers that do not mirror the struct layouts. */
void model_get_params(const model_t *m, model_params_t *out);
const gguf_file_t *model_gguf(const model_t *m);

#ifdef __cplusplus
}
#endif
#endif /* FIBER_MODEL_H */
