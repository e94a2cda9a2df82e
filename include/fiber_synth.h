/* fiber_synth.h — seeded synthetic GGUF models and K-quant blocks (host side).
 *
 * No counterpart in the reference, which ships no quantizer and no test models:
 * these build the random-init models the decode path is measured and checked on
 * (Llama-family GGUF v3 files with F16, Q4_K_M or Q5_K_M weights, a synthetic
 * SentencePiece vocabulary and the usual `llama.*` metadata) and the raw random
 * super-blocks of the single-GEMV workload.
 *
 * Quantizers are written from the block layouts the dequantizers read
 * (Q4_K/Q6_K: src/dequant.h:9-58; Q5_K: metal/kernels.metal:141-169 of the
 * reference). They aim at a small reconstruction error, nothing more: parity is
 * checked on whatever blocks they produce.
 */
#ifndef FIBER_SYNTH_H
#define FIBER_SYNTH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    FIBER_RECIPE_F16 = 0,    /* all matrices F16, norms F32 */
    FIBER_RECIPE_Q4_K_M = 1, /* Q4_K; Q6_K attn_v/ffn_down on even layers and output */
    FIBER_RECIPE_Q5_K_M = 2, /* Q5_K; Q6_K attn_v/ffn_down on all layers and output */
    FIBER_RECIPE_Q4_K = 3,   /* Q4_K everywhere (output too) */
    FIBER_RECIPE_Q6_K = 4,   /* Q6_K everywhere */
    FIBER_RECIPE_Q5_K = 5,   /* Q5_K everywhere */
};

typedef struct {
    uint32_t dim, n_layers, n_heads, n_kv_heads, ffn_dim, vocab, context_length;
    float rope_base, eps;
    int recipe;
    float weight_std; /* N(0, weight_std) for every matrix and the embedding */
    float norm_value; /* value of every RMSNorm weight */
    uint64_t seed;
    int tied;      /* 1: no output.weight (classifier = token_embd) */
    int n_threads; /* <= 0: all available */
    float ffn_norm_value; /* > 0: value of the ffn_norm weights instead of norm_value (a
                           * large value grows the residual stream layer by layer while the
                           * attention inputs stay normalised: activation-range tests) */
} fiber_synth_cfg_t;

/* Fill cfg with a named preset: "stories" (768/12/12/12/2048, F16, tied),
 * "tinyllama" (2048/22/32/4/5632, Q4_K_M), "tinyllama-q5" (Q5_K_M),
 * "llama7b" (4096/32/32/32/11008, Q4_K_M). Returns 0 on success. */
int fiber_synth_preset(const char *name, fiber_synth_cfg_t *cfg);

/* Write a complete model; returns 0 on success, -1 on error (message on stderr). */
int fiber_synth_write_gguf(const char *path, const fiber_synth_cfg_t *cfg);

/* Roles of the norm tensors in a fill callback (matrices use the recipe roles below). */
enum { FIBER_ROLE_OUTPUT_NORM = -1, FIBER_ROLE_ATTN_NORM = -2, FIBER_ROLE_FFN_NORM = -3 };

/* fp32 values of one tensor, rows x cols row-major ([out][in] for matrices; rows = 1 for
 * norms); role as fiber_synth_recipe_type's (0 wq .. 6 w3, 7 token_embd, 8 output) or a
 * FIBER_ROLE_*_NORM. Returns 0, or non-zero to abort the write. */
typedef int (*fiber_tensor_fill_fn)(void *user, int role, uint32_t layer, size_t rows, size_t cols, float *vals);

/* The same file layout and metadata as fiber_synth_write_gguf, with every tensor's values
 * from fill (quantized to cfg->recipe's types; cfg->seed only names the vocabulary). */
int fiber_write_gguf_from(const char *path, const fiber_synth_cfg_t *cfg, fiber_tensor_fill_fn fill, void *user);

/* Type the recipe gives tensor `role` of layer `layer` (role: 0 wq,1 wk,2 wv,
 * 3 wo,4 w1 gate,5 w2 down,6 w3 up,7 token_embd,8 output; layer ignored for 7/8). */
int fiber_synth_recipe_type(int recipe, int role, uint32_t layer, uint32_t n_layers);

/* Quantize `rows` rows of `cols` floats (cols % 256 == 0) into GGUF blocks of
 * `ggml_type` (Q4_K, Q5_K, Q6_K, F16, F32). dst needs rows*cols/256*block_bytes. */
int fiber_quantize_rows(int ggml_type, const float *src, void *dst, size_t rows, size_t cols);

/* Random super-blocks straight from the block fields: quants uniform over their
 * range, 6-bit scales/mins uniform 0..63 (Q6_K: int8 scales uniform -128..127),
 * d = fp16(|N(0,1)|*d_scale), dmin = fp16(|N(0,1)|*dmin_scale). */
int fiber_random_blocks(int ggml_type, void *dst, size_t rows, size_t cols, uint64_t seed,
                        float d_scale, float dmin_scale);

/* Seeded N(mean 0, std) floats (same generator the model writer uses). */
void fiber_randn(float *dst, size_t n, uint64_t seed, float std);

#ifdef __cplusplus
}
#endif
#endif
