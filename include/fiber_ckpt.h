/* fiber_ckpt.h — karpathy / llama2.c checkpoints (".bin") as Llama GGUF models.
 *
 * The reference reads these files with fiber_model_load_karpathy
 * (src/fiber_ckpt.m:125-259) into its own fiber_model_t for the ANE path. Here the
 * same file format feeds the decode path: the checkpoint is rewritten once as a
 * Llama GGUF (matrices and embedding rounded to fp16, as the reference's
 * f32_to_f16 does; RMSNorm weights kept in fp32) and opened with model_open, so
 * every entry point of this library (fiber_cuda_init, prefill, batched decode,
 * the CLI) runs it unchanged.
 *
 * File layout (llama2.c): 7 int32 (dim, hidden_dim, n_layers, n_heads, n_kv_heads,
 * vocab_size, seq_len; n_kv_heads 0 = n_heads; vocab_size < 0 = separate
 * classifier), then fp32 arrays: token_embedding [vocab][dim]; rms_att [L][dim];
 * wq [L][dim][dim]; wk, wv [L][kv_dim][dim]; wo [L][dim][dim]; rms_ffn [L][dim];
 * w1 [L][hidden][dim]; w2 [L][dim][hidden]; w3 [L][hidden][dim]; rms_final [dim];
 * freq_cis_real, freq_cis_imag [seq_len][head_dim / 2] each; wcls [vocab][dim]
 * when the classifier is separate.
 *
 * Differences from the reference loader, both in files it cannot read correctly:
 *  - it skips 2 * seq_len * head_dim floats of freq_cis before a separate
 *    classifier (src/fiber_ckpt.m:245); the tables hold seq_len * head_dim floats
 *    in all, which is what is skipped here;
 *  - it keeps at most 24 layers (FIBER_LAYERS) without skipping the rest of each
 *    array; here every layer is read.
 * Like the reference, q and k are used as stored (no row permutation), and RoPE
 * is the half-split form of the decode path. The vocabulary written to the GGUF is
 * the synthetic one of fiber_synth.h (token ids in and out; the text tokenizer of a
 * karpathy model, tokenizer.bin, is a separate file this library does not read).
 */
#ifndef FIBER_CKPT_H
#define FIBER_CKPT_H

#include <stdint.h>

#include "model.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int32_t dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len;
    int32_t shared_classifier; /* 1: the classifier is the embedding (vocab_size > 0 in the file) */
} fiber_karpathy_config_t;

/* Header of a checkpoint, n_kv_heads and vocab_size normalised. 0 or -1. */
int fiber_karpathy_config(const char *bin_path, fiber_karpathy_config_t *out);

/* Rewrite the checkpoint as a Llama GGUF at gguf_path (dim and hidden_dim must be
 * multiples of 256, the decode path's block size). 0 or -1 (reason on stderr). */
int fiber_karpathy_to_gguf(const char *bin_path, const char *gguf_path);

/* fiber_model_load_karpathy equivalent: convert to gguf_path, then model_open it.
 * NULL on failure. */
model_t *model_open_karpathy(const char *bin_path, const char *gguf_path);

#ifdef __cplusplus
}
#endif
#endif /* FIBER_CKPT_H */
