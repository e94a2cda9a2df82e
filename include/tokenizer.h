/* tokenizer.h — SentencePiece-style BPE over the GGUF vocabulary (host side).
 *
 * Same entry points and results as the reference tokenizer (src/tokenizer.h:11-24):
 * vocab and scores from tokenizer.ggml.tokens / tokenizer.ggml.scores, "▁"
 * prefix and space mapping, UTF-8 character split with <0xNN> byte fallback,
 * highest-score-leftmost pair merging, "▁" → ' ' on decode. The merge loop here
 * is a heap over a linked list (O(n log n)) instead of the reference's O(n²)
 * rescan; ties resolve the same way (highest score, then leftmost pair), so the
 * token sequences are identical.
 */
#ifndef FIBER_TOKENIZER_H
#define FIBER_TOKENIZER_H

#include "gguf.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct tokenizer tokenizer_t;

tokenizer_t *tokenizer_init(const gguf_file_t *gf);
void tokenizer_free(tokenizer_t *tok);
/* Returns the number of ids written (at most max_tokens). */
int tokenizer_encode(const tokenizer_t *tok, const char *text, int *tokens, int max_tokens);
/* Returned string is valid until the next decode call on this thread. */
const char *tokenizer_decode(const tokenizer_t *tok, int token_id);
int tokenizer_bos(const tokenizer_t *tok);
int tokenizer_eos(const tokenizer_t *tok);
int tokenizer_vocab_size(const tokenizer_t *tok);

#ifdef __cplusplus
}
#endif
#endif
