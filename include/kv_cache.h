/* kv_cache.h — HBM-resident paged fp16 KV cache (device side).
 *
 * Replaces the reference's per-layer Metal buffers (src/kv_cache.h:12-32,
 * src/kv_cache.m:8-38; layout [n_kv_heads][max_seq][head_dim] fp16, zeroed).
 * Same constructor arguments and meaning, with the Metal device handle replaced
 * by a CUDA device ordinal; returns NULL on failure (reason in
 * fiber_last_error()).
 *
 * Layout: a pool of pages; page p holds `page_size` consecutive positions of
 * every layer and KV head, K and V in separate pools:
 *     k_pool[p][layer][kv_head][page_size][head_dim]   (fp16, same for v_pool)
 * Sequence slot s maps logical page j to physical page page_table[s][j]. Pages
 * are assigned to slots at construction (slot s owns pages
 * s*max_pages_per_seq ... +max_pages_per_seq-1), so a captured decode graph
 * never needs host work when the sequence grows. The pool is zero-filled.
 */
#ifndef FIBER_KV_CACHE_H
#define FIBER_KV_CACHE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct kv_cache {
    int n_layers;
    int n_kv_heads;
    int head_dim;
    int max_seq;
    int device;
    int max_batch;         /* sequence slots */
    int page_size;         /* positions per page */
    int max_pages_per_seq; /* ceil(max_seq / page_size) */
    int n_pages;           /* pages in the pool */
    uint16_t *k_pool;      /* device, fp16 bits */
    uint16_t *v_pool;      /* device, fp16 bits */
    int32_t *page_table;   /* device, [max_batch][max_pages_per_seq] */
} kv_cache_t;

/* One sequence slot (src/kv_cache.h:28-29 with `id<MTLDevice>` -> device ordinal). */
kv_cache_t *kv_cache_init(int device, int n_layers, int n_kv_heads, int head_dim, int max_seq);
/* max_batch sequence slots; page_size must be a power of two in [16, 256]. */
kv_cache_t *kv_cache_init_paged(int device, int n_layers, int n_kv_heads, int head_dim, int max_seq,
                                int max_batch, int page_size);
void kv_cache_free(kv_cache_t *kv);

/* Host <-> cache copies of n_pos positions starting at pos for one slot and
 * layer; host buffers are fp32 [n_pos][n_kv_heads*head_dim], rounded to fp16
 * on write. Used to pre-fill long contexts and by tests. Return 0 or an error. */
int kv_cache_write(kv_cache_t *kv, int slot, int layer, int pos, int n_pos, const float *k,
                   const float *v);
int kv_cache_read(const kv_cache_t *kv, int slot, int layer, int pos, int n_pos, float *k, float *v);

#ifdef __cplusplus
}
#endif
#endif
