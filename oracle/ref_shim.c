/* ref_shim.c — glue that lets the reference's own C run here. TEST INFRASTRUCTURE.
 *
 * oracle/Makefile compiles this file together with the reference's unmodified
 * src/gguf.c, src/sampler.c and src/tokenizer.c, its src/dequant.h, and the
 * functions cpu_rmsnorm / cpu_rope / cpu_forward_token (src/fiber_proof.m:23-154)
 * and argmax (:245-249) cut out of src/fiber_proof.m at build time into
 * oracle/_ref/cpu_forward_extract.c. Output goes to oracle/_ref/libref.so, which
 * is git-ignored; nothing of the reference is committed.
 *
 * What this file adds:
 *  - cblas_sgemv: Accelerate is not available here. The stand-in is a row-major
 *    y = A.x with the same fixed 8-lane accumulation order as the restated
 *    oracle's orc_dot, parallel over rows (each row's order is fixed).
 *  - ref_model_load: builds the reference's fiber_model_t from a GGUF file using
 *    the reference's gguf.c and dequant.h (Q4_K/Q6_K rows to fp16, F16/F32
 *    directly), i.e. the "gguf.c + dequant.h driving the reference forward" path.
 *  - ref_forward_token: embedding row (fp16, as gpu_embed / the proof pipeline
 *    use it) then cpu_forward_token, logits copied out.
 *  - thin exports of the static inline dequantizers.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "dequant.h"
#include "fiber_arch.h"
#include "fiber_model.h"
#include "gguf.h"

enum { CblasRowMajor = 101 };
enum { CblasNoTrans = 111 };

static void cblas_sgemv(int order, int trans, int M, int N, float alpha, const float *A, int lda,
                        const float *x, int incx, float beta, float *y, int incy) {
    (void)order; (void)trans; (void)incx; (void)incy; (void)alpha; (void)beta;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < M; r++) {
        const float *a = A + (size_t)r * lda;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        int j = 0;
        for (; j + 8 <= N; j += 8)
            for (int u = 0; u < 8; u++) acc[u] += a[j + u] * x[j + u];
        for (int u = 0; j < N; j++, u++) acc[u] += a[j] * x[j];
        y[r] = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
    }
}

#include "cpu_forward_extract.c"

void ref_dequant_q4k_row_f16(const void *data, int row, _Float16 *out, int dim) {
    dequant_q4k_row_f16(data, row, out, dim);
}
void ref_dequant_q6k_row_f16(const void *data, int row, _Float16 *out, int dim) {
    dequant_q6k_row_f16(data, row, out, dim);
}
int ref_argmax(const float *v, int n) { return argmax(v, n); }

typedef struct {
    fiber_model_t *fm;
    gguf_file_t *gf;
    int dim, n_layers, heads, kv_heads, hd, ffn, vocab;
} ref_model_t;

static int rows_to_f16(const gguf_file_t *gf, const char *name, int rows, int cols, _Float16 *out) {
    const gguf_tensor_info_t *ti = gguf_find_tensor(gf, name);
    if (!ti || ti->dims[0] != (uint64_t)cols) return -1;
    const void *d = gguf_tensor_data(gf, ti);
    for (int r = 0; r < rows; r++) {
        _Float16 *o = out + (size_t)r * cols;
        switch (ti->type) {
        case GGML_TYPE_Q4_K: dequant_q4k_row_f16(d, r, o, cols); break;
        case GGML_TYPE_Q6_K: dequant_q6k_row_f16(d, r, o, cols); break;
        case GGML_TYPE_F16: memcpy(o, (const _Float16 *)d + (size_t)r * cols, (size_t)cols * 2); break;
        case GGML_TYPE_F32:
            for (int i = 0; i < cols; i++) o[i] = (_Float16)((const float *)d)[(size_t)r * cols + i];
            break;
        default: return -1;
        }
    }
    return 0;
}

static float *rows_to_f32(const gguf_file_t *gf, const char *name, int rows, int cols) {
    const gguf_tensor_info_t *ti = gguf_find_tensor(gf, name);
    if (!ti) return NULL;
    float *out = (float *)malloc((size_t)rows * cols * sizeof(float));
    if (!out) return NULL;
    if (ti->type == GGML_TYPE_F32) {
        memcpy(out, gguf_tensor_data(gf, ti), (size_t)rows * cols * 4);
        return out;
    }
    _Float16 *tmp = (_Float16 *)malloc((size_t)rows * cols * 2);
    if (!tmp || rows_to_f16(gf, name, rows, cols, tmp) != 0) {
        free(tmp);
        free(out);
        return NULL;
    }
    for (size_t i = 0; i < (size_t)rows * cols; i++) out[i] = (float)tmp[i];
    free(tmp);
    return out;
}

void ref_model_free(ref_model_t *rm) {
    if (!rm) return;
    if (rm->fm) {
        for (int l = 0; l < FIBER_LAYERS; l++) {
            free(rm->fm->wq_f32[l]); free(rm->fm->wk_f32[l]); free(rm->fm->wv_f32[l]);
            free(rm->fm->wo_f32[l]); free(rm->fm->w1_f32[l]); free(rm->fm->w2_f32[l]);
            free(rm->fm->w3_f32[l]); free(rm->fm->attn_norm_f32[l]); free(rm->fm->ffn_norm_f32[l]);
        }
        free(rm->fm->embedding);
        free(rm->fm->output);
        free(rm->fm->output_norm);
        free(rm->fm);
    }
    if (rm->gf) gguf_close(rm->gf);
    free(rm);
}

ref_model_t *ref_model_load(const char *path) {
    ref_model_t *rm = (ref_model_t *)calloc(1, sizeof(*rm));
    rm->gf = gguf_open(path);
    if (!rm->gf) {
        free(rm);
        return NULL;
    }
    gguf_file_t *gf = rm->gf;
    rm->dim = (int)gguf_get_u32(gf, "llama.embedding_length", 0);
    rm->n_layers = (int)gguf_get_u32(gf, "llama.block_count", 0);
    rm->heads = (int)gguf_get_u32(gf, "llama.attention.head_count", 0);
    rm->kv_heads = (int)gguf_get_u32(gf, "llama.attention.head_count_kv", (uint32_t)rm->heads);
    rm->ffn = (int)gguf_get_u32(gf, "llama.feed_forward_length", 0);
    const gguf_kv_t *vk = gguf_find_kv(gf, "tokenizer.ggml.tokens");
    rm->vocab = vk ? (int)vk->value.arr.count : 0;
    if (!rm->dim || !rm->heads || rm->n_layers < 1 || rm->n_layers > FIBER_LAYERS || !rm->vocab) {
        ref_model_free(rm);
        return NULL;
    }
    rm->hd = rm->dim / rm->heads;
    int dim = rm->dim, kvd = rm->kv_heads * rm->hd, ffn = rm->ffn;
    fiber_model_t *fm = (fiber_model_t *)calloc(1, sizeof(*fm));
    rm->fm = fm;
    char nm[128];
    int ok = 1;
    for (int l = 0; l < rm->n_layers && ok; l++) {
#define LOAD(field, suffix, rows, cols)                                   \
    snprintf(nm, sizeof(nm), "blk.%d." suffix ".weight", l);              \
    fm->field[l] = rows_to_f32(gf, nm, rows, cols);                       \
    ok = ok && fm->field[l];
        LOAD(attn_norm_f32, "attn_norm", 1, dim)
        LOAD(ffn_norm_f32, "ffn_norm", 1, dim)
        LOAD(wq_f32, "attn_q", dim, dim)
        LOAD(wk_f32, "attn_k", kvd, dim)
        LOAD(wv_f32, "attn_v", kvd, dim)
        LOAD(wo_f32, "attn_output", dim, dim)
        LOAD(w1_f32, "ffn_gate", ffn, dim)
        LOAD(w2_f32, "ffn_down", dim, ffn)
        LOAD(w3_f32, "ffn_up", ffn, dim)
#undef LOAD
    }
    fm->embedding = (_Float16 *)malloc((size_t)rm->vocab * dim * 2);
    fm->output = (_Float16 *)malloc((size_t)rm->vocab * dim * 2);
    fm->output_norm = (_Float16 *)malloc((size_t)dim * 2);
    ok = ok && fm->embedding && fm->output && fm->output_norm;
    ok = ok && rows_to_f16(gf, "token_embd.weight", rm->vocab, dim, fm->embedding) == 0;
    if (ok && gguf_find_tensor(gf, "output.weight"))
        ok = rows_to_f16(gf, "output.weight", rm->vocab, dim, fm->output) == 0;
    else if (ok)
        memcpy(fm->output, fm->embedding, (size_t)rm->vocab * dim * 2);
    ok = ok && rows_to_f16(gf, "output_norm.weight", 1, dim, fm->output_norm) == 0;
    if (!ok) {
        ref_model_free(rm);
        return NULL;
    }
    return rm;
}

void ref_model_dims(const ref_model_t *rm, int out[7]) {
    out[0] = rm->dim; out[1] = rm->n_layers; out[2] = rm->heads; out[3] = rm->kv_heads;
    out[4] = rm->hd; out[5] = rm->ffn; out[6] = rm->vocab;
}

typedef struct {
    float **k, **v;
    int n_layers, max_seq;
} ref_kv_t;

ref_kv_t *ref_kv_new(const ref_model_t *rm, int max_seq) {
    ref_kv_t *kv = (ref_kv_t *)calloc(1, sizeof(*kv));
    kv->n_layers = rm->n_layers;
    kv->max_seq = max_seq;
    kv->k = (float **)calloc((size_t)rm->n_layers, sizeof(float *));
    kv->v = (float **)calloc((size_t)rm->n_layers, sizeof(float *));
    for (int l = 0; l < rm->n_layers; l++) {
        kv->k[l] = (float *)calloc((size_t)max_seq * rm->kv_heads * rm->hd, 4);
        kv->v[l] = (float *)calloc((size_t)max_seq * rm->kv_heads * rm->hd, 4);
    }
    return kv;
}

void ref_kv_free(ref_kv_t *kv) {
    if (!kv) return;
    for (int l = 0; l < kv->n_layers; l++) {
        free(kv->k[l]);
        free(kv->v[l]);
    }
    free(kv->k);
    free(kv->v);
    free(kv);
}

/* Proof pipeline A step (src/fiber_proof.m:304-308): x = fp16 embedding row,
 * then cpu_forward_token. */
int ref_forward_token(ref_model_t *rm, ref_kv_t *kv, int token, int pos, float *logits) {
    if (token < 0 || token >= rm->vocab || pos < 0 || pos >= kv->max_seq) return -1;
    float *x = (float *)malloc((size_t)rm->dim * 4);
    for (int d = 0; d < rm->dim; d++) x[d] = (float)rm->fm->embedding[(size_t)token * rm->dim + d];
    float *lg = cpu_forward_token(x, pos, rm->fm, rm->n_layers, rm->dim, rm->heads, rm->kv_heads,
                                  rm->hd, rm->ffn, rm->vocab, kv->k, kv->v, kv->max_seq);
    memcpy(logits, lg, (size_t)rm->vocab * 4);
    free(lg);
    free(x);
    return 0;
}
