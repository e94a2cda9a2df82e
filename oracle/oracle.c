/* oracle.c — CPU restatement of the reference decode path (test infrastructure).
 * See oracle.h for what is restated and how it is pinned. Compile with
 * -ffp-contract=off so no multiply-add is fused and results do not depend on
 * the host CPU.
 */
#include "oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static float h2f(uint16_t u) {
    _Float16 h;
    memcpy(&h, &u, 2);
    return (float)h;
}

static uint16_t f2h(float f) {
    _Float16 h = (_Float16)f;
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}

/* 6-bit scale j and min j from the packed 12-byte field
 * (metal/kernels.metal:10-19; src/dequant.h:19-23). */
static void scale_min_k4(int j, const uint8_t *sc, int *s, int *m) {
    if (j < 4) {
        *s = sc[j] & 63;
        *m = sc[j + 4] & 63;
    } else {
        *s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
        *m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
}

/* src/dequant.h:9-31: out[64j+l] = fp16(d*s1*(q&15) - dmin*m1),
 * out[64j+l+32] = fp16(d*s2*(q>>4) - dmin*m2), q = qs[32j+l]. */
void orc_dequant_q4k_row_f16(const void *data, int row, uint16_t *out, int dim) {
    int nb = dim / 256;
    const uint8_t *rb = (const uint8_t *)data + (size_t)row * nb * 144;
    for (int b = 0; b < nb; b++) {
        const uint8_t *blk = rb + (size_t)b * 144;
        uint16_t dh, mh;
        memcpy(&dh, blk, 2);
        memcpy(&mh, blk + 2, 2);
        float d = h2f(dh), dmin = h2f(mh);
        const uint8_t *sc = blk + 4, *qs = blk + 16;
        for (int j = 0; j < 4; j++) {
            int s1, m1, s2, m2;
            scale_min_k4(2 * j, sc, &s1, &m1);
            scale_min_k4(2 * j + 1, sc, &s2, &m2);
            for (int l = 0; l < 32; l++) {
                uint8_t q = qs[32 * j + l];
                out[256 * b + 64 * j + l] = f2h(d * (float)s1 * (float)(q & 0xF) - dmin * (float)m1);
                out[256 * b + 64 * j + l + 32] = f2h(d * (float)s2 * (float)(q >> 4) - dmin * (float)m2);
            }
        }
    }
}

/* src/dequant.h:34-58: per 128-element half, ql[64] qh[32] int8 scales[8]. */
void orc_dequant_q6k_row_f16(const void *data, int row, uint16_t *out, int dim) {
    int nb = dim / 256;
    const uint8_t *rb = (const uint8_t *)data + (size_t)row * nb * 210;
    for (int b = 0; b < nb; b++) {
        const uint8_t *blk = rb + (size_t)b * 210;
        const uint8_t *ql = blk, *qh = blk + 128;
        const int8_t *sc = (const int8_t *)(blk + 192);
        uint16_t dh;
        memcpy(&dh, blk + 208, 2);
        float d = h2f(dh);
        for (int half = 0; half < 2; half++) {
            uint16_t *o = out + 256 * b + 128 * half;
            for (int l = 0; l < 32; l++) {
                int is = l / 16;
                int q1 = (int)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                o[l] = f2h(d * (float)sc[is + 0] * (float)q1);
                o[l + 32] = f2h(d * (float)sc[is + 2] * (float)q2);
                o[l + 64] = f2h(d * (float)sc[is + 4] * (float)q3);
                o[l + 96] = f2h(d * (float)sc[is + 6] * (float)q4);
            }
            ql += 64;
            qh += 32;
            sc += 8;
        }
    }
}

/* metal/kernels.metal:141-169: d@0 dmin@2 scales@4 qh[32]@16 qs[128]@48;
 * element e: g=e/64, s=(e/32)&1, w=e%32, nib from qs[32g+w], high bit
 * (qh[w] >> (2g+s)) & 1, value d*sc*(nib+16*hi) - dmin*m in fp32. */
void orc_dequant_q5k_row_f32(const void *data, int row, float *out, int dim) {
    int nb = dim / 256;
    const uint8_t *rb = (const uint8_t *)data + (size_t)row * nb * 176;
    for (int b = 0; b < nb; b++) {
        const uint8_t *blk = rb + (size_t)b * 176;
        uint16_t dh, mh;
        memcpy(&dh, blk, 2);
        memcpy(&mh, blk + 2, 2);
        float d = h2f(dh), dmin = h2f(mh);
        const uint8_t *sc = blk + 4, *qh = blk + 16, *qs = blk + 48;
        for (int e = 0; e < 256; e++) {
            int g = e / 64, s = (e / 32) & 1, w = e % 32;
            int sv, mv;
            scale_min_k4(2 * g + s, sc, &sv, &mv);
            float nib = (float)(s == 0 ? (qs[32 * g + w] & 0xF) : (qs[32 * g + w] >> 4));
            float hi = (float)((qh[w] >> (2 * g + s)) & 1);
            out[256 * b + e] = d * (float)sv * (nib + hi * 16.0f) - dmin * (float)mv;
        }
    }
}

int orc_dequant_row_f32(int type, const void *data, int row, float *out, int dim) {
    uint16_t *tmp;
    switch (type) {
    case ORC_F32: memcpy(out, (const float *)data + (size_t)row * dim, (size_t)dim * 4); return 0;
    case ORC_F16: {
        const uint16_t *p = (const uint16_t *)data + (size_t)row * dim;
        for (int i = 0; i < dim; i++) out[i] = h2f(p[i]);
        return 0;
    }
    case ORC_Q5_K: orc_dequant_q5k_row_f32(data, row, out, dim); return 0;
    case ORC_Q4_K:
    case ORC_Q6_K:
        tmp = (uint16_t *)malloc((size_t)dim * 2);
        if (!tmp) return -1;
        if (type == ORC_Q4_K)
            orc_dequant_q4k_row_f16(data, row, tmp, dim);
        else
            orc_dequant_q6k_row_f16(data, row, tmp, dim);
        for (int i = 0; i < dim; i++) out[i] = h2f(tmp[i]);
        free(tmp);
        return 0;
    default: return -1;
    }
}

/* gpu_embed (src/gpu_ffn.m:466-482) writes the row into the fp16 buf_x and
 * cpu_forward_token reads the fp16 embedding: the row is always fp16-rounded.
 * Q5_K, which the reference leaves as zeros, uses its fp32 decode rounded the
 * same way. */
int orc_embed_row(int type, const void *data, int row, float *out, int dim) {
    if (orc_dequant_row_f32(type, data, row, out, dim) != 0) return -1;
    for (int i = 0; i < dim; i++) out[i] = h2f(f2h(out[i]));
    return 0;
}

float orc_dot(const float *a, const float *x, int n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int j = 0;
    for (; j + 8 <= n; j += 8)
        for (int u = 0; u < 8; u++) acc[u] += a[j + u] * x[j + u];
    for (int u = 0; j < n; j++, u++) acc[u] += a[j] * x[j];
    return ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
}

static void set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int orc_gemv(int type, const void *w, const float *x, float *y, int rows, int dim, int n_threads) {
    set_threads(n_threads);
    int bad = 0;
#pragma omp parallel
    {
        float *row = (float *)malloc((size_t)dim * 4);
#pragma omp for schedule(static)
        for (int r = 0; r < rows; r++) {
            if (!row || orc_dequant_row_f32(type, w, r, row, dim) != 0) {
                bad = 1;
                continue;
            }
            y[r] = orc_dot(row, x, dim);
        }
        free(row);
    }
    return bad ? -1 : 0;
}

/* ---- minimal GGUF reader (independent of the product's parser) --------------- */

typedef struct {
    char name[96];
    uint64_t dims[4];
    uint32_t nd;
    int type;
    uint64_t off;
} orc_tensor_t;

typedef struct {
    const uint8_t *p;
    size_t n, i;
    int bad;
} rd_t;

static int rd(rd_t *r, void *dst, size_t n) {
    if (r->bad || n > r->n - r->i) {
        r->bad = 1;
        return 0;
    }
    if (dst) memcpy(dst, r->p + r->i, n);
    r->i += n;
    return 1;
}
static uint32_t rd32(rd_t *r) {
    uint32_t v = 0;
    rd(r, &v, 4);
    return v;
}
static uint64_t rd64(rd_t *r) {
    uint64_t v = 0;
    rd(r, &v, 8);
    return v;
}

static size_t scalar_bytes(uint32_t t) {
    static const size_t w[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    return t < 13 ? w[t] : 0;
}

static void skip_value(rd_t *r, uint32_t t) {
    if (t == 8) {
        uint64_t n = rd64(r);
        rd(r, NULL, (size_t)n);
    } else if (t == 9) {
        uint32_t et = rd32(r);
        uint64_t cnt = rd64(r);
        for (uint64_t i = 0; i < cnt && !r->bad; i++) skip_value(r, et);
    } else {
        size_t w = scalar_bytes(t);
        if (!w) r->bad = 1;
        rd(r, NULL, w);
    }
}

struct orc_model {
    int dim, n_layers, n_heads, n_kv, head_dim, ffn, vocab, ctx;
    float eps, rope_base;
    uint8_t *file;
    size_t file_size, data_off;
    /* embedding stays in its GGUF type; everything else is fp32 */
    int embd_type;
    const void *embd;
    float *output; /* [vocab][dim] */
    float *output_norm;
    float **attn_norm, **ffn_norm, **wq, **wk, **wv, **wo, **w1, **w2, **w3;
};

static const orc_tensor_t *find_t(const orc_tensor_t *ts, size_t n, const char *name) {
    for (size_t i = 0; i < n; i++)
        if (!strcmp(ts[i].name, name)) return &ts[i];
    return NULL;
}

static float *dequant_all(orc_model_t *m, const orc_tensor_t *t, int rows, int cols) {
    if (!t || t->dims[0] != (uint64_t)cols || (rows > 1 && t->dims[1] != (uint64_t)rows)) return NULL;
    float *out = (float *)malloc((size_t)rows * cols * 4);
    if (!out) return NULL;
    const uint8_t *data = m->file + m->data_off + t->off;
    int bad = 0;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++)
        if (orc_dequant_row_f32(t->type, data, r, out + (size_t)r * cols, cols) != 0) bad = 1;
    if (bad) {
        free(out);
        return NULL;
    }
    return out;
}

void orc_model_free(orc_model_t *m) {
    if (!m) return;
    float **arrs[9] = {m->attn_norm, m->ffn_norm, m->wq, m->wk, m->wv, m->wo, m->w1, m->w2, m->w3};
    for (int a = 0; a < 9; a++) {
        if (!arrs[a]) continue;
        for (int l = 0; l < m->n_layers; l++) free(arrs[a][l]);
        free(arrs[a]);
    }
    free(m->output);
    free(m->output_norm);
    free(m->file);
    free(m);
}

orc_model_t *orc_model_load(const char *path, int n_threads) {
    set_threads(n_threads);
    FILE *f = fopen(path, "rb");
    if (!f) return NULL;
    fseek(f, 0, SEEK_END);
    long fs = ftell(f);
    fseek(f, 0, SEEK_SET);
    orc_model_t *m = (orc_model_t *)calloc(1, sizeof(*m));
    m->file = (uint8_t *)malloc((size_t)fs);
    if (!m->file || fread(m->file, 1, (size_t)fs, f) != (size_t)fs) {
        fclose(f);
        orc_model_free(m);
        return NULL;
    }
    fclose(f);
    m->file_size = (size_t)fs;
    rd_t r = {m->file, m->file_size, 0, 0};
    if (rd32(&r) != 0x46554747u) {
        orc_model_free(m);
        return NULL;
    }
    uint32_t ver = rd32(&r);
    uint64_t nt = rd64(&r), nkv = rd64(&r);
    if (ver < 2 || ver > 3) {
        orc_model_free(m);
        return NULL;
    }
    uint32_t align = 32;
    m->ctx = 2048;
    m->rope_base = 10000.0f;
    m->eps = 1e-5f;
    m->n_kv = -1;
    for (uint64_t i = 0; i < nkv && !r.bad; i++) {
        uint64_t kl = rd64(&r);
        char key[128] = {0};
        if (kl < sizeof(key))
            rd(&r, key, (size_t)kl);
        else
            rd(&r, NULL, (size_t)kl);
        uint32_t t = rd32(&r);
        if (t == 4 || t == 5) {
            uint32_t v = rd32(&r);
            if (!strcmp(key, "llama.block_count")) m->n_layers = (int)v;
            else if (!strcmp(key, "llama.attention.head_count")) m->n_heads = (int)v;
            else if (!strcmp(key, "llama.attention.head_count_kv")) m->n_kv = (int)v;
            else if (!strcmp(key, "llama.embedding_length")) m->dim = (int)v;
            else if (!strcmp(key, "llama.feed_forward_length")) m->ffn = (int)v;
            else if (!strcmp(key, "llama.context_length")) m->ctx = (int)v;
            else if (!strcmp(key, "general.alignment") && t == 4) align = v;
        } else if (t == 6) {
            float v;
            rd(&r, &v, 4);
            if (!strcmp(key, "llama.rope.freq_base")) m->rope_base = v;
            else if (!strcmp(key, "llama.attention.layer_norm_rms_epsilon")) m->eps = v;
        } else if (t == 9 && !strcmp(key, "tokenizer.ggml.tokens")) {
            size_t save = r.i;
            rd32(&r);
            m->vocab = (int)rd64(&r);
            r.i = save;
            skip_value(&r, t);
        } else {
            skip_value(&r, t);
        }
    }
    if (m->n_kv < 0) m->n_kv = m->n_heads;
    orc_tensor_t *ts = (orc_tensor_t *)calloc(nt ? nt : 1, sizeof(orc_tensor_t));
    for (uint64_t i = 0; i < nt && !r.bad; i++) {
        uint64_t nl = rd64(&r);
        if (nl < sizeof(ts[i].name))
            rd(&r, ts[i].name, (size_t)nl);
        else
            rd(&r, NULL, (size_t)nl);
        ts[i].nd = rd32(&r);
        for (uint32_t d = 0; d < 4; d++) ts[i].dims[d] = (d < ts[i].nd && ts[i].nd <= 4) ? rd64(&r) : 1;
        ts[i].type = (int)rd32(&r);
        ts[i].off = rd64(&r);
    }
    if (r.bad || !m->dim || !m->n_heads || !m->n_layers) {
        free(ts);
        orc_model_free(m);
        return NULL;
    }
    m->data_off = (r.i + align - 1) / align * align;
    m->head_dim = m->dim / m->n_heads;
    int kvd = m->n_kv * m->head_dim;
    const orc_tensor_t *te = find_t(ts, nt, "token_embd.weight");
    if (!te) {
        free(ts);
        orc_model_free(m);
        return NULL;
    }
    if (!m->vocab) m->vocab = (int)te->dims[1];
    m->embd_type = te->type;
    m->embd = m->file + m->data_off + te->off;
    const orc_tensor_t *to = find_t(ts, nt, "output.weight");
    m->output = dequant_all(m, to ? to : te, m->vocab, m->dim);
    m->output_norm = dequant_all(m, find_t(ts, nt, "output_norm.weight"), 1, m->dim);
    float ***arrs[9] = {&m->attn_norm, &m->ffn_norm, &m->wq, &m->wk, &m->wv, &m->wo, &m->w1, &m->w2, &m->w3};
    const char *suf[9] = {"attn_norm", "ffn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_down", "ffn_up"};
    const int rows[9] = {1, 1, m->dim, kvd, kvd, m->dim, m->ffn, m->dim, m->ffn};
    const int cols[9] = {m->dim, m->dim, m->dim, m->dim, m->dim, m->dim, m->dim, m->ffn, m->dim};
    int ok = m->output && m->output_norm;
    for (int a = 0; a < 9 && ok; a++) {
        *arrs[a] = (float **)calloc((size_t)(unsigned)m->n_layers, sizeof(float *));
        for (int l = 0; l < m->n_layers && ok; l++) {
            char nm[96];
            snprintf(nm, sizeof(nm), "blk.%d.%s.weight", l, suf[a]);
            (*arrs[a])[l] = dequant_all(m, find_t(ts, nt, nm), rows[a], cols[a]);
            ok = (*arrs[a])[l] != NULL;
        }
    }
    free(ts);
    if (!ok) {
        orc_model_free(m);
        return NULL;
    }
    return m;
}

void orc_model_dims(const orc_model_t *m, int out[8]) {
    out[0] = m->dim;
    out[1] = m->n_layers;
    out[2] = m->n_heads;
    out[3] = m->n_kv;
    out[4] = m->head_dim;
    out[5] = m->ffn;
    out[6] = m->vocab;
    out[7] = m->ctx;
}

/* ---- forward (src/fiber_proof.m:23-154) ------------------------------------------ */

struct orc_state {
    const orc_model_t *m;
    int max_seq, kv_fp16, threads;
    float **k_cache, **v_cache; /* [layer][pos * kv_dim + ...] */
    float *x, *xnorm, *q, *k, *v, *att, *proj, *h1, *h3, *ffo, *scores;
};

void orc_state_free(orc_state_t *s) {
    if (!s) return;
    if (s->k_cache)
        for (int l = 0; l < s->m->n_layers; l++) free(s->k_cache[l]);
    if (s->v_cache)
        for (int l = 0; l < s->m->n_layers; l++) free(s->v_cache[l]);
    free(s->k_cache);
    free(s->v_cache);
    free(s->x); free(s->xnorm); free(s->q); free(s->k); free(s->v); free(s->att);
    free(s->proj); free(s->h1); free(s->h3); free(s->ffo); free(s->scores);
    free(s);
}

orc_state_t *orc_state_new(const orc_model_t *m, int max_seq, int kv_fp16, int n_threads) {
    orc_state_t *s = (orc_state_t *)calloc(1, sizeof(*s));
    s->m = m;
    s->max_seq = max_seq;
    s->kv_fp16 = kv_fp16;
    s->threads = n_threads;
    int kvd = m->n_kv * m->head_dim;
    s->k_cache = (float **)calloc((size_t)(unsigned)m->n_layers, sizeof(float *));
    s->v_cache = (float **)calloc((size_t)(unsigned)m->n_layers, sizeof(float *));
    int ok = s->k_cache && s->v_cache;
    for (int l = 0; l < m->n_layers && ok; l++) {
        s->k_cache[l] = (float *)calloc((size_t)max_seq * kvd, 4);
        s->v_cache[l] = (float *)calloc((size_t)max_seq * kvd, 4);
        ok = s->k_cache[l] && s->v_cache[l];
    }
    s->x = (float *)malloc((size_t)m->dim * 4);
    s->xnorm = (float *)malloc((size_t)m->dim * 4);
    s->q = (float *)malloc((size_t)m->dim * 4);
    s->k = (float *)malloc((size_t)m->dim * 4);
    s->v = (float *)malloc((size_t)m->dim * 4);
    s->att = (float *)malloc((size_t)m->dim * 4);
    s->proj = (float *)malloc((size_t)m->dim * 4);
    s->h1 = (float *)malloc((size_t)m->ffn * 4);
    s->h3 = (float *)malloc((size_t)m->ffn * 4);
    s->ffo = (float *)malloc((size_t)m->dim * 4);
    s->scores = (float *)malloc((size_t)max_seq * 4);
    ok = ok && s->x && s->xnorm && s->q && s->k && s->v && s->att && s->proj && s->h1 && s->h3 &&
         s->ffo && s->scores;
    if (!ok) {
        orc_state_free(s);
        return NULL;
    }
    return s;
}

static float kv_round(const orc_state_t *s, float v) { return s->kv_fp16 ? h2f(f2h(v)) : v; }

int orc_state_set_kv(orc_state_t *s, int layer, int pos, const float *k, const float *v) {
    const orc_model_t *m = s->m;
    if (layer < 0 || layer >= m->n_layers || pos < 0 || pos >= s->max_seq) return -1;
    int kvd = m->n_kv * m->head_dim;
    for (int i = 0; i < kvd; i++) {
        s->k_cache[layer][(size_t)pos * kvd + i] = kv_round(s, k[i]);
        s->v_cache[layer][(size_t)pos * kvd + i] = kv_round(s, v[i]);
    }
    return 0;
}

int orc_state_get_kv(const orc_state_t *s, int layer, int pos, float *k, float *v) {
    const orc_model_t *m = s->m;
    if (layer < 0 || layer >= m->n_layers || pos < 0 || pos >= s->max_seq) return -1;
    int kvd = m->n_kv * m->head_dim;
    memcpy(k, s->k_cache[layer] + (size_t)pos * kvd, (size_t)kvd * 4);
    memcpy(v, s->v_cache[layer] + (size_t)pos * kvd, (size_t)kvd * 4);
    return 0;
}

/* src/fiber_proof.m:23-28 */
static void rmsnorm(float *out, const float *x, const float *w, int dim, float eps) {
    float ss = 0;
    for (int i = 0; i < dim; i++) ss += x[i] * x[i];
    float rrms = 1.0f / sqrtf(ss / dim + eps);
    for (int i = 0; i < dim; i++) out[i] = x[i] * rrms * w[i];
}

/* src/fiber_proof.m:30-51: half-split pairs (i, i + hd/2) */
static void rope(float *q, float *k, int heads, int kv_heads, int hd, int pos, float base) {
    for (int h = 0; h < heads + kv_heads; h++) {
        float *v = h < heads ? q + h * hd : k + (h - heads) * hd;
        for (int i = 0; i < hd / 2; i++) {
            float freq = 1.0f / powf(base, 2.0f * i / (float)hd);
            float angle = pos * freq;
            float c = cosf(angle), sn = sinf(angle);
            float x1 = v[i], x2 = v[i + hd / 2];
            v[i] = x1 * c - x2 * sn;
            v[i + hd / 2] = x1 * sn + x2 * c;
        }
    }
}

static void matvec(const float *w, const float *x, float *y, int rows, int cols) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) y[r] = orc_dot(w + (size_t)r * cols, x, cols);
}

int orc_forward_token(orc_state_t *s, int token, int pos, float *logits) {
    const orc_model_t *m = s->m;
    if (token < 0 || token >= m->vocab || pos < 0 || pos >= s->max_seq) return -1;
    set_threads(s->threads);
    const int dim = m->dim, hd = m->head_dim, H = m->n_heads, KVH = m->n_kv, kvd = KVH * hd;
    const float eps = m->eps;
    if (orc_embed_row(m->embd_type, m->embd, token, s->x, dim) != 0) return -1;
    float *x = s->x;
    for (int l = 0; l < m->n_layers; l++) {
        rmsnorm(s->xnorm, x, m->attn_norm[l], dim, eps);
        matvec(m->wq[l], s->xnorm, s->q, dim, dim);
        matvec(m->wk[l], s->xnorm, s->k, kvd, dim);
        matvec(m->wv[l], s->xnorm, s->v, kvd, dim);
        rope(s->q, s->k, H, KVH, hd, pos, m->rope_base);
        for (int i = 0; i < kvd; i++) {
            s->k_cache[l][(size_t)pos * kvd + i] = kv_round(s, s->k[i]);
            s->v_cache[l][(size_t)pos * kvd + i] = kv_round(s, s->v[i]);
        }
        memset(s->att, 0, (size_t)dim * 4);
        const float scale = 1.0f / sqrtf((float)hd);
        for (int h = 0; h < H; h++) {
            int kvh = h * KVH / H;
            float *sc = s->scores;
            for (int t = 0; t <= pos; t++) {
                float dot = 0;
                for (int d = 0; d < hd; d++) dot += s->q[h * hd + d] * s->k_cache[l][(size_t)t * kvd + kvh * hd + d];
                sc[t] = dot * scale;
            }
            float mx = sc[0];
            for (int t = 1; t <= pos; t++)
                if (sc[t] > mx) mx = sc[t];
            float sum = 0;
            for (int t = 0; t <= pos; t++) {
                sc[t] = expf(sc[t] - mx);
                sum += sc[t];
            }
            for (int t = 0; t <= pos; t++) sc[t] /= sum;
            for (int t = 0; t <= pos; t++)
                for (int d = 0; d < hd; d++) s->att[h * hd + d] += sc[t] * s->v_cache[l][(size_t)t * kvd + kvh * hd + d];
        }
        matvec(m->wo[l], s->att, s->proj, dim, dim);
        for (int d = 0; d < dim; d++) x[d] += s->proj[d];
        rmsnorm(s->xnorm, x, m->ffn_norm[l], dim, eps);
        matvec(m->w1[l], s->xnorm, s->h1, m->ffn, dim);
        matvec(m->w3[l], s->xnorm, s->h3, m->ffn, dim);
        for (int i = 0; i < m->ffn; i++) {
            float sg = s->h1[i] / (1.0f + expf(-s->h1[i]));
            s->h1[i] = sg * s->h3[i];
        }
        matvec(m->w2[l], s->h1, s->ffo, dim, m->ffn);
        for (int d = 0; d < dim; d++) x[d] += s->ffo[d];
    }
    /* classifier: plain sequential dot per vocabulary row (src/fiber_proof.m:145-151) */
    rmsnorm(s->xnorm, x, m->output_norm, dim, eps);
    const float *xn = s->xnorm;
#pragma omp parallel for schedule(static)
    for (int v = 0; v < m->vocab; v++) {
        const float *w = m->output + (size_t)v * dim;
        float dot = 0;
        for (int d = 0; d < dim; d++) dot += w[d] * xn[d];
        logits[v] = dot;
    }
    return 0;
}

int orc_argmax(const float *v, int n) {
    int best = 0;
    for (int i = 1; i < n; i++)
        if (v[i] > v[best]) best = i;
    return best;
}

int orc_generate(orc_state_t *s, const int *prompt, int n_prompt, int start, int n_gen, int *out,
                 float *last_logits) {
    const orc_model_t *m = s->m;
    float *lg = (float *)malloc((size_t)m->vocab * 4);
    if (!lg || n_prompt < 1) {
        free(lg);
        return -1;
    }
    int pos = start;
    for (int i = 0; i < n_prompt; i++, pos++)
        if (orc_forward_token(s, prompt[i], pos, lg) != 0) {
            free(lg);
            return -1;
        }
    out[0] = orc_argmax(lg, m->vocab);
    for (int i = 0; i < n_gen; i++, pos++) {
        if (orc_forward_token(s, out[i], pos, lg) != 0) {
            free(lg);
            return -1;
        }
        out[i + 1] = orc_argmax(lg, m->vocab);
    }
    if (last_logits) memcpy(last_logits, lg, (size_t)m->vocab * 4);
    free(lg);
    return 0;
}
