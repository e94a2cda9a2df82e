/* synth.c — seeded synthetic GGUF models, K-quant quantizers and random blocks.
 *
 * Randomness is counter-based: every (tensor, row) pair gets its own splitmix64
 * seed, so rows can be generated in parallel with any thread count and the
 * bytes written do not depend on it.
 */
#include "fiber_synth.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "gguf.h"

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- random numbers ----------------------------------------------------------- */

static uint64_t splitmix64(uint64_t *s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static uint64_t mix_seed(uint64_t seed, uint64_t a, uint64_t b) {
    uint64_t s = seed ^ (a * 0xD1B54A32D192ED03ull) ^ (b * 0x8CB92BA72F3D8DD7ull);
    splitmix64(&s);
    return splitmix64(&s);
}

/* uniform in (0, 1] with 24 random bits */
static float unif01(uint64_t *s) { return ((float)(splitmix64(s) >> 40) + 1.0f) * (1.0f / 16777216.0f); }

/* Box-Muller pairs */
static void fill_normal(float *dst, size_t n, uint64_t *s, float std) {
    const float two_pi = 6.28318530717958647692f;
    size_t i = 0;
    for (; i + 1 < n; i += 2) {
        float u1 = unif01(s), u2 = unif01(s);
        float r = sqrtf(-2.0f * logf(u1)) * std;
        dst[i] = r * cosf(two_pi * u2);
        dst[i + 1] = r * sinf(two_pi * u2);
    }
    if (i < n) {
        float u1 = unif01(s), u2 = unif01(s);
        dst[i] = sqrtf(-2.0f * logf(u1)) * std * cosf(two_pi * u2);
    }
}

void fiber_randn(float *dst, size_t n, uint64_t seed, float std) {
    const size_t chunk = 4096;
    size_t nchunks = (n + chunk - 1) / chunk;
#pragma omp parallel for schedule(static)
    for (long long c = 0; c < (long long)nchunks; c++) {
        uint64_t s = mix_seed(seed, 0xABCDull, (uint64_t)c);
        size_t lo = (size_t)c * chunk, cnt = n - lo < chunk ? n - lo : chunk;
        fill_normal(dst + lo, cnt, &s, std);
    }
}

static uint16_t to_f16(float f) {
    _Float16 h = (_Float16)f;
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}

static float from_f16(uint16_t u) {
    _Float16 h;
    memcpy(&h, &u, 2);
    return (float)h;
}

static int iclamp(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* ---- K-quant quantizers (one 256-value super-block each) ---------------------- */

/* Pack 8 six-bit scales and mins into the 12-byte field read by
 * get_scale_min_k4 (metal/kernels.metal:10-19, src/dequant.h:19-23). */
static void pack_scale_min(uint8_t out[12], const int sc[8], const int mn[8]) {
    for (int j = 0; j < 4; j++) {
        out[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        out[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
        out[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
    }
}

/* Asymmetric sub-block fit shared by Q4_K (qmax 15) and Q5_K (qmax 31):
 * value ≈ d*sc*q - dmin*m with q in [0, qmax]. Writes header + q[256]. */
static void fit_asym(const float *x, int qmax, uint8_t *hdr, int q[256]) {
    float scale[8], mins[8], smax = 0.0f, mmax = 0.0f;
    for (int s = 0; s < 8; s++) {
        float lo = x[32 * s], hi = x[32 * s];
        for (int i = 1; i < 32; i++) {
            float v = x[32 * s + i];
            lo = v < lo ? v : lo;
            hi = v > hi ? v : hi;
        }
        if (lo > 0.0f) lo = 0.0f;
        scale[s] = (hi - lo) / (float)qmax;
        mins[s] = -lo;
        if (scale[s] > smax) smax = scale[s];
        if (mins[s] > mmax) mmax = mins[s];
    }
    uint16_t dh = to_f16(smax / 63.0f), mh = to_f16(mmax / 63.0f);
    float d = from_f16(dh), dm = from_f16(mh);
    int sc[8], mn[8];
    for (int s = 0; s < 8; s++) {
        sc[s] = d > 0.0f ? iclamp((int)lrintf(scale[s] / d), 0, 63) : 0;
        mn[s] = dm > 0.0f ? iclamp((int)lrintf(mins[s] / dm), 0, 63) : 0;
    }
    memcpy(hdr, &dh, 2);
    memcpy(hdr + 2, &mh, 2);
    pack_scale_min(hdr + 4, sc, mn);
    for (int s = 0; s < 8; s++) {
        float step = d * (float)sc[s], off = dm * (float)mn[s];
        for (int i = 0; i < 32; i++) {
            float v = x[32 * s + i];
            q[32 * s + i] = step > 0.0f ? iclamp((int)lrintf((v + off) / step), 0, qmax) : 0;
        }
    }
}

static void quant_q4k_block(const float *x, uint8_t *blk) {
    int q[256];
    fit_asym(x, 15, blk, q);
    uint8_t *qs = blk + 16;
    for (int j = 0; j < 4; j++)
        for (int l = 0; l < 32; l++)
            qs[32 * j + l] = (uint8_t)(q[64 * j + l] | (q[64 * j + 32 + l] << 4));
}

static void quant_q5k_block(const float *x, uint8_t *blk) {
    int q[256];
    fit_asym(x, 31, blk, q);
    uint8_t *qh = blk + 16, *qs = blk + 48;
    memset(qh, 0, 32);
    for (int g = 0; g < 4; g++)
        for (int w = 0; w < 32; w++) {
            int lo = q[64 * g + w], hi = q[64 * g + 32 + w];
            qs[32 * g + w] = (uint8_t)((lo & 15) | ((hi & 15) << 4));
            qh[w] |= (uint8_t)(((lo >> 4) & 1) << (2 * g));
            qh[w] |= (uint8_t)(((hi >> 4) & 1) << (2 * g + 1));
        }
}

static void quant_q6k_block(const float *x, uint8_t *blk) {
    float scale[16], amax_all = 0.0f;
    for (int s = 0; s < 16; s++) {
        float am = 0.0f;
        for (int i = 0; i < 16; i++) {
            float a = fabsf(x[16 * s + i]);
            am = a > am ? a : am;
        }
        scale[s] = am / 31.0f;
        if (scale[s] > amax_all) amax_all = scale[s];
    }
    uint16_t dh = to_f16(amax_all / 127.0f);
    float d = from_f16(dh);
    int8_t sc[16];
    int q[256];
    for (int s = 0; s < 16; s++) {
        int v = d > 0.0f ? iclamp((int)lrintf(scale[s] / d), -128, 127) : 0;
        sc[s] = (int8_t)v;
        float step = d * (float)v;
        for (int i = 0; i < 16; i++)
            q[16 * s + i] = step != 0.0f ? iclamp((int)lrintf(x[16 * s + i] / step), -32, 31) : 0;
    }
    /* layout of src/dequant.h:34-58: per 128-element half, ql[64] qh[32] sc[8] */
    uint8_t *ql = blk, *qh = blk + 128;
    memset(blk, 0, 210);
    for (int h = 0; h < 2; h++) {
        const int *qq = q + 128 * h;
        uint8_t *l8 = ql + 64 * h, *h8 = qh + 32 * h;
        for (int l = 0; l < 32; l++) {
            int u0 = qq[l] + 32, u1 = qq[l + 32] + 32, u2 = qq[l + 64] + 32, u3 = qq[l + 96] + 32;
            l8[l] = (uint8_t)((u0 & 15) | ((u2 & 15) << 4));
            l8[l + 32] = (uint8_t)((u1 & 15) | ((u3 & 15) << 4));
            h8[l] = (uint8_t)((u0 >> 4) | ((u1 >> 4) << 2) | ((u2 >> 4) << 4) | ((u3 >> 4) << 6));
        }
    }
    memcpy(blk + 192, sc, 16);
    memcpy(blk + 208, &dh, 2);
}

int fiber_quantize_rows(int type, const float *src, void *dst, size_t rows, size_t cols) {
    size_t bb = ggml_type_size((ggml_type_t)type), be = ggml_block_size((ggml_type_t)type);
    if (bb == 0 || cols % be != 0) return -1;
    size_t row_bytes = cols / be * bb;
#pragma omp parallel for schedule(static)
    for (long long r = 0; r < (long long)rows; r++) {
        const float *x = src + (size_t)r * cols;
        uint8_t *o = (uint8_t *)dst + (size_t)r * row_bytes;
        switch (type) {
        case GGML_TYPE_F32: memcpy(o, x, cols * 4); break;
        case GGML_TYPE_F16:
            for (size_t i = 0; i < cols; i++) {
                uint16_t h = to_f16(x[i]);
                memcpy(o + 2 * i, &h, 2);
            }
            break;
        case GGML_TYPE_Q4_K:
            for (size_t b = 0; b < cols / 256; b++) quant_q4k_block(x + 256 * b, o + 144 * b);
            break;
        case GGML_TYPE_Q5_K:
            for (size_t b = 0; b < cols / 256; b++) quant_q5k_block(x + 256 * b, o + 176 * b);
            break;
        case GGML_TYPE_Q6_K:
            for (size_t b = 0; b < cols / 256; b++) quant_q6k_block(x + 256 * b, o + 210 * b);
            break;
        default: break;
        }
    }
    return (type == GGML_TYPE_F32 || type == GGML_TYPE_F16 || type == GGML_TYPE_Q4_K ||
            type == GGML_TYPE_Q5_K || type == GGML_TYPE_Q6_K)
               ? 0
               : -1;
}

int fiber_random_blocks(int type, void *dst, size_t rows, size_t cols, uint64_t seed,
                        float d_scale, float dmin_scale) {
    if (cols % 256 != 0) return -1;
    size_t bb = ggml_type_size((ggml_type_t)type);
    if (type != GGML_TYPE_Q4_K && type != GGML_TYPE_Q5_K && type != GGML_TYPE_Q6_K) return -1;
    size_t nb = cols / 256;
#pragma omp parallel for schedule(static)
    for (long long r = 0; r < (long long)rows; r++) {
        uint64_t s = mix_seed(seed, 0x5151ull, (uint64_t)r);
        for (size_t b = 0; b < nb; b++) {
            uint8_t *blk = (uint8_t *)dst + ((size_t)r * nb + b) * bb;
            float nd[2];
            fill_normal(nd, 2, &s, 1.0f);
            uint16_t dh = to_f16(fabsf(nd[0]) * d_scale), mh = to_f16(fabsf(nd[1]) * dmin_scale);
            if (type == GGML_TYPE_Q6_K) {
                for (int i = 0; i < 192; i++) blk[i] = (uint8_t)(splitmix64(&s) >> 56);
                for (int i = 0; i < 16; i++) blk[192 + i] = (uint8_t)(splitmix64(&s) >> 56);
                memcpy(blk + 208, &dh, 2);
            } else {
                memcpy(blk, &dh, 2);
                memcpy(blk + 2, &mh, 2);
                int sc[8], mn[8];
                for (int i = 0; i < 8; i++) {
                    sc[i] = (int)(splitmix64(&s) >> 58);
                    mn[i] = (int)(splitmix64(&s) >> 58);
                }
                pack_scale_min(blk + 4, sc, mn);
                size_t rest = bb - 16; /* Q4_K: qs[128]; Q5_K: qh[32] + qs[128] */
                for (size_t i = 0; i < rest; i++) blk[16 + i] = (uint8_t)(splitmix64(&s) >> 56);
            }
        }
    }
    return 0;
}

/* ---- model recipe ------------------------------------------------------------- */

int fiber_synth_recipe_type(int recipe, int role, uint32_t layer, uint32_t n_layers) {
    (void)n_layers;
    switch (recipe) {
    case FIBER_RECIPE_F16: return GGML_TYPE_F16;
    case FIBER_RECIPE_Q4_K: return GGML_TYPE_Q4_K;
    case FIBER_RECIPE_Q5_K: return GGML_TYPE_Q5_K;
    case FIBER_RECIPE_Q6_K: return GGML_TYPE_Q6_K;
    case FIBER_RECIPE_Q4_K_M:
        if (role == 8) return GGML_TYPE_Q6_K;
        if ((role == 2 || role == 5) && layer % 2 == 0) return GGML_TYPE_Q6_K;
        return GGML_TYPE_Q4_K;
    case FIBER_RECIPE_Q5_K_M:
        if (role == 8 || role == 2 || role == 5) return GGML_TYPE_Q6_K;
        return GGML_TYPE_Q5_K;
    default: return -1;
    }
}

int fiber_synth_preset(const char *name, fiber_synth_cfg_t *c) {
    memset(c, 0, sizeof(*c));
    c->rope_base = 10000.0f;
    c->eps = 1e-5f;
    c->weight_std = 0.02f;
    c->norm_value = 1.0f;
    c->seed = 1234;
    c->vocab = 32000;
    if (!strcmp(name, "stories")) {
        c->dim = 768; c->n_layers = 12; c->n_heads = 12; c->n_kv_heads = 12;
        c->ffn_dim = 2048; c->context_length = 1024; c->recipe = FIBER_RECIPE_F16; c->tied = 1;
    } else if (!strcmp(name, "tinyllama")) {
        c->dim = 2048; c->n_layers = 22; c->n_heads = 32; c->n_kv_heads = 4;
        c->ffn_dim = 5632; c->context_length = 2048; c->recipe = FIBER_RECIPE_Q4_K_M;
    } else if (!strcmp(name, "tinyllama-q5")) {
        c->dim = 2048; c->n_layers = 22; c->n_heads = 32; c->n_kv_heads = 4;
        c->ffn_dim = 5632; c->context_length = 4096; c->recipe = FIBER_RECIPE_Q5_K_M;
    } else if (!strcmp(name, "llama7b")) {
        c->dim = 4096; c->n_layers = 32; c->n_heads = 32; c->n_kv_heads = 32;
        c->ffn_dim = 11008; c->context_length = 4096; c->recipe = FIBER_RECIPE_Q4_K_M;
    } else {
        return -1;
    }
    return 0;
}

/* ---- GGUF writer ---------------------------------------------------------------- */

typedef struct {
    uint8_t *p;
    size_t n, cap;
    int oom;
} wbuf_t;

static void wb_put(wbuf_t *b, const void *src, size_t n) {
    if (b->oom) return;
    if (b->n + n > b->cap) {
        size_t nc = b->cap ? b->cap : 1 << 16;
        while (nc < b->n + n) nc *= 2;
        uint8_t *np = (uint8_t *)realloc(b->p, nc);
        if (!np) {
            b->oom = 1;
            return;
        }
        b->p = np;
        b->cap = nc;
    }
    memcpy(b->p + b->n, src, n);
    b->n += n;
}
static void wb_u32(wbuf_t *b, uint32_t v) { wb_put(b, &v, 4); }
static void wb_u64(wbuf_t *b, uint64_t v) { wb_put(b, &v, 8); }
static void wb_f32(wbuf_t *b, float v) { wb_put(b, &v, 4); }
static void wb_str(wbuf_t *b, const char *s, size_t n) {
    wb_u64(b, n);
    wb_put(b, s, n);
}
static void kv_key(wbuf_t *b, const char *k, uint32_t type) {
    wb_str(b, k, strlen(k));
    wb_u32(b, type);
}
static void kv_u32(wbuf_t *b, const char *k, uint32_t v) { kv_key(b, k, GGUF_TYPE_UINT32); wb_u32(b, v); }
static void kv_f32(wbuf_t *b, const char *k, float v) { kv_key(b, k, GGUF_TYPE_FLOAT32); wb_f32(b, v); }
static void kv_s(wbuf_t *b, const char *k, const char *v) {
    kv_key(b, k, GGUF_TYPE_STRING);
    wb_str(b, v, strlen(v));
}

/* Synthetic SentencePiece vocabulary: <unk> <s> </s>, 256 byte tokens, "▁",
 * printable ASCII, "▁"+letter, letter pairs, then filler pieces. */
static void build_vocab(uint32_t vocab, uint64_t seed, wbuf_t *toks, wbuf_t *scores,
                        wbuf_t *types) {
    uint64_t s = mix_seed(seed, 0x70C0ull, 0);
    char piece[32];
    uint32_t id = 0;
#define ADD(str, len, score, ty)                          \
    do {                                                  \
        if (id < vocab) {                                 \
            wb_str(toks, (str), (len));                   \
            wb_f32(scores, (score));                      \
            int32_t t_ = (ty);                            \
            wb_put(types, &t_, 4);                        \
            id++;                                         \
        }                                                 \
    } while (0)
    ADD("<unk>", 5, 0.0f, 2);
    ADD("<s>", 3, 0.0f, 3);
    ADD("</s>", 4, 0.0f, 3);
    for (int b = 0; b < 256; b++) {
        snprintf(piece, sizeof(piece), "<0x%02X>", b);
        ADD(piece, 6, 0.0f, 6);
    }
    const char mark[3] = {(char)0xE2, (char)0x96, (char)0x81};
    ADD(mark, 3, -1.0f, 1);
    for (int ch = 33; ch < 127; ch++) {
        piece[0] = (char)ch;
        ADD(piece, 1, -2.0f - (float)(splitmix64(&s) >> 40) / 16777216.0f, 1);
    }
    for (int ch = 'a'; ch <= 'z'; ch++) {
        memcpy(piece, mark, 3);
        piece[3] = (char)ch;
        ADD(piece, 4, -10.0f - (float)(splitmix64(&s) >> 40) / 1677721.6f, 1);
    }
    for (int a = 'a'; a <= 'z'; a++)
        for (int c = 'a'; c <= 'z'; c++) {
            piece[0] = (char)a;
            piece[1] = (char)c;
            ADD(piece, 2, -20.0f - (float)(splitmix64(&s) >> 40) / 1677721.6f, 1);
        }
    for (uint32_t k = 0; id < vocab; k++) {
        int n = snprintf(piece, sizeof(piece), "\xE2\x96\x81w%u", k);
        ADD(piece, (size_t)n, -100.0f - (float)k * 1e-3f, 1);
    }
#undef ADD
}

typedef struct {
    char name[64];
    uint32_t n_dims;
    uint64_t dims[2];
    int type;
    uint64_t offset;
    size_t bytes;
    int role;      /* recipe role, or a FIBER_ROLE_*_NORM value */
    uint32_t layer;
} tdesc_t;

/* Writes the Llama GGUF of cfg's shape; fill (or, when NULL, the seeded generator)
 * gives every tensor's fp32 values before they are quantized to the recipe's type. */
static int write_gguf(const char *path, const fiber_synth_cfg_t *cfg, fiber_tensor_fill_fn fill, void *user) {
    const uint32_t L = cfg->n_layers, D = cfg->dim, F = cfg->ffn_dim;
    const uint32_t KV = cfg->n_kv_heads * (cfg->dim / cfg->n_heads);
    if (!L || !D || !F || !cfg->n_heads || !cfg->n_kv_heads || D % cfg->n_heads ||
        cfg->n_heads % cfg->n_kv_heads || D % 256 || F % 256 || cfg->vocab < 300) {
        fprintf(stderr, "synth: unsupported shape\n");
        return -1;
    }
#ifdef _OPENMP
    if (cfg->n_threads > 0) omp_set_num_threads(cfg->n_threads);
#endif
    size_t nt = 2 + (cfg->tied ? 0 : 1) + 9 * (size_t)L;
    tdesc_t *td = (tdesc_t *)calloc(nt, sizeof(tdesc_t));
    if (!td) return -1;
    size_t k = 0;
#define T(nm, in, out, ty, rl, ly)                                                     \
    do {                                                                               \
        snprintf(td[k].name, sizeof(td[k].name), "%s", (nm));                          \
        td[k].dims[0] = (in);                                                          \
        td[k].dims[1] = (out);                                                         \
        td[k].n_dims = (out) > 1 ? 2 : 1;                                              \
        td[k].type = (ty);                                                             \
        td[k].role = (rl);                                                             \
        td[k].layer = (ly);                                                            \
        k++;                                                                           \
    } while (0)
    T("token_embd.weight", D, cfg->vocab, fiber_synth_recipe_type(cfg->recipe, 7, 0, L), 7, 0);
    T("output_norm.weight", D, 1, GGML_TYPE_F32, FIBER_ROLE_OUTPUT_NORM, 0);
    if (!cfg->tied)
        T("output.weight", D, cfg->vocab, fiber_synth_recipe_type(cfg->recipe, 8, 0, L), 8, 0);
    for (uint32_t l = 0; l < L; l++) {
        char nm[64];
        static const char *suf[7] = {"attn_q", "attn_k", "attn_v", "attn_output",
                                     "ffn_gate", "ffn_down", "ffn_up"};
        const uint64_t in[7] = {D, D, D, D, D, F, D}, out[7] = {D, KV, KV, D, F, D, F};
        snprintf(nm, sizeof(nm), "blk.%u.attn_norm.weight", l);
        T(nm, D, 1, GGML_TYPE_F32, FIBER_ROLE_ATTN_NORM, l);
        for (int r = 0; r < 7; r++) {
            snprintf(nm, sizeof(nm), "blk.%u.%s.weight", l, suf[r]);
            T(nm, in[r], out[r], fiber_synth_recipe_type(cfg->recipe, r, l, L), r, l);
            if (r == 3) {
                snprintf(nm, sizeof(nm), "blk.%u.ffn_norm.weight", l);
                T(nm, D, 1, GGML_TYPE_F32, FIBER_ROLE_FFN_NORM, l);
            }
        }
    }
#undef T
    nt = k;
    const size_t align = 32;
    uint64_t off = 0;
    for (size_t i = 0; i < nt; i++) {
        size_t bb = ggml_type_size((ggml_type_t)td[i].type), be = ggml_block_size((ggml_type_t)td[i].type);
        if (bb == 0 || td[i].dims[0] % be) {
            fprintf(stderr, "synth: bad type for %s\n", td[i].name);
            free(td);
            return -1;
        }
        td[i].bytes = (size_t)(td[i].dims[0] * td[i].dims[1] / be * bb);
        td[i].offset = off;
        off += (td[i].bytes + align - 1) & ~(uint64_t)(align - 1);
    }

    wbuf_t h = {0}, toks = {0}, scores = {0}, types = {0};
    build_vocab(cfg->vocab, cfg->seed, &toks, &scores, &types);
    const uint64_t n_kv = 16;
    wb_u32(&h, GGUF_MAGIC);
    wb_u32(&h, 3);
    wb_u64(&h, nt);
    wb_u64(&h, n_kv);
    kv_s(&h, "general.architecture", "llama");
    kv_s(&h, "general.name", "fiber-synthetic");
    kv_u32(&h, "general.alignment", (uint32_t)align);
    kv_u32(&h, "llama.block_count", L);
    kv_u32(&h, "llama.embedding_length", D);
    kv_u32(&h, "llama.feed_forward_length", F);
    kv_u32(&h, "llama.attention.head_count", cfg->n_heads);
    kv_u32(&h, "llama.attention.head_count_kv", cfg->n_kv_heads);
    kv_u32(&h, "llama.context_length", cfg->context_length);
    kv_f32(&h, "llama.rope.freq_base", cfg->rope_base);
    kv_f32(&h, "llama.attention.layer_norm_rms_epsilon", cfg->eps);
    kv_s(&h, "tokenizer.ggml.model", "llama");
    kv_key(&h, "tokenizer.ggml.tokens", GGUF_TYPE_ARRAY);
    wb_u32(&h, GGUF_TYPE_STRING);
    wb_u64(&h, cfg->vocab);
    wb_put(&h, toks.p, toks.n);
    kv_key(&h, "tokenizer.ggml.scores", GGUF_TYPE_ARRAY);
    wb_u32(&h, GGUF_TYPE_FLOAT32);
    wb_u64(&h, cfg->vocab);
    wb_put(&h, scores.p, scores.n);
    kv_key(&h, "tokenizer.ggml.token_type", GGUF_TYPE_ARRAY);
    wb_u32(&h, GGUF_TYPE_INT32);
    wb_u64(&h, cfg->vocab);
    wb_put(&h, types.p, types.n);
    kv_u32(&h, "tokenizer.ggml.bos_token_id", 1);
    free(toks.p);
    free(scores.p);
    free(types.p);
    /* n_kv counts: 3 general + 8 llama + model + tokens + scores + token_type + bos = 16 */
    for (size_t i = 0; i < nt; i++) {
        wb_str(&h, td[i].name, strlen(td[i].name));
        wb_u32(&h, td[i].n_dims);
        for (uint32_t d = 0; d < td[i].n_dims; d++) wb_u64(&h, td[i].dims[d]);
        wb_u32(&h, (uint32_t)td[i].type);
        wb_u64(&h, td[i].offset);
    }
    while (h.n % align) {
        uint8_t z = 0;
        wb_put(&h, &z, 1);
    }
    if (h.oom) {
        free(h.p);
        free(td);
        return -1;
    }

    FILE *f = fopen(path, "wb");
    if (!f) {
        perror("synth: fopen");
        free(h.p);
        free(td);
        return -1;
    }
    int ok = fwrite(h.p, 1, h.n, f) == h.n;
    free(h.p);

    size_t max_elems = 0, max_bytes = 0;
    for (size_t i = 0; i < nt; i++) {
        size_t ne = (size_t)(td[i].dims[0] * td[i].dims[1]);
        if (ne > max_elems) max_elems = ne;
        if (td[i].bytes > max_bytes) max_bytes = td[i].bytes;
    }
    float *vals = (float *)malloc(max_elems * sizeof(float));
    uint8_t *blob = (uint8_t *)malloc(max_bytes + align);
    if (!vals || !blob) ok = 0;
    for (size_t i = 0; i < nt && ok; i++) {
        size_t rows = (size_t)td[i].dims[1], cols = (size_t)td[i].dims[0];
        if (fill) {
            if (fill(user, td[i].role, td[i].layer, rows, cols, vals) != 0) ok = 0;
        } else if (td[i].role < 0) {
            const float nv = td[i].role == FIBER_ROLE_FFN_NORM && cfg->ffn_norm_value > 0.0f ? cfg->ffn_norm_value
                                                                                               : cfg->norm_value;
            for (size_t e = 0; e < cols; e++) vals[e] = nv;
        } else {
#pragma omp parallel for schedule(static)
            for (long long r = 0; r < (long long)rows; r++) {
                uint64_t s = mix_seed(cfg->seed, (uint64_t)i + 1, (uint64_t)r);
                fill_normal(vals + (size_t)r * cols, cols, &s, cfg->weight_std);
            }
        }
        if (fiber_quantize_rows(td[i].type, vals, blob, rows, cols) != 0) ok = 0;
        size_t padded = (td[i].bytes + align - 1) & ~(size_t)(align - 1);
        memset(blob + td[i].bytes, 0, padded - td[i].bytes);
        if (ok && fwrite(blob, 1, padded, f) != padded) ok = 0;
    }
    free(vals);
    free(blob);
    free(td);
    if (fclose(f) != 0) ok = 0;
    if (!ok) fprintf(stderr, "synth: failed writing %s\n", path);
    return ok ? 0 : -1;
}

int fiber_synth_write_gguf(const char *path, const fiber_synth_cfg_t *cfg) { return write_gguf(path, cfg, NULL, NULL); }

int fiber_write_gguf_from(const char *path, const fiber_synth_cfg_t *cfg, fiber_tensor_fill_fn fill, void *user) {
    if (!fill) return -1;
    return write_gguf(path, cfg, fill, user);
}
