/* ckpt.c — karpathy / llama2.c checkpoints rewritten as Llama GGUF files (fiber_ckpt.h).
 *
 * Follows the file layout read by fiber_model_load_karpathy (src/fiber_ckpt.m:125-259):
 * a 7-int header, then fp32 arrays, each array holding that tensor for every layer. */
#include "fiber_ckpt.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <fcntl.h>
#include <unistd.h>

#include "fiber_synth.h"

typedef struct {
    fiber_karpathy_config_t c;
    const float *base;  /* first float after the header */
    size_t n_floats;    /* floats in the file after the header */
    /* float offsets of each array */
    size_t embd, rms_att, wq, wk, wv, wo, rms_ffn, w1, w2, w3, rms_final, wcls;
} ckpt_t;

static int parse_header(const int32_t h[7], fiber_karpathy_config_t *c) {
    c->dim = h[0];
    c->hidden_dim = h[1];
    c->n_layers = h[2];
    c->n_heads = h[3];
    c->n_kv_heads = h[4] == 0 ? h[3] : h[4];  /* 0 = multi-head */
    c->shared_classifier = h[5] > 0;           /* negative vocab = separate classifier */
    c->vocab_size = h[5] < 0 ? -h[5] : h[5];
    c->seq_len = h[6];
    if (c->dim <= 0 || c->hidden_dim <= 0 || c->n_layers <= 0 || c->n_heads <= 0 || c->n_kv_heads <= 0 ||
        c->vocab_size <= 0 || c->seq_len <= 0 || c->dim % c->n_heads || c->n_heads % c->n_kv_heads)
        return -1;
    return 0;
}

int fiber_karpathy_config(const char *bin_path, fiber_karpathy_config_t *out) {
    FILE *f = fopen(bin_path, "rb");
    if (!f) {
        fprintf(stderr, "karpathy: cannot open %s\n", bin_path);
        return -1;
    }
    int32_t h[7];
    int rc = fread(h, sizeof(int32_t), 7, f) == 7 ? parse_header(h, out) : -1;
    fclose(f);
    if (rc) fprintf(stderr, "karpathy: %s: bad header\n", bin_path);
    return rc;
}

/* Offsets of every array; the file must hold them all. */
static int layout(ckpt_t *k) {
    const fiber_karpathy_config_t *c = &k->c;
    const size_t D = (size_t)c->dim, H = (size_t)c->hidden_dim, L = (size_t)c->n_layers, V = (size_t)c->vocab_size;
    const size_t hd = D / (size_t)c->n_heads, KV = (size_t)c->n_kv_heads * hd;
    size_t o = 0;
    k->embd = o;      o += V * D;
    k->rms_att = o;   o += L * D;
    k->wq = o;        o += L * D * D;
    k->wk = o;        o += L * KV * D;
    k->wv = o;        o += L * KV * D;
    k->wo = o;        o += L * D * D;
    k->rms_ffn = o;   o += L * D;
    k->w1 = o;        o += L * H * D;
    k->w2 = o;        o += L * D * H;
    k->w3 = o;        o += L * H * D;
    k->rms_final = o; o += D;
    o += (size_t)c->seq_len * hd;  /* freq_cis_real + freq_cis_imag: seq_len x hd/2 each */
    k->wcls = c->shared_classifier ? k->embd : o;
    if (!c->shared_classifier) o += V * D;
    return o <= k->n_floats ? 0 : -1;
}

static int fill(void *user, int role, uint32_t layer, size_t rows, size_t cols, float *vals) {
    const ckpt_t *k = (const ckpt_t *)user;
    const fiber_karpathy_config_t *c = &k->c;
    const size_t D = (size_t)c->dim, H = (size_t)c->hidden_dim;
    const size_t KV = (size_t)c->n_kv_heads * (D / (size_t)c->n_heads);
    size_t src;
    switch (role) {
    case FIBER_ROLE_OUTPUT_NORM: src = k->rms_final; break;
    case FIBER_ROLE_ATTN_NORM: src = k->rms_att + layer * D; break;
    case FIBER_ROLE_FFN_NORM: src = k->rms_ffn + layer * D; break;
    case 0: src = k->wq + layer * D * D; break;
    case 1: src = k->wk + layer * KV * D; break;
    case 2: src = k->wv + layer * KV * D; break;
    case 3: src = k->wo + layer * D * D; break;
    case 4: src = k->w1 + layer * H * D; break;  /* gate */
    case 5: src = k->w2 + layer * D * H; break;  /* down */
    case 6: src = k->w3 + layer * H * D; break;  /* up */
    case 7: src = k->embd; break;
    case 8: src = k->wcls; break;
    default: return -1;
    }
    if (src + rows * cols > k->n_floats) return -1;
    memcpy(vals, k->base + src, rows * cols * sizeof(float));
    return 0;
}

int fiber_karpathy_to_gguf(const char *bin_path, const char *gguf_path) {
    int fd = open(bin_path, O_RDONLY);
    if (fd < 0) {
        fprintf(stderr, "karpathy: cannot open %s\n", bin_path);
        return -1;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || (size_t)st.st_size < 28) {
        fprintf(stderr, "karpathy: %s is too short\n", bin_path);
        close(fd);
        return -1;
    }
    void *map = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) {
        perror("karpathy: mmap");
        return -1;
    }
    ckpt_t k;
    memset(&k, 0, sizeof(k));
    int rc = parse_header((const int32_t *)map, &k.c);
    if (rc) {
        fprintf(stderr, "karpathy: %s: bad header\n", bin_path);
        munmap(map, (size_t)st.st_size);
        return -1;
    }
    k.base = (const float *)((const uint8_t *)map + 28);
    k.n_floats = ((size_t)st.st_size - 28) / sizeof(float);
    if (layout(&k) != 0) {
        fprintf(stderr, "karpathy: %s is shorter than its header says\n", bin_path);
        munmap(map, (size_t)st.st_size);
        return -1;
    }
    if (k.c.dim % 256 || k.c.hidden_dim % 256) {
        fprintf(stderr, "karpathy: dim %d / hidden_dim %d must be multiples of 256\n", k.c.dim, k.c.hidden_dim);
        munmap(map, (size_t)st.st_size);
        return -1;
    }
    fiber_synth_cfg_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.dim = (uint32_t)k.c.dim;
    cfg.n_layers = (uint32_t)k.c.n_layers;
    cfg.n_heads = (uint32_t)k.c.n_heads;
    cfg.n_kv_heads = (uint32_t)k.c.n_kv_heads;
    cfg.ffn_dim = (uint32_t)k.c.hidden_dim;
    cfg.vocab = (uint32_t)k.c.vocab_size;
    cfg.context_length = (uint32_t)k.c.seq_len;
    cfg.rope_base = 10000.0f; /* llama2.c's theta */
    cfg.eps = 1e-5f;          /* llama2.c's RMSNorm epsilon */
    cfg.recipe = FIBER_RECIPE_F16;
    cfg.tied = k.c.shared_classifier;
    rc = fiber_write_gguf_from(gguf_path, &cfg, fill, &k);
    munmap(map, (size_t)st.st_size);
    return rc;
}

model_t *model_open_karpathy(const char *bin_path, const char *gguf_path) {
    if (fiber_karpathy_to_gguf(bin_path, gguf_path) != 0) return NULL;
    return model_open(gguf_path);
}
