/* model.c — open a Llama-family GGUF and resolve its tensors once.
 *
 * Hyperparameters come from the same `<arch>.*` keys with the same defaults as
 * the reference's extract_params (src/model.m:41-102): context 2048, RoPE base
 * 10000, eps 1e-5, n_kv_heads = n_heads, vocab from tokenizer.ggml.tokens (else
 * token_embd dims[1]), head_dim = dim / n_heads. Tensor names are
 * `blk.N.{attn_norm,attn_q,attn_k,attn_v,attn_output,ffn_norm,ffn_gate,ffn_down,ffn_up}.weight`
 * (src/model.m:144-177) and the classifier falls back to token_embd when
 * `output.weight` is absent (src/model.m:124-127).
 *
 * Added checks: every layer tensor must exist with the GGUF shape
 * [in, out] the decode path assumes, so a malformed model fails at load time
 * instead of in a kernel.
 */
#include "model.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static const gguf_tensor_info_t *find_layer(const gguf_file_t *gf, uint32_t l, const char *suffix) {
    char name[256];
    snprintf(name, sizeof(name), "blk.%u.%s", l, suffix);
    return gguf_find_tensor(gf, name);
}

static int extract_params(model_t *m) {
    gguf_file_t *gf = m->gf;
    model_params_t *p = &m->params;
    char key[256];

    p->arch = gguf_get_str(gf, "general.architecture");
    if (!p->arch) {
        fprintf(stderr, "model: missing general.architecture\n");
        return 0;
    }
#define ARCH_KEY(suffix) (snprintf(key, sizeof(key), "%s." suffix, p->arch), key)
    p->n_layers = gguf_get_u32(gf, ARCH_KEY("block_count"), 0);
    p->n_heads = gguf_get_u32(gf, ARCH_KEY("attention.head_count"), 0);
    p->n_kv_heads = gguf_get_u32(gf, ARCH_KEY("attention.head_count_kv"), p->n_heads);
    p->dim = gguf_get_u32(gf, ARCH_KEY("embedding_length"), 0);
    p->ffn_dim = gguf_get_u32(gf, ARCH_KEY("feed_forward_length"), 0);
    p->context_length = gguf_get_u32(gf, ARCH_KEY("context_length"), 2048);
    p->rope_freq_base = gguf_get_f32(gf, ARCH_KEY("rope.freq_base"), 10000.0f);
    p->rms_norm_eps = gguf_get_f32(gf, ARCH_KEY("attention.layer_norm_rms_epsilon"), 1e-5f);
#undef ARCH_KEY

    const gguf_kv_t *vkv = gguf_find_kv(gf, "tokenizer.ggml.tokens");
    if (vkv && vkv->type == GGUF_TYPE_ARRAY) {
        p->vocab_size = (uint32_t)vkv->value.arr.count;
    } else {
        const gguf_tensor_info_t *e = gguf_find_tensor(gf, "token_embd.weight");
        if (e && e->n_dims >= 2) p->vocab_size = (uint32_t)e->dims[1];
    }
    p->head_dim = p->n_heads ? p->dim / p->n_heads : 0;

    if (p->n_layers == 0 || p->dim == 0 || p->n_heads == 0) {
        fprintf(stderr, "model: incomplete hyperparameters (layers=%u, dim=%u, heads=%u)\n",
                p->n_layers, p->dim, p->n_heads);
        return 0;
    }
    if (p->head_dim * p->n_heads != p->dim || p->n_kv_heads == 0 ||
        p->n_heads % p->n_kv_heads != 0 || (p->head_dim & 1)) {
        fprintf(stderr, "model: inconsistent heads (dim=%u heads=%u kv_heads=%u)\n", p->dim,
                p->n_heads, p->n_kv_heads);
        return 0;
    }
    return 1;
}

static int check_shape(const gguf_tensor_info_t *ti, uint64_t in, uint64_t out, const char *what,
                       uint32_t l) {
    if (ti->n_dims < 1 || ti->dims[0] != in || (out > 1 && (ti->n_dims < 2 || ti->dims[1] != out))) {
        fprintf(stderr, "model: blk.%u.%s has shape [%llu, %llu], expected [%llu, %llu]\n", l, what,
                (unsigned long long)ti->dims[0], (unsigned long long)ti->dims[1],
                (unsigned long long)in, (unsigned long long)out);
        return 0;
    }
    return 1;
}

static int resolve_layers(model_t *m) {
    const gguf_file_t *gf = m->gf;
    const model_params_t *p = &m->params;
    uint64_t dim = p->dim, kv_dim = (uint64_t)p->n_kv_heads * p->head_dim, ffn = p->ffn_dim;
    m->layers = (layer_weights_t *)calloc(p->n_layers, sizeof(layer_weights_t));
    m->layer_off = (layer_offsets_t *)calloc(p->n_layers, sizeof(layer_offsets_t));
    if (!m->layers || !m->layer_off) return 0;

    struct {
        const char *suffix;
        uint64_t in, out;
    } spec[9] = {
        {"attn_norm.weight", dim, 1},       {"attn_q.weight", dim, dim},
        {"attn_k.weight", dim, kv_dim},     {"attn_v.weight", dim, kv_dim},
        {"attn_output.weight", dim, dim},   {"ffn_norm.weight", dim, 1},
        {"ffn_gate.weight", dim, ffn},      {"ffn_down.weight", ffn, dim},
        {"ffn_up.weight", dim, ffn},
    };
    for (uint32_t l = 0; l < p->n_layers; l++) {
        const gguf_tensor_info_t *ti[9];
        for (int k = 0; k < 9; k++) {
            ti[k] = find_layer(gf, l, spec[k].suffix);
            if (!ti[k]) {
                fprintf(stderr, "model: missing blk.%u.%s\n", l, spec[k].suffix);
                return 0;
            }
            if (!check_shape(ti[k], spec[k].in, spec[k].out, spec[k].suffix, l)) return 0;
        }
        layer_weights_t *lw = &m->layers[l];
        layer_offsets_t *lo = &m->layer_off[l];
#define SET(k, ptr_f, type_f, off_f)               \
    lw->ptr_f = gguf_tensor_data(gf, ti[k]);       \
    lw->type_f = ti[k]->type;                      \
    lo->off_f = ti[k]->offset;
        SET(0, attn_norm, attn_norm_type, attn_norm)
        SET(1, wq, wq_type, wq)
        SET(2, wk, wk_type, wk)
        SET(3, wv, wv_type, wv)
        SET(4, wo, wo_type, wo)
        SET(5, ffn_norm, ffn_norm_type, ffn_norm)
        SET(6, w1, w1_type, w1)
        SET(7, w2, w2_type, w2)
        SET(8, w3, w3_type, w3)
#undef SET
        lw->wq_size = ti[1]->size_bytes;
        lw->wk_size = ti[2]->size_bytes;
        lw->wv_size = ti[3]->size_bytes;
        lw->wo_size = ti[4]->size_bytes;
        lw->w1_size = ti[6]->size_bytes;
        lw->w2_size = ti[7]->size_bytes;
        lw->w3_size = ti[8]->size_bytes;
    }
    return 1;
}

void model_close(model_t *m) {
    if (!m) return;
    gguf_close(m->gf);
    free(m->layers);
    free(m->layer_off);
    free(m);
}

model_t *model_open(const char *path) {
    gguf_file_t *gf = gguf_open(path);
    if (!gf) return NULL;
    model_t *m = (model_t *)calloc(1, sizeof(*m));
    if (!m) {
        gguf_close(gf);
        return NULL;
    }
    m->gf = gf;
    if (!extract_params(m)) {
        model_close(m);
        return NULL;
    }
    const gguf_tensor_info_t *te = gguf_find_tensor(gf, "token_embd.weight");
    const gguf_tensor_info_t *tn = gguf_find_tensor(gf, "output_norm.weight");
    const gguf_tensor_info_t *to = gguf_find_tensor(gf, "output.weight");
    if (!te) {
        fprintf(stderr, "model: missing token_embd.weight\n");
        model_close(m);
        return NULL;
    }
    m->token_embd = gguf_tensor_data(gf, te);
    m->token_embd_type = te->type;
    m->token_embd_off = te->offset;
    if (tn) {
        m->output_norm = gguf_tensor_data(gf, tn);
        m->output_norm_type = tn->type;
        m->output_norm_off = tn->offset;
    }
    if (to) {
        m->output = gguf_tensor_data(gf, to);
        m->output_type = to->type;
        m->output_off = to->offset;
    } else {
        m->output = m->token_embd;
        m->output_type = m->token_embd_type;
        m->output_off = m->token_embd_off;
    }
    if (te->dims[0] != m->params.dim) {
        fprintf(stderr, "model: token_embd row length %llu != dim %u\n",
                (unsigned long long)te->dims[0], m->params.dim);
        model_close(m);
        return NULL;
    }
    if (!resolve_layers(m)) {
        model_close(m);
        return NULL;
    }
    return m;
}

bool model_layer_weights(const model_t *m, uint32_t layer_idx, layer_weights_t *lw) {
    memset(lw, 0, sizeof(*lw));
    if (!m || layer_idx >= m->params.n_layers || !m->layers) return false;
    *lw = m->layers[layer_idx];
    return lw->wq && lw->wk && lw->wv && lw->wo;
}

size_t model_get_rss(void) {
    FILE *f = fopen("/proc/self/statm", "r");
    if (!f) return 0;
    unsigned long pages_total = 0, pages_res = 0;
    int n = fscanf(f, "%lu %lu", &pages_total, &pages_res);
    fclose(f);
    if (n != 2) return 0;
    return (size_t)pages_res * 4096u;
}

void model_print_info(const model_t *m) {
    const model_params_t *p = &m->params;
    printf("=== Fiber-Inference Model Info ===\n");
    printf("Architecture:    %s\n", p->arch);
    printf("Layers:          %u\n", p->n_layers);
    printf("Dimension:       %u\n", p->dim);
    printf("Heads:           %u (KV: %u)\n", p->n_heads, p->n_kv_heads);
    printf("Head dim:        %u\n", p->head_dim);
    printf("FFN dim:         %u\n", p->ffn_dim);
    printf("Vocab size:      %u\n", p->vocab_size);
    printf("Context length:  %u\n", p->context_length);
    printf("RoPE freq base:  %.1f\n", p->rope_freq_base);
    printf("RMS norm eps:    %e\n", p->rms_norm_eps);
    printf("File size:       %.2f GB\n", m->gf->file_size / (1024.0 * 1024.0 * 1024.0));
    printf("Tensors:         %llu\n", (unsigned long long)m->gf->n_tensors);
    printf("Data offset:     0x%zx\n", m->gf->data_offset);
    printf("Current RSS:     %.1f MB\n", model_get_rss() / (1024.0 * 1024.0));
    printf("Embedding type:  %s\n", ggml_type_name(m->token_embd_type));
    if (m->layers) {
        const layer_weights_t *lw = &m->layers[0];
        printf("Layer 0 types:   Q=%s K=%s V=%s O=%s\n", ggml_type_name(lw->wq_type),
               ggml_type_name(lw->wk_type), ggml_type_name(lw->wv_type),
               ggml_type_name(lw->wo_type));
        printf("                 W1=%s W2=%s W3=%s\n", ggml_type_name(lw->w1_type),
               ggml_type_name(lw->w2_type), ggml_type_name(lw->w3_type));
    }
    printf("=================================\n");
}

void model_get_params(const model_t *m, model_params_t *out) {
    if (m && out) *out = m->params;
}

const gguf_file_t *model_gguf(const model_t *m) { return m ? m->gf : NULL; }
