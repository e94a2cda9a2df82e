/* tokenizer.c — SentencePiece-style BPE over the GGUF vocabulary.
 *
 * Encoding rules are those of the reference tokenizer (src/tokenizer.c:157-272):
 *  1. prefix the text with "▁" (E2 96 81) and replace every ' ' with "▁";
 *  2. split into UTF-8 characters (length from the lead byte, clipped at the
 *     end of the buffer); a character found in the vocabulary becomes that
 *     token, otherwise each of its bytes becomes the "<0xNN>" token (upper-case
 *     hex), or id 0 carrying the raw byte when that token is missing; at most
 *     8191 initial symbols;
 *  3. repeatedly merge the adjacent pair whose concatenation is a vocabulary
 *     entry with the highest score (strictly above -1e30), leftmost pair on
 *     ties, concatenations of 128 bytes or more never merging.
 * The merge loop is a max-heap of candidate pairs over a doubly linked symbol
 * list with lazy invalidation, which picks the same pair at every step as the
 * reference's full rescan.
 * Decoding maps "<0xNN>" to the byte and "▁" to ' ' (src/tokenizer.c:276-304).
 */
#include "tokenizer.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define TOK_MAX_PIECE 128
#define TOK_MAX_SYMBOLS 8192

struct tokenizer {
    int n_vocab;
    char **piece; /* NUL-terminated vocabulary strings */
    int *piece_len;
    float *score;
    int bos, eos;
    /* open-addressing table of vocabulary ids keyed by piece bytes */
    int *slot;
    uint32_t slot_mask;
};

static uint32_t hash_bytes(const char *s, int n) {
    /* 32-bit murmur-style finaliser over a running multiply-xor */
    uint32_t h = 0x9747b28cu ^ (uint32_t)n;
    for (int i = 0; i < n; i++) {
        h ^= (uint8_t)s[i];
        h *= 0x5bd1e995u;
        h ^= h >> 15;
    }
    h ^= h >> 13;
    h *= 0xc2b2ae35u;
    h ^= h >> 16;
    return h;
}

static int lookup(const tokenizer_t *t, const char *s, int n) {
    uint32_t i = hash_bytes(s, n) & t->slot_mask;
    for (;;) {
        int id = t->slot[i];
        if (id < 0) return -1;
        if (t->piece_len[id] == n && memcmp(t->piece[id], s, (size_t)n) == 0) return id;
        i = (i + 1) & t->slot_mask;
    }
}

tokenizer_t *tokenizer_init(const gguf_file_t *gf) {
    const gguf_kv_t *vk = gguf_find_kv(gf, "tokenizer.ggml.tokens");
    if (!vk || vk->type != GGUF_TYPE_ARRAY || vk->value.arr.elem_type != GGUF_TYPE_STRING) {
        fprintf(stderr, "tokenizer: missing tokenizer.ggml.tokens\n");
        return NULL;
    }
    const gguf_kv_t *sk = gguf_find_kv(gf, "tokenizer.ggml.scores");
    const float *raw_scores = NULL;
    if (sk && sk->type == GGUF_TYPE_ARRAY && sk->value.arr.elem_type == GGUF_TYPE_FLOAT32 &&
        sk->value.arr.count >= vk->value.arr.count)
        raw_scores = (const float *)sk->value.arr.data;

    int n = (int)vk->value.arr.count;
    tokenizer_t *t = (tokenizer_t *)calloc(1, sizeof(*t));
    if (!t) return NULL;
    t->n_vocab = n;
    t->piece = (char **)calloc((size_t)n, sizeof(char *));
    t->piece_len = (int *)calloc((size_t)n, sizeof(int));
    t->score = (float *)calloc((size_t)n, sizeof(float));
    uint32_t cap = 16;
    while (cap < (uint32_t)n * 4u) cap <<= 1;
    t->slot = (int *)malloc(cap * sizeof(int));
    t->slot_mask = cap - 1;
    if (!t->piece || !t->piece_len || !t->score || !t->slot) {
        tokenizer_free(t);
        return NULL;
    }
    for (uint32_t i = 0; i < cap; i++) t->slot[i] = -1;

    const uint8_t *p = (const uint8_t *)vk->value.arr.data;
    for (int id = 0; id < n; id++) {
        uint64_t len;
        memcpy(&len, p, 8);
        p += 8;
        t->piece[id] = (char *)malloc((size_t)len + 1);
        if (!t->piece[id]) {
            tokenizer_free(t);
            return NULL;
        }
        memcpy(t->piece[id], p, (size_t)len);
        t->piece[id][len] = '\0';
        t->piece_len[id] = (int)len;
        p += len;
        float sc = 0.0f;
        if (raw_scores) memcpy(&sc, (const uint8_t *)raw_scores + 4 * (size_t)id, 4);
        t->score[id] = sc;
        /* first occurrence of a duplicated piece keeps the slot, like the
         * reference's insert-then-probe lookup */
        uint32_t h = hash_bytes(t->piece[id], (int)len) & t->slot_mask;
        int dup = 0;
        while (t->slot[h] >= 0) {
            int o = t->slot[h];
            if (t->piece_len[o] == (int)len && memcmp(t->piece[o], t->piece[id], (size_t)len) == 0) {
                dup = 1;
                break;
            }
            h = (h + 1) & t->slot_mask;
        }
        if (!dup) t->slot[h] = id;
    }
    t->bos = (int)gguf_get_u32(gf, "tokenizer.ggml.bos_token_id", 1);
    t->eos = (int)gguf_get_u32(gf, "tokenizer.ggml.eos_token_id", 2);
    printf("Tokenizer: %d tokens, BOS=%d, EOS=%d\n", n, t->bos, t->eos);
    return t;
}

void tokenizer_free(tokenizer_t *t) {
    if (!t) return;
    if (t->piece)
        for (int i = 0; i < t->n_vocab; i++) free(t->piece[i]);
    free(t->piece);
    free(t->piece_len);
    free(t->score);
    free(t->slot);
    free(t);
}

/* ---- encoder ---------------------------------------------------------------- */

typedef struct {
    int id;
    int len;
    int prev, next; /* -1 at the ends */
    int version;    /* bumped whenever the symbol changes or dies */
    int alive;
    char text[TOK_MAX_PIECE];
} sym_t;

typedef struct {
    float score;
    int left;  /* symbol index; symbols are created in text order */
    int right;
    int id;
    int vl, vr;
} cand_t;

/* max-heap order: higher score first, then the leftmost pair */
static int cand_before(const cand_t *a, const cand_t *b) {
    if (a->score != b->score) return a->score > b->score;
    return a->left < b->left;
}

typedef struct {
    cand_t *v;
    int n, cap;
} heap_t;

static int heap_push(heap_t *h, cand_t c) {
    if (h->n == h->cap) {
        int nc = h->cap ? h->cap * 2 : 64;
        cand_t *nv = (cand_t *)realloc(h->v, (size_t)nc * sizeof(cand_t));
        if (!nv) return 0;
        h->v = nv;
        h->cap = nc;
    }
    int i = h->n++;
    h->v[i] = c;
    while (i > 0) {
        int p = (i - 1) / 2;
        if (!cand_before(&h->v[i], &h->v[p])) break;
        cand_t tmp = h->v[i];
        h->v[i] = h->v[p];
        h->v[p] = tmp;
        i = p;
    }
    return 1;
}

static cand_t heap_pop(heap_t *h) {
    cand_t top = h->v[0];
    h->v[0] = h->v[--h->n];
    int i = 0;
    for (;;) {
        int l = 2 * i + 1, r = l + 1, m = i;
        if (l < h->n && cand_before(&h->v[l], &h->v[m])) m = l;
        if (r < h->n && cand_before(&h->v[r], &h->v[m])) m = r;
        if (m == i) break;
        cand_t tmp = h->v[i];
        h->v[i] = h->v[m];
        h->v[m] = tmp;
        i = m;
    }
    return top;
}

static void offer_pair(const tokenizer_t *t, const sym_t *s, int a, int b, heap_t *h) {
    if (a < 0 || b < 0) return;
    int ml = s[a].len + s[b].len;
    if (ml >= TOK_MAX_PIECE) return;
    char buf[TOK_MAX_PIECE];
    memcpy(buf, s[a].text, (size_t)s[a].len);
    memcpy(buf + s[a].len, s[b].text, (size_t)s[b].len);
    int id = lookup(t, buf, ml);
    if (id < 0 || !(t->score[id] > -1e30f)) return;
    cand_t c = {t->score[id], a, b, id, s[a].version, s[b].version};
    heap_push(h, c);
}

static int utf8_width(uint8_t lead) {
    if ((lead & 0x80) == 0) return 1;
    if ((lead & 0xE0) == 0xC0) return 2;
    if ((lead & 0xF0) == 0xE0) return 3;
    if ((lead & 0xF8) == 0xF0) return 4;
    return 1;
}

int tokenizer_encode(const tokenizer_t *t, const char *text, int *tokens, int max_tokens) {
    if (!text || !text[0]) return 0;
    size_t tl = strlen(text);
    char *buf = (char *)malloc(tl * 3 + 4);
    sym_t *s = (sym_t *)malloc(TOK_MAX_SYMBOLS * sizeof(sym_t));
    if (!buf || !s) {
        free(buf);
        free(s);
        return 0;
    }
    size_t bl = 0;
    static const char space_mark[3] = {(char)0xE2, (char)0x96, (char)0x81};
    memcpy(buf, space_mark, 3);
    bl = 3;
    for (size_t i = 0; i < tl; i++) {
        if (text[i] == ' ') {
            memcpy(buf + bl, space_mark, 3);
            bl += 3;
        } else {
            buf[bl++] = text[i];
        }
    }

    int n = 0;
    for (size_t i = 0; i < bl && n < TOK_MAX_SYMBOLS - 1;) {
        int w = utf8_width((uint8_t)buf[i]);
        if (i + (size_t)w > bl) w = 1;
        int id = lookup(t, buf + i, w);
        if (id >= 0) {
            s[n].id = id;
            s[n].len = w;
            memcpy(s[n].text, buf + i, (size_t)w);
            n++;
        } else {
            for (int b = 0; b < w && n < TOK_MAX_SYMBOLS - 1; b++) {
                char hex[8];
                snprintf(hex, sizeof(hex), "<0x%02X>", (uint8_t)buf[i + b]);
                int bid = lookup(t, hex, 6);
                if (bid >= 0) {
                    s[n].id = bid;
                    s[n].len = 6;
                    memcpy(s[n].text, hex, 6);
                } else {
                    s[n].id = 0;
                    s[n].len = 1;
                    s[n].text[0] = buf[i + b];
                }
                n++;
            }
        }
        i += (size_t)w;
    }
    free(buf);
    for (int i = 0; i < n; i++) {
        s[i].prev = i - 1;
        s[i].next = i + 1 < n ? i + 1 : -1;
        s[i].version = 0;
        s[i].alive = 1;
    }

    heap_t h = {NULL, 0, 0};
    for (int i = 0; i + 1 < n; i++) offer_pair(t, s, i, i + 1, &h);
    while (h.n > 0) {
        cand_t c = heap_pop(&h);
        sym_t *a = &s[c.left], *b = &s[c.right];
        if (!a->alive || !b->alive || a->next != c.right || a->version != c.vl ||
            b->version != c.vr)
            continue;
        memcpy(a->text + a->len, b->text, (size_t)b->len);
        a->len += b->len;
        a->id = c.id;
        a->version++;
        b->alive = 0;
        b->version++;
        a->next = b->next;
        if (b->next >= 0) s[b->next].prev = c.left;
        offer_pair(t, s, a->prev, c.left, &h);
        offer_pair(t, s, c.left, a->next, &h);
    }
    free(h.v);

    int out = 0;
    for (int i = 0; i >= 0 && n > 0 && out < max_tokens; i = s[i].next) tokens[out++] = s[i].id;
    free(s);
    return out;
}

const char *tokenizer_decode(const tokenizer_t *t, int token_id) {
    static __thread char out[512];
    if (token_id < 0 || token_id >= t->n_vocab) return "";
    const char *p = t->piece[token_id];
    int n = t->piece_len[token_id];
    if (n == 6 && p[0] == '<' && p[1] == '0' && p[2] == 'x' && p[5] == '>') {
        out[0] = (char)strtol(p + 3, NULL, 16);
        out[1] = '\0';
        return out;
    }
    int j = 0;
    for (int i = 0; i < n && j < 510;) {
        if (i + 2 < n && (uint8_t)p[i] == 0xE2 && (uint8_t)p[i + 1] == 0x96 &&
            (uint8_t)p[i + 2] == 0x81) {
            out[j++] = ' ';
            i += 3;
        } else {
            out[j++] = p[i++];
        }
    }
    out[j] = '\0';
    return out;
}

int tokenizer_bos(const tokenizer_t *t) { return t->bos; }
int tokenizer_eos(const tokenizer_t *t) { return t->eos; }
int tokenizer_vocab_size(const tokenizer_t *t) { return t->n_vocab; }
