/* sampler.c — host sampler; algorithm and random stream of the reference
 * sampler (src/sampler.c:10-112). The scored-pair layout and the qsort
 * comparator's ordering are kept because the order qsort leaves equal logits
 * in depends on both, and the sampled id must match the reference's.
 */
#include "sampler.h"

#include <math.h>
#include <stdlib.h>

/* xorshift64* step, 24-bit mantissa draw in [0, 1) (src/sampler.c:10-15). */
static float draw_uniform(unsigned long long *st) {
    unsigned long long x = *st;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *st = x;
    return (float)((x * 0x2545F4914F6CDD1DULL) >> 40) / (float)(1 << 24);
}

void sampler_init(sampler_t *s, int vocab_size, float temp, int top_k, float top_p) {
    s->vocab_size = vocab_size;
    s->temperature = temp;
    s->top_k = top_k > 0 ? top_k : vocab_size;
    s->top_p = top_p;
    s->rng_state = 42;
}

typedef struct {
    float val;
    int idx;
} cand_t;

static int by_val_desc(const void *pa, const void *pb) {
    float a = ((const cand_t *)pa)->val, b = ((const cand_t *)pb)->val;
    return (a < b) - (a > b);
}

int sampler_sample(sampler_t *s, const float *logits) {
    const int n = s->vocab_size;
    const float temp = s->temperature;
    if (temp <= 0.0f || temp < 1e-6f) {
        int best = 0;
        for (int i = 1; i < n; i++)
            if (logits[i] > logits[best]) best = i;
        return best;
    }
    cand_t *c = (cand_t *)malloc((size_t)n * sizeof(cand_t));
    if (!c) return 0;
    const float inv_t = 1.0f / temp;
    for (int i = 0; i < n; i++) {
        c[i].val = logits[i] * inv_t;
        c[i].idx = i;
    }
    const int k = s->top_k < n ? s->top_k : n;
    if (k < n) qsort(c, (size_t)n, sizeof(cand_t), by_val_desc);

    /* Softmax over the first k candidates, shifted by the first one's value
     * (the true maximum whenever the list was sorted). */
    const float shift = c[0].val;
    float total = 0.0f;
    for (int i = 0; i < k; i++) {
        c[i].val = expf(c[i].val - shift);
        total += c[i].val;
    }
    for (int i = 0; i < k; i++) c[i].val /= total;

    int keep = k;
    if (s->top_p < 1.0f) {
        float acc = 0.0f;
        for (int i = 0; i < k; i++) {
            acc += c[i].val;
            if (acc >= s->top_p) {
                keep = i + 1;
                break;
            }
        }
        total = 0.0f;
        for (int i = 0; i < keep; i++) total += c[i].val;
        for (int i = 0; i < keep; i++) c[i].val /= total;
    }

    const float r = draw_uniform(&s->rng_state);
    float acc = 0.0f;
    int pick = c[0].idx;
    for (int i = 0; i < keep; i++) {
        acc += c[i].val;
        if (r <= acc) {
            pick = c[i].idx;
            break;
        }
    }
    free(c);
    return pick;
}
