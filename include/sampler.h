/* sampler.h — temperature / top-k / top-p sampling over fp32 logits (host side).
 *
 * Same entry points, defaults and random stream as the reference sampler
 * (src/sampler.h:15-18, src/sampler.c:10-112): greedy argmax (first maximum wins)
 * when temperature <= 0, otherwise temperature scaling, descending sort, softmax
 * over the top k, nucleus truncation at top_p and an xorshift64* draw seeded
 * with 42. The greedy case is also computed on the device, fused with the
 * lm_head (see fiber_cuda.h), so the decode loop never copies logits back.
 */
#ifndef FIBER_SAMPLER_H
#define FIBER_SAMPLER_H

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int vocab_size;
    float temperature;
    int top_k;
    float top_p;
    unsigned long long rng_state;
} sampler_t;

void sampler_init(sampler_t *s, int vocab_size, float temp, int top_k, float top_p);
int sampler_sample(sampler_t *s, const float *logits);

#ifdef __cplusplus
}
#endif
#endif
