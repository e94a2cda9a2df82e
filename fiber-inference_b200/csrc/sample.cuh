// sample.cuh — temperature / top-k / top-p sampling on the device, one CTA per logits row,
// with the reference sampler's exact procedure (src/sampler.c:48-112):
//   v_i = logit_i * (1 / T)                                  (multiply by the reciprocal)
//   k < n: candidates sorted by v descending, equal values in index order (qsort with a
//          stable merge sort, as glibc's); k == n: candidates left in index order
//   e_i = exp(v_i - v_first) for the first k candidates, total = e_0 + e_1 + ... (fp32,
//          in candidate order), p_i = e_i / total
//   top_p < 1: the first candidates whose running fp32 sum reaches top_p are kept and
//          renormalised the same way
//   r = xorshift64* draw (state per row); the first candidate whose running sum of p
//          reaches r is the token (candidate 0 when none does)
// Sums run on one thread in the reference's order (fp32 addition is not associative); the
// exponentials and divisions, which do not depend on order, run on all threads. exp is
// CUDA's expf: the probabilities can differ from the host's libm expf by an ulp, so a
// draw that lands within an ulp of a boundary can pick the neighbouring candidate.
//
// Top-k selection: 64-bit keys (value ordered descending, then index ascending) and an
// MSB-first radix select (8 passes of 8 bits) find the k-th key; the k keys at or above
// it are gathered and sorted with a bitonic sort in shared memory.
#pragma once
#include "quant.cuh"

namespace fiber {

constexpr int SMP_THREADS = 1024;
constexpr int SMP_MAX_K = 1024;         // top_k < vocab handled up to this k
constexpr int SMP_MAX_UNSORTED = 49152;  // vocab limit of the k == vocab (unsorted) case

struct SampleParams {
    const float *logits;  // [rows][ld]
    int ld, vocab, rows;
    float inv_temp;       // 1 / temperature (computed on the host as the reference does)
    int k;                // min(top_k, vocab); top_k <= 0 means vocab
    float top_p;
    unsigned long long *rng;  // [rows] xorshift64* states
    int32_t *out;             // [rows] sampled tokens
    // device-resident decode loop (optional): token / position advance and record
    int32_t *adv_token, *adv_pos;  // next step's token and position (single sequence)
    int32_t *rec;                  // [steps] recorded tokens
    int32_t *rec_step;             // step counter (incremented here)
};

// float -> order-preserving uint32 (ascending); -0 is taken as +0 (the qsort comparator
// treats them as equal)
FDEV uint32_t smp_ord(float v) {
    uint32_t b = __float_as_uint(v);
    if (b == 0x80000000u) b = 0;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
FDEV float smp_unord(uint32_t o) { return __uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o); }
FDEV unsigned long long smp_key(float v, int i) {
    return ((unsigned long long)smp_ord(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)i);
}

FDEV float smp_draw(unsigned long long *st) {  // the reference's rng_float
    unsigned long long x = *st;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *st = x;
    return (float)((x * 0x2545F4914F6CDD1DULL) >> 40) / (float)(1 << 24);
}

// Dynamic shared memory: k < vocab: SMP_MAX_K keys (8 B) + SMP_MAX_K floats;
// k == vocab: vocab floats.
__global__ void __launch_bounds__(SMP_THREADS) sample_rows_kernel(const SampleParams p) {
    extern __shared__ __align__(16) uint8_t smp_smem[];
    __shared__ unsigned int hist[256];
    __shared__ unsigned long long prefix_s;
    __shared__ int remain_s, count_s, keep_s, pick_s;
    __shared__ float total_s;
    const int row = blockIdx.x, tid = threadIdx.x, n = p.vocab;
    const float *lg = p.logits + (size_t)row * p.ld;
    const int k = p.k;
    float *val;  // candidate values, then probabilities, in candidate order
    int cand;
    unsigned long long *keys = reinterpret_cast<unsigned long long *>(smp_smem);
    if (k < n) {
        // ---- radix select of the k-th largest key, MSB first
        unsigned long long prefix = 0, mask = 0;
        int remain = k;
        for (int shift = 56; shift >= 0; shift -= 8) {
            for (int b = tid; b < 256; b += SMP_THREADS) hist[b] = 0;
            __syncthreads();
            for (int i = tid; i < n; i += SMP_THREADS) {
                const unsigned long long key = smp_key(lg[i] * p.inv_temp, i);
                if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xFF], 1u);
            }
            __syncthreads();
            if (tid == 0) {
                int d = 255;
                while (d > 0 && (int)hist[d] < remain) remain -= (int)hist[d--];
                prefix_s = prefix | ((unsigned long long)d << shift);
                remain_s = remain;
            }
            __syncthreads();
            prefix = prefix_s;
            remain = remain_s;
            mask |= 0xFFull << shift;
        }
        // prefix is now the k-th largest key (keys are unique): gather the keys >= it
        if (tid == 0) count_s = 0;
        __syncthreads();
        for (int i = tid; i < n; i += SMP_THREADS) {
            const unsigned long long key = smp_key(lg[i] * p.inv_temp, i);
            if (key >= prefix) keys[atomicAdd(&count_s, 1)] = key;
        }
        __syncthreads();
        int np2 = 1;
        while (np2 < k) np2 <<= 1;
        for (int i = k + tid; i < np2; i += SMP_THREADS) keys[i] = 0;  // below every real key
        __syncthreads();
        // bitonic sort, descending
        for (int size = 2; size <= np2; size <<= 1)
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                for (int i = tid; i < np2; i += SMP_THREADS) {
                    const int j = i ^ stride;
                    if (j > i) {
                        const bool desc = (i & size) == 0;
                        const unsigned long long a = keys[i], b = keys[j];
                        if (desc ? (a < b) : (a > b)) {
                            keys[i] = b;
                            keys[j] = a;
                        }
                    }
                }
                __syncthreads();
            }
        val = reinterpret_cast<float *>(smp_smem + (size_t)SMP_MAX_K * 8);
        for (int i = tid; i < k; i += SMP_THREADS) val[i] = smp_unord((uint32_t)(keys[i] >> 32));
        cand = k;
    } else {
        val = reinterpret_cast<float *>(smp_smem);
        for (int i = tid; i < n; i += SMP_THREADS) val[i] = lg[i] * p.inv_temp;
        cand = n;
    }
    __syncthreads();
    // ---- softmax over the candidates, shifted by the first one's value
    const float shift = val[0];
    __syncthreads();
    for (int i = tid; i < cand; i += SMP_THREADS) val[i] = expf(val[i] - shift);
    __syncthreads();
    if (tid == 0) {
        float t = 0.0f;
        for (int i = 0; i < cand; i++) t += val[i];
        total_s = t;
    }
    __syncthreads();
    {
        const float t = total_s;
        for (int i = tid; i < cand; i += SMP_THREADS) val[i] /= t;
    }
    __syncthreads();
    // ---- nucleus truncation
    if (tid == 0) {
        int keep = cand;
        if (p.top_p < 1.0f) {
            float acc = 0.0f;
            for (int i = 0; i < cand; i++) {
                acc += val[i];
                if (acc >= p.top_p) {
                    keep = i + 1;
                    break;
                }
            }
            float t = 0.0f;
            for (int i = 0; i < keep; i++) t += val[i];
            total_s = t;
        }
        keep_s = keep;
    }
    __syncthreads();
    if (p.top_p < 1.0f) {
        const float t = total_s;
        for (int i = tid; i < keep_s; i += SMP_THREADS) val[i] /= t;
        __syncthreads();
    }
    // ---- the draw
    if (tid == 0) {
        const int keep = keep_s;
        unsigned long long st = p.rng[row];
        const float r = smp_draw(&st);
        p.rng[row] = st;
        float acc = 0.0f;
        int pick = 0;
        for (int i = 0; i < keep; i++) {
            acc += val[i];
            if (r <= acc) {
                pick = i;
                break;
            }
        }
        pick_s = pick;
    }
    __syncthreads();
    if (tid == 0) {
        const int pick = pick_s;
        const int32_t token = k < n ? (int32_t)(0xFFFFFFFFu - (uint32_t)(keys[pick] & 0xFFFFFFFFull)) : pick;
        p.out[row] = token;
        if (p.adv_token) {  // single-sequence device loop
            *p.adv_token = token;
            *p.adv_pos += 1;
            const int s = *p.rec_step;
            p.rec[s] = token;
            *p.rec_step = s + 1;
        }
    }
}

}  // namespace fiber
