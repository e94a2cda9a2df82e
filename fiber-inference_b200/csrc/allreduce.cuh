// allreduce.cuh — one-shot all-reduce (sum) of a small fp32 vector across the ranks of a
// tensor-parallel group, over peer memory (NVLink / NVSwitch), for the two exchanges of
// every layer (after Wo and after W_down).
//
// Every rank owns a slot area [2 sets][world][n_max] of 8-byte words in its own HBM,
// mapped into every other rank's address space (CUDA IPC). A word carries one value and
// the call's epoch (low half: the fp32 bits, high half: the epoch), stored with one
// 8-byte store, which a reader sees whole: a word whose epoch is the current call's
// holds this call's value, so no fence and no separate flag are needed. One call, one CTA:
//   1. push: word (epoch, x[i]) into slot [set][rank][i] of every other rank (peer stores);
//   2. read: for each source rank, poll slot [set][source][i] in this rank's area until
//      its epoch is the call's (at most AR_WAIT_NS, then error 7, no sum);
//   3. sum in rank order 0, 1, ... (fp32; this rank's own term from x), so all ranks hold
//      bit-identical results.
// The epoch is a device counter advanced by the kernel (CUDA-graph replays need no host
// work); the two slot sets alternate by epoch parity, so a rank may start the next call
// while a slower peer still reads the previous one (it cannot get two calls ahead: each
// call needs every rank's words). No multicast, no TMA: plain peer stores and local loads.
#pragma once
#include "quant.cuh"

namespace fiber {

constexpr int AR_MAX_WORLD = 8;
constexpr int AR_THREADS = 1024;
constexpr unsigned long long AR_WAIT_NS = 2000000000ull;

struct ArParams {
    float *buf;                                 // the vector, reduced in place
    int n, n_max, rank, world;
    unsigned long long *slots[AR_MAX_WORLD];    // rank p's slot area (this rank's: local)
    unsigned int *epoch;                        // local call counter
    int *err;                                   // set to 7 when a peer's data did not arrive
};

FDEV unsigned long long ar_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
FDEV void ar_st(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
FDEV unsigned long long ar_ld(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(AR_THREADS) ar_oneshot_kernel(const ArParams a) {
    __shared__ unsigned int epoch_s;
    __shared__ int fail_s;
    const int tid = threadIdx.x, W = a.world, n = a.n;
    if (tid == 0) {
        epoch_s = *a.epoch + 1u;
        fail_s = 0;
    }
    __syncthreads();
    const unsigned int e = epoch_s;
    const size_t set = e & 1u;
    const unsigned long long tag = (unsigned long long)e << 32;
    // 1. push to every other rank
    for (int i = tid; i < n; i += AR_THREADS) {
        const unsigned long long w = tag | __float_as_uint(a.buf[i]);
        for (int p = 0; p < W; p++)
            if (p != a.rank) ar_st(a.slots[p] + (set * W + a.rank) * a.n_max + i, w);
    }
    // 2 + 3. read each source's words (bounded) and sum in rank order
    const unsigned long long *mine = a.slots[a.rank] + set * W * a.n_max;
    const unsigned long long t0 = ar_now();
    bool ok = true;
    for (int i = tid; i < n && ok; i += AR_THREADS) {
        float s = 0.f;
        for (int r = 0; r < W && ok; r++) {
            float v;
            if (r == a.rank) {
                v = a.buf[i];
            } else {
                const unsigned long long *src = mine + (size_t)r * a.n_max + i;
                unsigned long long w = ar_ld(src);
                int spins = 0;
                while ((unsigned int)(w >> 32) != e) {
                    if ((++spins & 255) == 0 && (*(volatile int *)&fail_s || ar_now() - t0 > AR_WAIT_NS)) {
                        ok = false;
                        break;
                    }
                    w = ar_ld(src);
                }
                v = __uint_as_float((unsigned int)w);
            }
            s = r == 0 ? v : __fadd_rn(s, v);
        }
        if (ok) a.buf[i] = s;  // only element i: its own term was read above
    }
    if (!ok) *(volatile int *)&fail_s = 1;
    __syncthreads();
    if (tid == 0) {
        if (fail_s) *a.err = 7;
        *a.epoch = e;
    }
}

}  // namespace fiber
