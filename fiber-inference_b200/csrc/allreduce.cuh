// allreduce.cuh — one-shot all-reduce (sum) of a small fp32 vector across the ranks of a
// tensor-parallel group, over peer memory (NVLink / NVSwitch), for the two exchanges of
// every layer (after Wo and after W_down).
//
// Every rank owns a slot area [2 sets][world][n_max] fp32 and a flag area [2 sets][world]
// u32 in its own HBM, mapped into every other rank's address space (CUDA IPC). One call,
// one CTA:
//   1. push: the rank's vector into slot [set][rank] of every rank (peer stores);
//   2. each thread fences its stores (system scope); thread 0 then stores, with release
//      semantics, the call's epoch into flag [set][rank] of every rank;
//   3. one thread per source rank waits (acquire) until its flag in this rank's area
//      reaches the epoch, at most AR_WAIT_NS (then error 7, no sum);
//   4. every rank adds the world slots in rank order 0, 1, ... (fp32), so all ranks hold
//      bit-identical results.
// The epoch is a device counter advanced by the kernel (CUDA-graph replays need no host
// work); the two slot sets alternate by epoch parity, so a rank may start the next call
// while a slower peer still reads the previous one (it cannot get two calls ahead: each
// call waits for every rank's flag). No multicast, no TMA: plain peer stores and loads.
#pragma once
#include "quant.cuh"

namespace fiber {

constexpr int AR_MAX_WORLD = 8;
constexpr int AR_THREADS = 1024;
constexpr unsigned long long AR_WAIT_NS = 2000000000ull;

struct ArParams {
    float *buf;                          // the vector, reduced in place
    int n, n_max, rank, world;
    float *slots[AR_MAX_WORLD];          // rank p's slot area (this rank's: local)
    unsigned int *flags[AR_MAX_WORLD];   // rank p's flag area
    unsigned int *epoch;                 // local call counter
    int *err;                            // set to 7 when a peer's flag did not arrive
};

FDEV unsigned int ar_ld_acquire(const unsigned int *p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
FDEV void ar_st_release(unsigned int *p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
FDEV unsigned long long ar_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
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
    const int set = (int)(e & 1u);
    // 1. push
    const bool vec = (n % 4) == 0 && (a.n_max % 4) == 0;
    for (int p = 0; p < W; p++) {
        float *dst = a.slots[p] + ((size_t)set * W + a.rank) * a.n_max;
        if (vec) {
            for (int i = tid; i < n / 4; i += AR_THREADS)
                reinterpret_cast<float4 *>(dst)[i] = reinterpret_cast<const float4 *>(a.buf)[i];
        } else {
            for (int i = tid; i < n; i += AR_THREADS) dst[i] = a.buf[i];
        }
    }
    // 2. publish
    __threadfence_system();
    __syncthreads();
    if (tid == 0)
        for (int p = 0; p < W; p++) ar_st_release(a.flags[p] + set * W + a.rank, e);
    // 3. wait for every source's flag in this rank's area
    if (tid < W && tid != a.rank) {
        const unsigned int *f = a.flags[a.rank] + set * W + tid;
        const unsigned long long t0 = ar_now();
        while ((int)(ar_ld_acquire(f) - e) < 0) {
            if (ar_now() - t0 > AR_WAIT_NS) {
                fail_s = 1;
                break;
            }
        }
        __threadfence_system();
    }
    __syncthreads();
    if (fail_s) {
        if (tid == 0) {
            *a.err = 7;
            *a.epoch = e;
        }
        return;
    }
    // 4. sum in rank order
    const float *base = a.slots[a.rank] + (size_t)set * W * a.n_max;
    if (vec) {
        for (int i = tid; i < n / 4; i += AR_THREADS) {
            float4 s = __ldcv(reinterpret_cast<const float4 *>(base) + i);
            for (int r = 1; r < W; r++) {
                const float4 v = __ldcv(reinterpret_cast<const float4 *>(base + (size_t)r * a.n_max) + i);
                s.x = __fadd_rn(s.x, v.x);
                s.y = __fadd_rn(s.y, v.y);
                s.z = __fadd_rn(s.z, v.z);
                s.w = __fadd_rn(s.w, v.w);
            }
            reinterpret_cast<float4 *>(a.buf)[i] = s;
        }
    } else {
        for (int i = tid; i < n; i += AR_THREADS) {
            float s = __ldcv(base + i);
            for (int r = 1; r < W; r++) s = __fadd_rn(s, __ldcv(base + (size_t)r * a.n_max + i));
            a.buf[i] = s;
        }
    }
    if (tid == 0) *a.epoch = e;
}

}  // namespace fiber
