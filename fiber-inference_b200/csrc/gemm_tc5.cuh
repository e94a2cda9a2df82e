// gemm_tc5.cuh — dequant-GEMM for batched prefill on the 5th-generation tensor cores.
//
// Y[t][out_off + r] (op)= sum_k W[r][k] * xn[t][k] for a GGUF weight matrix W (Q4_K,
// Q6_K or F16 super-blocks, rows x cols) and ntok input rows x (fp32, optionally
// RMS-normalised per token: xn = x * rrms[t] * nw[k]).
//
// One CTA computes a 128-row x 64-token tile with tcgen05.mma (kind::f16, M=128,
// N=128, fp32 accumulators in tensor memory):
//   * A = the weights, decoded exactly to fp16 (the reference dequantizer's
//     arithmetic, quant.cuh) into shared memory in the canonical no-swizzle K-major
//     layout (8x16-byte core matrices: rows 16 B apart, K halves 128 B apart, row
//     groups 2048 B apart), 128 K columns per chunk, double buffered;
//   * B = the inputs split into fp16 hi and lo parts (x = hi + lo to ~22 bits) as
//     two B rows per token (n = 2t: hi, n = 2t+1: lo), same layout;
//   * one thread issues the 8 MMAs of a chunk (K = 16 each) and commits them to the
//     chunk buffer's mbarrier; the other threads decode / stage the next chunk;
//   * epilogue: warps 0..3 read their 32 accumulator lanes (rows) with tcgen05.ld,
//     add each token's hi and lo columns and store (or add to) Y.
// Every wait is bounded (%globaltimer); on timeout the CTA records an error,
// waits (bounded) for its committed MMAs, frees its tensor memory and returns.
#pragma once
#include "quant.cuh"

namespace fiber {

constexpr int G5_M = 128;        // weight rows per CTA (MMA M)
constexpr int G5_T = 64;         // tokens per CTA (MMA N = 2 * G5_T)
constexpr int G5_N = 2 * G5_T;
constexpr int G5_KC = 128;       // K per chunk (8 MMAs)
constexpr int G5_THREADS = 256;
constexpr int G5_A_BYTES = G5_M * G5_KC * 2;  // 32 KB
constexpr int G5_B_BYTES = G5_N * G5_KC * 2;  // 32 KB
constexpr unsigned long long G5_WAIT_NS = 2000000000ull;

enum : int { G5_STORE = 0, G5_RESID = 1 };

struct G5Params {
    const uint8_t *w;      // weights, rows x cols in GGUF super-blocks
    int type;              // T_Q4_K / T_Q6_K / T_F16
    int rows, cols, ntok;
    const float *x;        // [ntok][ldx]
    int ldx;
    const float *rrms;     // [ntok] or null
    const float *nw;       // [cols] or null
    float *y;              // [ntok][ldy]
    int ldy, out_off;
    int epi;               // G5_STORE: y = acc; G5_RESID: y += acc
    int *err;              // set to 6 when a wait gave up
};

FDEV uint64_t g5_desc(uint32_t saddr) {
    // SWIZZLE_NONE K-major: start >> 4, LBO = 128 B (next K half), SBO = 2048 B
    // (next 8-row group), version 1 (bits 46-47)
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(2048 >> 4) << 32) |
           (1ull << 46);
}

// kind::f16 instruction descriptor: D f32, A and B f16, both K-major, N, M
constexpr uint32_t g5_idesc() {
    return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(G5_N >> 3) << 17) | ((uint32_t)(G5_M >> 4) << 24);
}

FDEV uint32_t g5_saddr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
FDEV unsigned long long g5_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
FDEV bool g5_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(g5_saddr(bar)), "r"(parity), "r"(20000u)
        : "memory");
    return ok != 0;
}
FDEV bool g5_wait(uint64_t *bar, uint32_t parity) {
    const unsigned long long t0 = g5_now();
    while (!g5_try_wait(bar, parity))
        if (g5_now() - t0 > G5_WAIT_NS) return false;
    return true;
}

// canonical offset of (row r, k) inside a 128-K chunk tile: core matrix (r/8, k/8)
FDEV int g5_off(int r, int k) { return ((r >> 3) * (G5_KC / 8) + (k >> 3)) * 128 + (r & 7) * 16 + (k & 7) * 2; }

FDEV uint32_t g5_pack(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Decode half `half` (elements 128*half .. +127) of the super-block `blk` of weight row
// r into A; this thread handles elements [64*sub, 64*sub + 64) of that half.
template <int T>
FDEV void g5_decode(const uint8_t *blk, int half, int sub, int r, uint8_t *A);

template <>
FDEV void g5_decode<T_Q4_K>(const uint8_t *blk, int half, int sub, int r, uint8_t *A) {
    const uint16_t *h = reinterpret_cast<const uint16_t *>(blk);
    const float d = h2f(h[0]), dmin = h2f(h[1]);
    uint32_t s[3];
    for (int i = 0; i < 3; i++)
        s[i] = (uint32_t)blk[4 + 4 * i] | ((uint32_t)blk[5 + 4 * i] << 8) | ((uint32_t)blk[6 + 4 * i] << 16) |
               ((uint32_t)blk[7 + 4 * i] << 24);
    const int g = 2 * half + sub;  // 64-element group: sub-blocks 2g (low nibbles), 2g+1 (high)
    int sc0, m0, sc1, m1;
    scale_min_k4(2 * g, s[0], s[1], s[2], sc0, m0);
    scale_min_k4(2 * g + 1, s[0], s[1], s[2], sc1, m1);
    const float dsc0 = __fmul_rn(d, (float)sc0), dmm0 = __fmul_rn(dmin, (float)m0);
    const float dsc1 = __fmul_rn(d, (float)sc1), dmm1 = __fmul_rn(dmin, (float)m1);
    const uint8_t *q = blk + 16 + 32 * g;
    for (int l0 = 0; l0 < 32; l0 += 8) {
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int a = q[l0 + 2 * j], b = q[l0 + 2 * j + 1];
            lo[j] = g5_pack(q4k_weight(dsc0, dmm0, a & 15), q4k_weight(dsc0, dmm0, b & 15));
            hi[j] = g5_pack(q4k_weight(dsc1, dmm1, a >> 4), q4k_weight(dsc1, dmm1, b >> 4));
        }
        const int k = 64 * sub + l0;
        *reinterpret_cast<uint4 *>(A + g5_off(r, k)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<uint4 *>(A + g5_off(r, k + 32)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    }
}

template <>
FDEV void g5_decode<T_Q6_K>(const uint8_t *blk, int half, int sub, int r, uint8_t *A) {
    // the Q6_K super-block is two independent 128-element halves: chunk half = block half
    for (int k0 = 64 * sub; k0 < 64 * sub + 64; k0 += 8) {
        uint32_t v[4];
#pragma unroll
        for (int j = 0; j < 4; j++)
            v[j] = g5_pack(decode_elem<T_Q6_K>(blk, 128 * half + k0 + 2 * j),
                           decode_elem<T_Q6_K>(blk, 128 * half + k0 + 2 * j + 1));
        *reinterpret_cast<uint4 *>(A + g5_off(r, k0)) = make_uint4(v[0], v[1], v[2], v[3]);
    }
}

template <>
FDEV void g5_decode<T_F16>(const uint8_t *blk, int half, int sub, int r, uint8_t *A) {
    const uint16_t *e = reinterpret_cast<const uint16_t *>(blk) + 128 * half + 64 * sub;
    for (int k0 = 0; k0 < 64; k0 += 8) {
        uint32_t v[4];
#pragma unroll
        for (int j = 0; j < 4; j++) v[j] = (uint32_t)e[k0 + 2 * j] | ((uint32_t)e[k0 + 2 * j + 1] << 16);
        *reinterpret_cast<uint4 *>(A + g5_off(r, 64 * sub + k0)) = make_uint4(v[0], v[1], v[2], v[3]);
    }
}

template <int T>
__global__ void __launch_bounds__(G5_THREADS, 1) gemm_tc5_kernel(const G5Params p) {
    extern __shared__ __align__(1024) uint8_t g5_smem[];
    __shared__ __align__(8) uint64_t done[2];
    __shared__ uint32_t tmem_slot;
    __shared__ int fail;
    constexpr int BB = T == T_Q4_K ? 144 : (T == T_Q6_K ? 210 : 512);
    uint8_t *A[2] = {g5_smem, g5_smem + G5_A_BYTES};
    uint8_t *B[2] = {g5_smem + 2 * G5_A_BYTES, g5_smem + 2 * G5_A_BYTES + G5_B_BYTES};
    uint8_t *raw = g5_smem + 2 * G5_A_BYTES + 2 * G5_B_BYTES;  // [128 rows][one super-block]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row0 = blockIdx.x * G5_M, tok0 = blockIdx.y * G5_T;
    const int nb = p.cols / 256, nchunk = p.cols / G5_KC;
    const size_t row_bytes = (size_t)nb * BB;

    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(g5_saddr(&done[0])) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(g5_saddr(&done[1])) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fail = 0;
    }
    if (warp == 0) {  // 128 fp32 accumulator columns x 128 lanes
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(g5_saddr(&tmem_slot)),
                     "r"(G5_N)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_slot;

    int issued = 0;  // chunks whose MMAs were committed
    for (int c = 0; c < nchunk; c++) {
        const int buf = c & 1;
        if (c >= 2) {  // the MMAs of chunk c - 2 have read this buffer
            if (tid == 0 && !g5_wait(&done[buf], (uint32_t)(((c - 2) >> 1) & 1))) fail = 1;
            __syncthreads();
            if (fail) break;
        }
        if ((c & 1) == 0 || G5_KC == 256) {  // raw super-block column c*128/256 of the 128 rows
            const int b = c * G5_KC / 256;
            __syncthreads();  // previous raw block fully decoded
            for (int i = tid; i < G5_M * BB / 2; i += G5_THREADS) {
                const int r = i / (BB / 2), o = i % (BB / 2);
                uint16_t v = 0;
                if (row0 + r < p.rows)
                    v = reinterpret_cast<const uint16_t *>(p.w + (size_t)(row0 + r) * row_bytes + (size_t)b * BB)[o];
                reinterpret_cast<uint16_t *>(raw + r * BB)[o] = v;
            }
            __syncthreads();
        }
        // A: decode this chunk's half of the super-block for the 128 rows
        {
            const int r = tid >> 1, sub = tid & 1, half = c & 1;
            g5_decode<T>(raw + r * BB, half, sub, r, A[buf]);
        }
        // B: the inputs of the chunk as hi / lo rows
        for (int i = tid; i < G5_T * (G5_KC / 8); i += G5_THREADS) {
            const int t = i / (G5_KC / 8), k8 = (i % (G5_KC / 8)) * 8, k = c * G5_KC + k8;
            uint32_t vh[4] = {0, 0, 0, 0}, vl[4] = {0, 0, 0, 0};
            if (tok0 + t < p.ntok) {
                const float *xr = p.x + (size_t)(tok0 + t) * p.ldx + k;
                const float rr = p.rrms ? p.rrms[tok0 + t] : 1.0f;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    float a = xr[2 * j], b = xr[2 * j + 1];
                    if (p.nw) {
                        a = __fmul_rn(__fmul_rn(a, rr), p.nw[k + 2 * j]);
                        b = __fmul_rn(__fmul_rn(b, rr), p.nw[k + 2 * j + 1]);
                    }
                    const __half ah = __float2half_rn(a), bh = __float2half_rn(b);
                    const __half al = __float2half_rn(a - __half2float(ah)), bl = __float2half_rn(b - __half2float(bh));
                    vh[j] = (uint32_t)__half_as_ushort(ah) | ((uint32_t)__half_as_ushort(bh) << 16);
                    vl[j] = (uint32_t)__half_as_ushort(al) | ((uint32_t)__half_as_ushort(bl) << 16);
                }
            }
            *reinterpret_cast<uint4 *>(B[buf] + g5_off(2 * t, k8)) = make_uint4(vh[0], vh[1], vh[2], vh[3]);
            *reinterpret_cast<uint4 *>(B[buf] + g5_off(2 * t + 1, k8)) = make_uint4(vl[0], vl[1], vl[2], vl[3]);
        }
        // generic-proxy shared-memory writes -> visible to the tensor core
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a0 = g5_saddr(A[buf]), b0 = g5_saddr(B[buf]);
#pragma unroll
            for (int s = 0; s < G5_KC / 16; s++) {
                const uint64_t da = g5_desc(a0 + s * 256), db = g5_desc(b0 + s * 256);
                const uint32_t acc = (c > 0 || s > 0) ? 1u : 0u;
                asm volatile(
                    "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                    " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
                    "l"(da), "l"(db), "r"(g5_idesc()), "r"(acc)
                    : "memory");
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             g5_saddr(&done[buf]))
                         : "memory");
        }
        issued = c + 1;
    }
    // all committed MMAs complete (a commit covers every earlier MMA of the thread)
    if (issued > 0 && tid == 0) {
        const int c = issued - 1;
        if (!g5_wait(&done[c & 1], (uint32_t)((c >> 1) & 1))) fail = 1;
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (fail) {
        if (tid == 0) *p.err = 6;
    } else if (warp < 4) {
        // lanes 32*warp .. +31 = weight rows; 16 columns (8 tokens) per load
        const int r = warp * 32 + lane;
        for (int c0 = 0; c0 < G5_N; c0 += 16) {
            uint32_t v[16];
            const uint32_t addr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0;
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                  "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                  "=r"(v[15])
                : "r"(addr)
                : "memory");
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (row0 + r < p.rows) {
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int t = tok0 + c0 / 2 + j;
                    if (t < p.ntok) {
                        const float y = __fadd_rn(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
                        float *dst = p.y + (size_t)t * p.ldy + p.out_off + row0 + r;
                        *dst = p.epi == G5_RESID ? __fadd_rn(*dst, y) : y;
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(G5_N) : "memory");
    }
}

constexpr int g5_smem_bytes(int type) {
    return 2 * G5_A_BYTES + 2 * G5_B_BYTES + G5_M * (type == T_Q4_K ? 144 : (type == T_Q6_K ? 210 : 512));
}

}  // namespace fiber
