// gemm_tc5.cuh — dequant-GEMM for batched prefill on the 5th-generation tensor cores.
//
// Y[t][out_off + r] (op)= sum_k W[r][k] * xn[t][k] for a GGUF weight matrix W (Q4_K,
// Q5_K, Q6_K or F16 super-blocks, rows x cols) and ntok input rows x (fp32, optionally
// RMS-normalised per token: xn = x * rrms[t] * nw[k]).
//
// Two kernels:
//   * g5_pack_kernel turns the inputs once into the MMA's B operand: per 64-token
//     tile and 128-wide K chunk a 32 KB block in the canonical no-swizzle K-major
//     layout (8x16-byte core matrices: rows 16 B apart, K groups of 8 128 B apart,
//     row groups 2048 B apart), two B rows per token (n = 2t: fp16 hi part, n = 2t+1:
//     fp16 lo part, x = hi + lo to ~22 bits), RMSNorm folded in;
//   * gemm_tc5_kernel: one CTA per 128-row x 64-token tile, tcgen05.mma (kind::f16,
//     M = 128, N = 128, fp32 accumulators in tensor memory), warp-specialised:
//       warp 0      producer: the raw weight rows of each K unit (a super-block
//                   column of 128 rows, one 2D tensor copy; Q6_K matrices whose rows
//                   are not a multiple of 16 bytes long are given a copy with padded
//                   rows) into a ring of raw stages, and each chunk's packed B block
//                   (one bulk copy) into a ring of B stages;
//       warp 1      one lane issues the 8 MMAs (K = 16) of each chunk and commits them
//                   to the barriers that free the B stage and the A buffer;
//       warps 2-9   decode the chunk's weights exactly to fp16 (the reference
//                   dequantizer's arithmetic, with the packed instructions of the
//                   GEMV: quants -> half2 by LOP3 / byte permute, HFMA2, mixed-precision
//                   FMA, cvt.rn.f16x2) into one of two A buffers, then run the epilogue
//                   (tcgen05.ld, hi + lo columns added, Y stored or accumulated).
// Q5_K weights are fp32 values (the Metal kernel's arithmetic, no fp16 rounding): they
// are split into fp16 hi and lo parts, two A tiles per chunk whose MMAs accumulate into
// the same tensor-memory tile (w = hi + lo to ~22 bits, like x).
// Inside every group of 4 K positions the decoded pairs come out as (k0, k2), (k1, k3);
// A and B both use that order (slots 0..3 hold k0, k2, k1, k3), so the products are
// unchanged.
// Every wait is bounded (%globaltimer); on timeout the CTA records an error, waits
// (bounded) for its copies and committed MMAs, frees its tensor memory and returns.
#pragma once
#include <cuda.h>

#include "gemv_tc.cuh"

namespace fiber {

// Instrumentation hook (event id, chunk); compiles to nothing unless a timing harness
// defines it before including this file.
#ifndef G5_MARK
#define G5_MARK(ev, c)
#endif

constexpr int G5_M = 128;        // weight rows per CTA (MMA M)
constexpr int G5_T = 64;         // tokens per CTA (MMA N = 2 * G5_T)
constexpr int G5_N = 2 * G5_T;
constexpr int G5_KC = 128;       // K per chunk (8 MMAs)
constexpr int G5_DW = 8;         // decoder warps
constexpr int G5_THREADS = 64 + 32 * G5_DW;
constexpr int G5_A_BYTES = G5_M * G5_KC * 2;  // 32 KB
constexpr int G5_B_BYTES = G5_N * G5_KC * 2;  // 32 KB: one packed B block
constexpr unsigned long long G5_WAIT_NS = 2000000000ull;

enum : int { G5_STORE = 0, G5_RESID = 1 };

struct G5Params {
    CUtensorMap wmap;      // 2D map of the weights: box 128 rows x one K unit (bytes / fp16)
    const uint8_t *w;      // weights, rows x cols in GGUF super-blocks; rows 16-byte aligned
    int type;              // T_Q4_K / T_Q5_K / T_Q6_K / T_F16
    int rows, cols, ntok;
    const uint8_t *bp;     // packed B: [ceil(ntok / 64)][cols / 128] blocks of 32 KB
    float *y;              // [ntok][ldy]
    int ldy, out_off;
    int epi;               // G5_STORE: y = acc; G5_RESID: y += acc
    const float *resid;    // non-null: y = resid + acc (same layout as y; out of place)
    int *err;              // set to 6 when a wait gave up
};
// Split-K: gridDim.z = ks CTAs per tile, launched as one thread-block cluster (1, 1, ks).
// CTA z covers K units [z U / ks, (z+1) U / ks) of the U = cols / 256 super-block
// columns (F16: cols / 128 chunks) and leaves its fp32 tile in shared memory; CTA z
// then adds slice z of the tile over the cluster's CTAs in order 0 .. ks-1
// (distributed shared memory) and stores it.

constexpr int G5_MAX_KSPLIT = 8;  // portable cluster size

// Splits of K for a launch of rows x ntok over cols: only when the tiles alone leave
// most SMs idle; whole K units per split, at most one split per unit.
HDCE int g5_choose_ksplit(int type, int rows, int cols, int ntok, int n_sm) {
    const int base = ((rows + G5_M - 1) / G5_M) * ((ntok + G5_T - 1) / G5_T);
    const int units = type == T_F16 ? cols / G5_KC : cols / 256;
    if (base * 3 >= n_sm * 2) return 1;
    int ks = (n_sm + base - 1) / base;
    if (ks > units) ks = units;
    if (ks > G5_MAX_KSPLIT) ks = G5_MAX_KSPLIT;
    return ks < 1 ? 1 : ks;
}

FDEV uint64_t g5_desc(uint32_t saddr) {
    // SWIZZLE_NONE K-major: start >> 4, LBO = 128 B (next K group), SBO = 2048 B
    // (next 8-row group), version 1 (bits 46-47)
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(2048 >> 4) << 32) |
           (1ull << 46);
}

// kind::f16 instruction descriptor: D f32, A and B f16, both K-major, N, M
HDCE uint32_t g5_idesc() {
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
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(g5_saddr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait for the phase of parity `parity` to complete; gives up when another thread of
// the CTA has failed, or after G5_WAIT_NS (then marks the CTA failed).
FDEV bool g5_wait(uint64_t *bar, uint32_t parity, volatile int *fail) {
    const unsigned long long t0 = g5_now();
    while (!g5_try_wait(bar, parity)) {
        if (*fail) return false;
        if (g5_now() - t0 > G5_WAIT_NS) {
            *fail = 1;
            return false;
        }
    }
    return true;
}
// Same, ignoring the failure flag (drains in-flight work after a failure).
FDEV bool g5_drain(uint64_t *bar, uint32_t parity) {
    const unsigned long long t0 = g5_now();
    while (!g5_try_wait(bar, parity))
        if (g5_now() - t0 > G5_WAIT_NS) return false;
    return true;
}
FDEV void g5_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(g5_saddr(bar)) : "memory");
}
FDEV void g5_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(g5_saddr(bar)), "r"(bytes) : "memory");
}
FDEV void g5_bulk(void *sdst, const void *gsrc, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     g5_saddr(sdst)),
                 "l"(gsrc), "r"(bytes), "r"(g5_saddr(bar))
                 : "memory");
}
FDEV void g5_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(g5_saddr(bar))
                 : "memory");
}

FDEV uint32_t g5_cluster_addr(const void *p, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(g5_saddr(p)), "r"(rank));
    return r;
}
FDEV float4 g5_ld_cluster4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}
FDEV void g5_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

struct G5PackParams {
    const float *x;        // [ntok][ldx]
    int ldx, ntok, cols;
    const float *rrms;     // [ntok] or null: 1 / rms per token
    const float *nw;       // [cols] or null: no normalisation
    int own_rms;           // 1: compute rrms here (eps) instead of reading it
    float eps;
    uint8_t *bp;
    int *err;              // set to 5 when a value does not fit fp16
};

// canonical offset of (row r, K slot k) inside a 128-K chunk tile: core matrix (r/8, k/8)
FDEV int g5_off(int r, int k) { return ((r >> 3) * (G5_KC / 8) + (k >> 3)) * 128 + (r & 7) * 16 + (k & 7) * 2; }

// Bytes of one row's weights per K unit in a raw stage. Q4_K / Q5_K: the 144 / 176-byte
// super-block (two chunks). Q6_K: the super-block (two chunks) is 210 bytes at an even
// offset, so the 224-byte span from the 16-byte boundary at or below it (a tensor copy
// must start on a 16-byte boundary). F16: the chunk's 128 values (256 bytes).
template <int T>
HDCE int g5_bb() { return T == T_Q4_K ? 144 : (T == T_Q5_K ? 176 : (T == T_Q6_K ? 210 : 512)); }
template <int T>
HDCE int g5_slot() { return T == T_Q4_K ? 144 : (T == T_Q5_K ? 176 : (T == T_Q6_K ? 224 : 256)); }
template <int T>
HDCE int g5_cpu() { return T == T_F16 ? 1 : 2; }  // chunks per K unit
template <int T>
HDCE int g5_aparts() { return T == T_Q5_K ? 2 : 1; }  // A tiles per chunk (Q5_K: hi, lo)
template <int T>
HDCE int g5_bstages() { return T == T_Q5_K ? 2 : 3; }
template <int T>
HDCE int g5_rstages() { return T == T_Q4_K ? 3 : (T == T_Q5_K ? 1 : 2); }
template <int T>
HDCE int g5_smem() {
    return 2 * g5_aparts<T>() * G5_A_BYTES + g5_bstages<T>() * G5_B_BYTES + g5_rstages<T>() * G5_M * g5_slot<T>();
}

// Decode the 64 weights of row r that chunk c gives this thread (K slots 64*sub ..
// 64*sub + 63 of the chunk) from the staged bytes `blk` into A (slot order k0 k2 k1 k3;
// Q5_K: fp16 hi parts into A, lo parts into A2).
template <int T>
FDEV void g5_decode(const uint8_t *blk, int c, int sub, int r, uint8_t *A, uint8_t *A2);

// Q4_K: chunk c covers half c & 1 of the super-block, i.e. quarter 2 (c & 1) + sub;
// quarter t holds sub-block 2t (low nibbles: chunk K 64 sub + l) and 2t + 1 (high
// nibbles: 64 sub + 32 + l), l = 0..31, from the 32 quant bytes at 16 + 32 t.
template <>
FDEV void g5_decode<T_Q4_K>(const uint8_t *blk, int c, int sub, int r, uint8_t *A, uint8_t *) {
    using D = TcDot<T_Q4_K>;
    D::Row row;
    D::load_row(blk, 2 * (c & 1) + sub, row);
#pragma unroll
    for (int v = 0; v < 4; v++) {  // words 2v, 2v+1: l = 8v .. 8v+7
        uint32_t l0, h0, l1, h1, l2, h2, l3, h3;
        D::frags(row, 2 * v, l0, h0, l1, h1);      // (l0: k 0,2) (l1: k 1,3) low; h: high
        D::frags(row, 2 * v + 1, l2, h2, l3, h3);  // k 4,6 / 5,7
        *reinterpret_cast<uint4 *>(A + g5_off(r, 64 * sub + 8 * v)) = make_uint4(l0, l1, l2, l3);
        *reinterpret_cast<uint4 *>(A + g5_off(r, 64 * sub + 32 + 8 * v)) = make_uint4(h0, h1, h2, h3);
    }
}

// Q6_K: chunk c covers half h = c & 1 (128 elements: planes k = 0..3, l = 0..31,
// element 32 k + l); this thread takes l in [16 sub, 16 sub + 16) of every plane.
template <>
FDEV void g5_decode<T_Q6_K>(const uint8_t *blk, int c, int sub, int r, uint8_t *A, uint8_t *) {
    using D = TcDot<T_Q6_K>;
    D::Row row;
    D::load_row(blk, 2 * (c & 1) + sub, row);
#pragma unroll
    for (int k = 0; k < 4; k++) {
#pragma unroll
        for (int v = 0; v < 2; v++) {  // words 2v, 2v+1: l = 16 sub + 8v .. +7
            uint32_t a0, b0, a1, b1;
            D::frags(row, 2 * v, k, a0, b0);
            D::frags(row, 2 * v + 1, k, a1, b1);
            *reinterpret_cast<uint4 *>(A + g5_off(r, 32 * k + 16 * sub + 8 * v)) = make_uint4(a0, b0, a1, b1);
        }
    }
}

// Q5_K (layout as Q4_K plus qh[32] at 16, qs at 48): element 64 t + 32 s + l has quant
// q = nib + 16 * ((qh[l] >> (2 t + s)) & 1), nib the low (s = 0) or high (s = 1) nibble
// of qs[32 t + l]; value fp32((d*sc) * q - dmin*m) (both products exact in fp32, one
// rounding). Packed: half2 (1024 + q) by LOP3; n = q * sc / 2 exactly in fp16 by HFMA2
// ((1024 + q) * sc/2 - 512 sc, all terms exact); then (2d) * n - dmin*m with one
// mixed-precision FMA (one rounding) = the fp32 value; hi = fp16(v), lo = fp16(v - hi).
template <>
FDEV void g5_decode<T_Q5_K>(const uint8_t *blk, int c, int sub, int r, uint8_t *A, uint8_t *A2) {
    const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
    const int t = 2 * (c & 1) + sub;
    int sc0, m0, sc1, m1;
    TcDot<T_Q4_K>::scales(hdr, t, sc0, m0, sc1, m1);
    const float dmin = h2f(hdr.x >> 16);
    const uint16_t d2 = __half_as_ushort(__float2half_rn(2.0f * h2f(hdr.x & 0xFFFFu)));  // exact
    const uint32_t A0 = h2_splat(0.5f * (float)sc0), B0 = h2_splat(-512.0f * (float)sc0);
    const uint32_t A1 = h2_splat(0.5f * (float)sc1), B1 = h2_splat(-512.0f * (float)sc1);
    const float c0 = -__fmul_rn(dmin, (float)m0), c1 = -__fmul_rn(dmin, (float)m1);
    const uint4 q0 = *reinterpret_cast<const uint4 *>(blk + 48 + 32 * t);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(blk + 64 + 32 * t);
    const uint4 h0 = *reinterpret_cast<const uint4 *>(blk + 16);
    const uint4 h1 = *reinterpret_cast<const uint4 *>(blk + 32);
    const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    // one pair -> (hi word, lo word) of fp16 parts
    auto pair = [&](uint32_t h, uint32_t Am, uint32_t Bm, float cm, uint32_t &hi, uint32_t &lo) {
        float a, b;
        mixed_fma2(hfma2_u(h, Am, Bm), d2, cm, a, b);
        hi = pack_f16x2(a, b);
        const __half2 hh = *reinterpret_cast<const __half2 *>(&hi);
        const float2 hf = __half22float2(hh);
        lo = pack_f16x2(__fsub_rn(a, hf.x), __fsub_rn(b, hf.y));
    };
#pragma unroll
    for (int v = 0; v < 4; v++) {  // words 2v, 2v+1: l = 8v .. 8v+7
        uint32_t lh[4], ll[4], hh4[4], hl4[4];
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const uint32_t w = qw[2 * v + k], hb = hw[2 * v + k];
            // bytes 0, 2 and 1, 3 of the word as (1024 + q) half2 pairs; qh bit 2t (low
            // nibbles) / 2t + 1 (high nibbles) moved to bit 4 of each half
            const uint32_t e02l = lop3_or_and(w, 0x000F000Fu, 0x64006400u) | (((hb >> (2 * t)) & 0x00010001u) << 4);
            const uint32_t e13l = lop3_or_and(w >> 8, 0x000F000Fu, 0x64006400u) | (((hb >> (8 + 2 * t)) & 0x00010001u) << 4);
            const uint32_t e02h = lop3_or_and(w >> 4, 0x000F000Fu, 0x64006400u) | (((hb >> (2 * t + 1)) & 0x00010001u) << 4);
            const uint32_t e13h = lop3_or_and(w >> 12, 0x000F000Fu, 0x64006400u) | (((hb >> (9 + 2 * t)) & 0x00010001u) << 4);
            pair(e02l, A0, B0, c0, lh[2 * k], ll[2 * k]);
            pair(e13l, A0, B0, c0, lh[2 * k + 1], ll[2 * k + 1]);
            pair(e02h, A1, B1, c1, hh4[2 * k], hl4[2 * k]);
            pair(e13h, A1, B1, c1, hh4[2 * k + 1], hl4[2 * k + 1]);
        }
        // slot order k0 k2 | k1 k3 | k4 k6 | k5 k7 = (e02, e13) of word 2v, then of 2v+1
        *reinterpret_cast<uint4 *>(A + g5_off(r, 64 * sub + 8 * v)) = make_uint4(lh[0], lh[1], lh[2], lh[3]);
        *reinterpret_cast<uint4 *>(A2 + g5_off(r, 64 * sub + 8 * v)) = make_uint4(ll[0], ll[1], ll[2], ll[3]);
        *reinterpret_cast<uint4 *>(A + g5_off(r, 64 * sub + 32 + 8 * v)) = make_uint4(hh4[0], hh4[1], hh4[2], hh4[3]);
        *reinterpret_cast<uint4 *>(A2 + g5_off(r, 64 * sub + 32 + 8 * v)) = make_uint4(hl4[0], hl4[1], hl4[2], hl4[3]);
    }
}

// F16: the chunk's 128 values of the row; pairs regrouped to (k0, k2), (k1, k3)
template <>
FDEV void g5_decode<T_F16>(const uint8_t *blk, int c, int sub, int r, uint8_t *A, uint8_t *) {
    (void)c;
    const uint4 *e = reinterpret_cast<const uint4 *>(blk) + 8 * sub;
#pragma unroll
    for (int g = 0; g < 8; g++) {
        const uint4 w = e[g];
        *reinterpret_cast<uint4 *>(A + g5_off(r, 64 * sub + 8 * g)) =
            make_uint4(__byte_perm(w.x, w.y, 0x5410), __byte_perm(w.x, w.y, 0x7632), __byte_perm(w.z, w.w, 0x5410),
                       __byte_perm(w.z, w.w, 0x7632));
    }
}

// ---- input packing ----------------------------------------------------------------------

// Byte offset of (B row n of token tile `tile`, K group g = k / 8) in the packed input.
FDEV size_t g5_bp_off(int tile, int nchunk, int n, int g) {
    return ((size_t)(tile * nchunk + (g >> 4)) << 15) + (size_t)((((n >> 3) * 16) + (g & 15)) << 7) + ((n & 7) << 4);
}

// One CTA (128 threads) per 4 tokens (one 8-row group of a token tile) and 256 columns:
// optional per-token 1/rms (over the whole row), then for each K group of 8 the hi or
// lo fp16 parts in slot order k0 k2 k1 k3 k4 k6 k5 k7. Tokens past ntok get zero rows.
constexpr int G5_PACK_COLS = 256;

__global__ void __launch_bounds__(128) g5_pack_kernel(const G5PackParams a) {
    __shared__ float rr[4];
    const int tile = blockIdx.x >> 4, grp = blockIdx.x & 15, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = tile * G5_T + 4 * grp, nchunk = a.cols / G5_KC, col0 = blockIdx.y * G5_PACK_COLS;
    pdl_trigger();  // launched with programmatic stream serialization: x comes from the
    pdl_wait();     // previous kernel
    {
        const int t = t0 + warp;
        float r = 1.0f;
        if (t < a.ntok && a.nw) {
            if (a.own_rms) {
                const float4 *x = reinterpret_cast<const float4 *>(a.x + (size_t)t * a.ldx);
                float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
                for (int i = lane; i < a.cols / 4; i += 32) {
                    const float4 v = x[i];
                    s0 = fmaf(v.x, v.x, s0);
                    s1 = fmaf(v.y, v.y, s1);
                    s2 = fmaf(v.z, v.z, s2);
                    s3 = fmaf(v.w, v.w, s3);
                }
                float ss = (s0 + s1) + (s2 + s3);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
                r = 1.0f / sqrtf(ss / (float)a.cols + a.eps);
            } else if (a.rrms) {
                r = a.rrms[t];
            }
        }
        if (lane == 0) rr[warp] = r;
    }
    __syncthreads();
    bool bad = false;
#pragma unroll
    for (int it = 0; it < G5_PACK_COLS / 128; it++) {  // items (K group g, B row nr): 2 per thread
        const int i = tid + 128 * it, g = (col0 >> 3) + (i >> 3), nr = i & 7, tt = nr >> 1, t = t0 + tt;
        uint4 out = make_uint4(0u, 0u, 0u, 0u);
        if (t < a.ntok) {
            const float4 *xp = reinterpret_cast<const float4 *>(a.x + (size_t)t * a.ldx + 8 * g);
            const float4 x0 = xp[0], x1 = xp[1];
            float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            if (a.nw) {
                const float4 n0 = reinterpret_cast<const float4 *>(a.nw + 8 * g)[0];
                const float4 n1 = reinterpret_cast<const float4 *>(a.nw + 8 * g)[1];
                const float nv[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
#pragma unroll
                for (int j = 0; j < 8; j++) v[j] = __fmul_rn(__fmul_rn(v[j], rr[tt]), nv[j]);
            }
            uint16_t h[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                bad |= !(fabsf(v[j]) < 65504.0f);
                const __half hi = __float2half_rn(v[j]);
                h[j] = (nr & 1) ? __half_as_ushort(__float2half_rn(v[j] - __half2float(hi))) : __half_as_ushort(hi);
            }
            out = make_uint4((uint32_t)h[0] | ((uint32_t)h[2] << 16), (uint32_t)h[1] | ((uint32_t)h[3] << 16),
                             (uint32_t)h[4] | ((uint32_t)h[6] << 16), (uint32_t)h[5] | ((uint32_t)h[7] << 16));
        }
        *reinterpret_cast<uint4 *>(a.bp + g5_bp_off(tile, nchunk, 8 * grp + nr, g)) = out;
    }
    if (bad) *a.err = 5;
}

// ---- the GEMM ------------------------------------------------------------------------------

template <int T>
__global__ void __launch_bounds__(G5_THREADS, 1) gemm_tc5_kernel(const __grid_constant__ G5Params p) {
    constexpr int BB = g5_bb<T>(), S = g5_slot<T>(), CPU = g5_cpu<T>(), NB = g5_bstages<T>(), NR = g5_rstages<T>();
    constexpr int AP = g5_aparts<T>(), AS = AP * G5_A_BYTES;  // A tiles per chunk, bytes per A stage
    extern __shared__ __align__(1024) uint8_t g5_smem[];
    __shared__ __align__(8) uint64_t bfull[NB], bempty[NB], rfull[NR], rempty[NR], afull[2], afree[2], accb;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int fail;
    __shared__ int n_issued;
    uint8_t *const Abuf = g5_smem;                             // [2][AP][G5_A_BYTES]
    uint8_t *const Bbuf = g5_smem + 2 * AS;                    // [NB][G5_B_BYTES]
    uint8_t *const Rbuf = g5_smem + 2 * AS + NB * G5_B_BYTES;  // [NR][128 rows x S]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row0 = blockIdx.x * G5_M, tile = blockIdx.y, ks = gridDim.z, kz = blockIdx.z;
    const int nchunk = p.cols / G5_KC, nunit = nchunk / CPU;
    // this CTA's chunks: [cb, ce) = whole K units of its split
    const int cb = (int)((long long)kz * nunit / ks) * CPU, ce = (int)((long long)(kz + 1) * nunit / ks) * CPU;
    const int nloc = ce - cb;
    const int vrows = min(G5_M, p.rows - row0);

    if (tid == 0) {
        for (int s = 0; s < NB; s++) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(g5_saddr(&bfull[s])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(g5_saddr(&bempty[s])) : "memory");
        }
        for (int s = 0; s < NR; s++) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(g5_saddr(&rfull[s])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(g5_saddr(&rempty[s])), "r"(G5_DW) : "memory");
        }
        for (int a = 0; a < 2; a++) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(g5_saddr(&afull[a])), "r"(G5_DW) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(g5_saddr(&afree[a])) : "memory");
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(g5_saddr(&accb)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fail = 0;
        n_issued = 0;
    }
    if (warp == 1) {  // 128 fp32 accumulator columns x 128 lanes
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(g5_saddr(&tmem_slot)),
                     "r"(G5_N)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_slot;
    G5_MARK(11, 0);
    // Programmatic dependent launch: the next kernel may set up while this one runs; this
    // one's weights (constant) stream in before the previous kernel has finished, the
    // packed inputs only after it (producer's pdl_wait below; every later use of the
    // inputs or of y is ordered after that wait through the mbarriers).
    pdl_trigger();
    G5_MARK(16, 0);

    if (warp == 0) {
        // ---- producer: raw stage u % NR <- K unit u of the 128 rows; B stage c % NB <- the
        // packed inputs of chunk c. Issue order: unit u before its chunks.
        int i = 0, ui = 0;  // local chunk / unit counters (ring slots and parities)
        bool ok = true;
        for (; i < nloc && ok; i++) {
            const int c = cb + i;
            if (i % CPU == 0) {
                const int rs = ui % NR, u = c / CPU;
                if (ui >= NR) ok = g5_wait(&rempty[rs], (uint32_t)((ui / NR - 1) & 1), &fail);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
                G5_MARK(0, i);
                uint8_t *dst = Rbuf + rs * (G5_M * S);
                if (lane == 0) {
                    // box = 128 rows x one unit (rows past the matrix and bytes past a row
                    // read as zeros); Q6_K: the 224 bytes from the 16-byte boundary at or
                    // below the 210-byte block
                    g5_expect_tx(&rfull[rs], (uint32_t)(G5_M * S));
                    const int x = T == T_F16 ? u * 128 : (T == T_Q6_K ? (u * BB) & ~15 : u * BB);
                    asm volatile(
                        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, "
                        "{%2, %3}], [%4];" ::"r"(g5_saddr(dst)),
                        "l"(reinterpret_cast<uint64_t>(&p.wmap)), "r"(x), "r"(row0), "r"(g5_saddr(&rfull[rs]))
                        : "memory");
                }
                ui++;
            }
            const int s = i % NB;
            if (i >= NB) ok = g5_wait(&bempty[s], (uint32_t)((i / NB - 1) & 1), &fail);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            if (i == 0) pdl_wait();  // the packed inputs were written by an earlier kernel
            if (lane == 0) {
                g5_expect_tx(&bfull[s], (uint32_t)G5_B_BYTES);
                g5_bulk(Bbuf + s * G5_B_BYTES, p.bp + ((size_t)(tile * nchunk + c) << 15), (uint32_t)G5_B_BYTES,
                        &bfull[s]);
            }
            G5_MARK(1, i);
        }
        // every copy issued has landed before the CTA exits
        if (lane == 0) {
            for (int s = 0; s < NB && s < i; s++)
                g5_drain(&bfull[s], (uint32_t)(((s + ((i - 1 - s) / NB) * NB) / NB) & 1));
            for (int s = 0; s < NR && s < ui; s++)
                g5_drain(&rfull[s], (uint32_t)(((s + ((ui - 1 - s) / NR) * NR) / NR) & 1));
        }
    } else if (warp == 1) {
        // ---- MMA issuer
        if (lane == 0) {
            int i = 0;
            for (; i < nloc; i++) {
                const int s = i % NB, a = i & 1;
                if (!g5_wait(&bfull[s], (uint32_t)((i / NB) & 1), &fail)) break;
                G5_MARK(6, i);
                if (!g5_wait(&afull[a], (uint32_t)((i >> 1) & 1), &fail)) break;
                G5_MARK(7, i);
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t b0 = g5_saddr(Bbuf + s * G5_B_BYTES);
#pragma unroll
                for (int part = 0; part < AP; part++) {
                    const uint32_t a0 = g5_saddr(Abuf + a * AS + part * G5_A_BYTES);
#pragma unroll
                    for (int k = 0; k < G5_KC / 16; k++) {
                        const uint64_t da = g5_desc(a0 + k * 256), db = g5_desc(b0 + k * 256);
                        const uint32_t acc = (i > 0 || part > 0 || k > 0) ? 1u : 0u;
                        asm volatile(
                            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                            " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
                            "l"(da), "l"(db), "r"(g5_idesc()), "r"(acc)
                            : "memory");
                    }
                }
                g5_commit(&bempty[s]);
                g5_commit(&afree[a]);
                G5_MARK(8, i);
            }
            if (i > 0) g5_commit(&accb);  // completes when every issued MMA has
            n_issued = i;
        }
    } else {
        // ---- decoders: thread (row r, half sub of the chunk's 128 K)
        const int i = tid - 64, r = i >> 1, sub = i & 1;
        bool ok = true;
        for (int i = 0; i < nloc && ok; i++) {
            const int c = cb + i, u = c / CPU, ui = i / CPU, rs = ui % NR, a = i & 1;
            ok = g5_wait(&rfull[rs], (uint32_t)((ui / NR) & 1), &fail);
            G5_MARK(2, i);
            if (ok && i >= 2) ok = g5_wait(&afree[a], (uint32_t)(((i >> 1) - 1) & 1), &fail);
            G5_MARK(3, i);
            ok = __all_sync(0xffffffffu, ok);  // warp-uniform exit (the warp arrives as one)
            if (!ok) break;
            // Q6_K: the span starts at the 16-byte boundary at or below the block
            const uint8_t *blk = Rbuf + rs * (G5_M * S) + r * S;
            if (T == T_Q6_K) blk += (u * BB) & 15;
            g5_decode<T>(blk, c, sub, r, Abuf + a * AS, Abuf + a * AS + (AP - 1) * G5_A_BYTES);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core
            __syncwarp();
            if (lane == 0) {
                g5_arrive(&afull[a]);
                if (i % CPU == CPU - 1) g5_arrive(&rempty[rs]);
            }
            G5_MARK(4, i);
        }
        // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (= weight rows), column
        // half (w - 2) / 4 (32 tokens x hi / lo)
        const bool epi = ok && nloc > 0 && g5_wait(&accb, 0u, &fail);
        if (__all_sync(0xffffffffu, epi)) {  // tcgen05.ld needs the whole warp
            G5_MARK(9, 0);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int q = warp & 3, rr = 32 * q + lane, ch = (warp - 2) >> 2;
            for (int c0 = 64 * ch; c0 < 64 * ch + 64; c0 += 16) {
                uint32_t v[16];
                const uint32_t addr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0;
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                    "[%16];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                      "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                      "=r"(v[15])
                    : "r"(addr)
                    : "memory");
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (ks > 1) {  // this split's partial tile, [token][row], over the B stages
                    float *w = reinterpret_cast<float *>(Bbuf);
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        w[(c0 / 2 + j) * G5_M + rr] = __fadd_rn(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
                } else if (rr < vrows) {
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int t = tile * G5_T + c0 / 2 + j;
                        if (t < p.ntok) {
                            const float y = __fadd_rn(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
                            const size_t o = (size_t)t * p.ldy + p.out_off + row0 + rr;
                            p.y[o] = p.resid ? __fadd_rn(p.resid[o], y) : (p.epi == G5_RESID ? __fadd_rn(p.y[o], y) : y);
                        }
                    }
                }
            }
        }
    }
    G5_MARK(10, 0);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (ks > 1) {
        // every CTA of the cluster holds its partial tile; CTA kz adds slice kz of the
        // tile over the cluster in split order (every CTA reaches both cluster barriers)
        g5_cluster_sync();
        G5_MARK(12, 0);
        if (!fail) {
            constexpr int Q = G5_T * G5_M / 4;  // float4s per tile
            const int q0 = kz * Q / ks, q1 = (kz + 1) * Q / ks;
            for (int q = q0 + tid; q < q1; q += G5_THREADS) {
                const uint32_t off = (uint32_t)q * 16u;
                float4 acc = g5_ld_cluster4(g5_cluster_addr(Bbuf, 0) + off);
                for (int z = 1; z < ks; z++) {
                    const float4 v = g5_ld_cluster4(g5_cluster_addr(Bbuf, z) + off);
                    acc.x = __fadd_rn(acc.x, v.x);
                    acc.y = __fadd_rn(acc.y, v.y);
                    acc.z = __fadd_rn(acc.z, v.z);
                    acc.w = __fadd_rn(acc.w, v.w);
                }
                const int t = tile * G5_T + (4 * q) / G5_M, r0 = (4 * q) % G5_M;
                if (t >= p.ntok) continue;
                const float vals[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    if (r0 + j >= vrows) break;
                    const size_t o = (size_t)t * p.ldy + p.out_off + row0 + r0 + j;
                    p.y[o] = p.resid ? __fadd_rn(p.resid[o], vals[j]) : (p.epi == G5_RESID ? __fadd_rn(p.y[o], vals[j]) : vals[j]);
                }
            }
        }
        G5_MARK(13, 0);
        g5_cluster_sync();  // peers read this CTA's tile until here
        G5_MARK(14, 0);
    }
    if (fail) {
        // let the committed MMAs finish before the tensor memory is released
        if (tid == 0) {
            if (n_issued > 0) g5_drain(&accb, 0u);
            *p.err = 6;
        }
        __syncthreads();
    }
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(G5_N) : "memory");
    }
    G5_MARK(15, 0);
}

HDCE int g5_smem_bytes(int type) {
    return type == T_Q4_K   ? g5_smem<T_Q4_K>()
           : type == T_Q5_K ? g5_smem<T_Q5_K>()
           : type == T_Q6_K ? g5_smem<T_Q6_K>()
                            : g5_smem<T_F16>();
}

}  // namespace fiber
