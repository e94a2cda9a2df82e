// gemv_tc.cuh — batch-1 dequant GEMV, v2: TMA-staged tiles, exact decode on the
// CUDA cores, dot products on the tensor cores.
//
// Per CTA: 8 warps, tiles of 16 weight rows over the whole input length K. One
// elected thread streams tiles into a shared-memory ring with bulk async copies
// (cp.async.bulk, completion on an mbarrier); the warps split each tile's
// super-blocks among themselves.
//
// Decode. A lane owns, for rows g = lane/4 and g+8 of the tile, one quarter of
// each super-block (64 weights per row). It rebuilds every weight exactly as the
// reference's dequantizer (src/dequant.h:9-58) does -- fp32 products d*sc*q and
// dmin*m, one rounding to fp32, one to fp16 -- with packed instructions:
//   * quants -> half2 (1024+q) by a LOP3 against 0x6400 (Q4_K) or a byte permute
//     (Q6_K); no integer->float conversion;
//   * Q4_K: n = sc*q exactly in fp16 (HFMA2), then v = d*n - dmin*m with one
//     mixed-precision FMA (fp16 x fp16 + fp32, single rounding) = the reference's
//     fp32 value; Q6_K: d*(q-32) by the mixed FMA, times sc (exact) in fp32;
//   * two weights packed and rounded to fp16 by one cvt.rn.f16x2.f32.
// The packed fp16 weights are exactly an m16n8k16 A fragment. The input vector x
// (fp32) is scaled by a power of two and split into x_hi + x_lo (fp16 each; 22
// significant bits) and sent as the first two columns of the B fragment, so one
// mma.sync accumulates 256 exact-weight products into fp32 per warp. The
// quantized super-block is never expanded in memory.
#pragma once
#include <cuda_fp16.h>

#include "gemv.cuh"

namespace fiber {

constexpr int TC_WARPS = 8;
constexpr int TC_THREADS = TC_WARPS * 32;
constexpr int TC_M = 16;  // rows per tile
constexpr long long TC_WAIT_LIMIT = 1ll << 22;

// ---- small PTX helpers --------------------------------------------------------------

FDEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

FDEV void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
FDEV void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
FDEV void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
FDEV bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: gives up after TC_WAIT_LIMIT polls and reports it.
FDEV bool mbar_wait(uint64_t *bar, uint32_t parity) {
    for (long long i = 0; i < TC_WAIT_LIMIT; i++)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
FDEV void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

FDEV uint32_t lop3_or_and(uint32_t a, uint32_t b, uint32_t c) {  // (a & b) | c
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
FDEV uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// two fp32 results d*h.lo + c and d*h.hi + c, each a single rounding of the exact value
FDEV void mixed_fma2(uint32_t h, uint16_t d16, float c, float &lo, float &hi) {
    asm("{\n .reg .f16 l, h;\n mov.b32 {l, h}, %2;\n fma.rn.f32.f16 %0, %3, l, %4;\n fma.rn.f32.f16 %1, %3, h, %4;\n}\n"
        : "=f"(lo), "=f"(hi)
        : "r"(h), "h"(d16), "f"(c));
}
FDEV uint32_t pack_f16x2(float lo, float hi) {  // lo -> bits 0..15, hi -> bits 16..31
    uint32_t d;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}
FDEV uint32_t prmt_b32(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
FDEV uint32_t hsub2_u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
FDEV uint32_t hmul2_u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
// d * (fp16 low half of h) + c in fp32, one rounding
FDEV float mixed_fma_lo(uint32_t h, uint16_t d16, float c) {
    float r;
    asm("{\n .reg .f16 l, h;\n mov.b32 {l, h}, %1;\n fma.rn.f32.f16 %0, %2, l, %3;\n}\n"
        : "=f"(r)
        : "r"(h), "h"(d16), "f"(c));
    return r;
}
FDEV uint32_t h2_splat(float v) {  // exact for the small integers used here
    const __half h = __float2half_rn(v);
    const uint32_t u = __half_as_ushort(h);
    return u | (u << 16);
}
FDEV void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---- per-type geometry and x-fragment mapping ------------------------------------------
// A lane (g, t) feeds mma k-slots {2t, 2t+1, 2t+8, 2t+9} of each k-step s (16 per
// super-block). Which weights of the super-block those slots hold is the type's
// choice (it follows the quant layout); x must be staged with the same mapping:
// elem(t, s, i), i = 0..3 for slots 2t, 2t+1, 2t+8, 2t+9.

template <int T>
struct TcType;

#define HDCE __host__ __device__ constexpr inline

// elem(t, s, i): element (0..255) of a super-block that lane t's k-slot i of
// k-step s holds; pos(kk, t, s, i) is its inverse (checked exhaustively below).
template <>
struct TcType<T_Q4_K> {
    static constexpr int BB = 144;
    // word u = s/2 of the lane's 32 quant bytes [32t, 32t+32); v = s%2
    static HDCE int elem(int t, int s, int i) {
        const int u = s >> 1, v = s & 1;
        const int base = 64 * t + 4 * u + v;
        return base + (i & 1) * 2 + (i >> 1) * 32;
    }
    static HDCE void pos(int kk, int &t, int &s, int &i) {
        t = kk >> 6;
        const int r = kk & 63, r2 = r & 31;
        s = 2 * (r2 >> 2) + (r2 & 1);
        i = 2 * (r >> 5) + ((r2 >> 1) & 1);
    }
};

// Q5_K: the low four quant bits sit in the same nibble layout as Q4_K (qs at byte 48),
// so the k-slot map is Q4_K's; the fifth bit of element 64g + 32s + w is bit 2g + s of
// qh[w] (metal/kernels.metal:141-169).
template <>
struct TcType<T_Q5_K> {
    static constexpr int BB = 176;
    static HDCE int elem(int t, int s, int i) { return TcType<T_Q4_K>::elem(t, s, i); }
    static HDCE void pos(int kk, int &t, int &s, int &i) { TcType<T_Q4_K>::pos(kk, t, s, i); }
};

template <>
struct TcType<T_Q6_K> {
    static constexpr int BB = 210;
    // lane t: half h = t/2, positions l in [16*(t%2), +16); step s = 4u + k
    static HDCE int elem(int t, int s, int i) {
        const int h = t >> 1, lh = t & 1, u = s >> 2, k = s & 3;
        const int l0 = 16 * lh + 4 * u;
        const int di = (i == 0) ? 0 : (i == 1) ? 2 : (i == 2) ? 1 : 3;
        return 128 * h + l0 + di + 32 * k;
    }
    static HDCE void pos(int kk, int &t, int &s, int &i) {
        const int h = kk >> 7, r = kk & 127, k = r >> 5, l = r & 31;
        const int di = l & 3;
        t = 2 * h + (l >> 4);
        s = 4 * ((l >> 2) & 3) + k;
        i = (di == 1) ? 2 : (di == 2) ? 1 : di;
    }
};

template <>
struct TcType<T_F16> {
    static constexpr int BB = 512;
    static HDCE int elem(int t, int s, int i) { return 16 * s + 2 * t + (i & 1) + (i >> 1) * 8; }
    static HDCE void pos(int kk, int &t, int &s, int &i) {
        s = kk >> 4;
        const int r = kk & 15, r2 = r & 7;
        t = r2 >> 1;
        i = 2 * (r >> 3) + (r2 & 1);
    }
};

template <int T>
HDCE bool tc_pos_roundtrip() {
    for (int kk = 0; kk < 256; kk++) {
        int t = 0, s = 0, i = 0;
        TcType<T>::pos(kk, t, s, i);
        if (t < 0 || t > 3 || s < 0 || s > 15 || i < 0 || i > 3 || TcType<T>::elem(t, s, i) != kk) return false;
    }
    return true;
}
static_assert(tc_pos_roundtrip<T_Q4_K>() && tc_pos_roundtrip<T_Q5_K>() && tc_pos_roundtrip<T_Q6_K>() &&
                  tc_pos_roundtrip<T_F16>(),
              "fragment slot maps must be inverse bijections on a super-block");

// ---- per-type tile dot: accumulate one super-block of rows g, g+8 --------------------

template <int T>
struct TcDot;

template <>
struct TcDot<T_Q4_K> {
    // Returns the two 16-bit halves of sub-block j's scale/min as (sc, mn) for j = 2t (lo) and 2t+1 (hi).
    static FDEV void scales(uint4 hdr, int t, int &sc_lo, int &mn_lo, int &sc_hi, int &mn_hi) {
        // j = 2t and 2t+1; j < 4 <=> t < 2 (branch-free select)
        const int j0 = 2 * t, j1 = 2 * t + 1;
        const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
        const int k0 = j0 & 3, k1 = j1 & 3;
        const uint32_t a0 = (s0 >> (8 * k0)) & 0xFF, a1 = (s0 >> (8 * k1)) & 0xFF;
        const uint32_t b0 = (s1 >> (8 * k0)) & 0xFF, b1 = (s1 >> (8 * k1)) & 0xFF;
        const uint32_t c0 = (s2 >> (8 * k0)) & 0xFF, c1 = (s2 >> (8 * k1)) & 0xFF;
        if (t < 2) {
            sc_lo = a0 & 63; mn_lo = b0 & 63;
            sc_hi = a1 & 63; mn_hi = b1 & 63;
        } else {
            sc_lo = (c0 & 15) | ((a0 >> 6) << 4); mn_lo = (c0 >> 4) | ((b0 >> 6) << 4);
            sc_hi = (c1 & 15) | ((a1 >> 6) << 4); mn_hi = (c1 >> 4) | ((b1 >> 6) << 4);
        }
    }

    // one row's fragments for all 16 steps are produced word by word
    struct Row {
        uint32_t A_lo, B_lo, A_hi, B_hi;
        float c_lo, c_hi;
        uint16_t d16;
        uint32_t w[8];
    };

    // Lane t's two sub-blocks 2t, 2t+1: their 6-bit scales as the byte pair scp
    // (lo, hi) and mins as mp, then every constant by exact fp16 arithmetic on
    // 1024 + n (byte permutes, no integer-to-float conversions):
    // A_lo = (sc, sc), B_lo = -1024 sc, A_hi = sc'/16, B_hi = -64 sc',
    // c = -dmin * m as one exact mixed-precision product.
    static FDEV void load_row(const uint8_t *blk, int t, Row &r) {
        const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
        const uint4 q0 = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * t);
        const uint4 q1 = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * t);
        r.w[0] = q0.x; r.w[1] = q0.y; r.w[2] = q0.z; r.w[3] = q0.w;
        r.w[4] = q1.x; r.w[5] = q1.y; r.w[6] = q1.z; r.w[7] = q1.w;
        const int sh = 16 * (t & 1);
        const uint32_t A = hdr.y >> sh, B = hdr.z >> sh, C = hdr.w >> sh;
        uint32_t scp, mp;
        if (t < 2) {  // sub-blocks 0..3: low 6 bits of bytes 0..3 / 4..7
            scp = A & 0x3F3Fu;
            mp = B & 0x3F3Fu;
        } else {      // sub-blocks 4..7: nibbles of bytes 8..11, top bits of bytes 0..7
            scp = (C & 0x0F0Fu) | ((A >> 2) & 0x3030u);
            mp = ((C >> 4) & 0x0F0Fu) | ((B >> 2) & 0x3030u);
        }
        constexpr uint32_t M1024 = 0x64006400u;
        const uint32_t sl2 = hsub2_u(prmt_b32(scp, 0x64646464u, 0x4040u), M1024);   // (sc, sc)
        const uint32_t sh2 = hsub2_u(prmt_b32(scp, 0x64646464u, 0x4141u), M1024);   // (sc', sc')
        const uint32_t mneg = hsub2_u(M1024, prmt_b32(mp, 0x64646464u, 0x4140u));  // (-m, -m')
        r.A_lo = sl2;
        r.B_lo = hmul2_u(sl2, 0xE400E400u);  // x -1024
        r.A_hi = hmul2_u(sh2, 0x2C002C00u);  // x 1/16
        r.B_hi = hmul2_u(sh2, 0xD400D400u);  // x -64
        const uint16_t dmin16 = (uint16_t)(hdr.x >> 16);
        r.c_lo = mixed_fma_lo(mneg, dmin16, 0.0f);
        r.c_hi = mixed_fma_lo(mneg >> 16, dmin16, 0.0f);
        r.d16 = (uint16_t)(hdr.x & 0xFFFF);
    }

    // fragments (a0a1 for step 2u, a4a5 for step 2u, a0a1 for step 2u+1, a4a5 for step 2u+1)
    static FDEV void frags(const Row &r, int u, uint32_t &f0, uint32_t &f2, uint32_t &f1, uint32_t &f3) {
        const uint32_t w = r.w[u], w8 = w >> 8;
        const uint32_t h0 = lop3_or_and(w, 0x000F000Fu, 0x64006400u);
        const uint32_t h1 = lop3_or_and(w8, 0x000F000Fu, 0x64006400u);
        const uint32_t h2 = lop3_or_and(w, 0x00F000F0u, 0x64006400u);
        const uint32_t h3 = lop3_or_and(w8, 0x00F000F0u, 0x64006400u);
        const uint32_t n0 = hfma2_u(h0, r.A_lo, r.B_lo), n1 = hfma2_u(h1, r.A_lo, r.B_lo);
        const uint32_t n2 = hfma2_u(h2, r.A_hi, r.B_hi), n3 = hfma2_u(h3, r.A_hi, r.B_hi);
        float a, b;
        mixed_fma2(n0, r.d16, r.c_lo, a, b);
        f0 = pack_f16x2(a, b);
        mixed_fma2(n1, r.d16, r.c_lo, a, b);
        f1 = pack_f16x2(a, b);
        mixed_fma2(n2, r.d16, r.c_hi, a, b);
        f2 = pack_f16x2(a, b);
        mixed_fma2(n3, r.d16, r.c_hi, a, b);
        f3 = pack_f16x2(a, b);
    }

    // two accumulator chains (even / odd k-steps), added at the end
    static FDEV void run(const uint8_t *rowg, const uint8_t *rowg8, const uint2 *xf, int g, int t, float (&acc)[4]) {
        Row ra, rb;
        load_row(rowg, t, ra);
        load_row(rowg8, t, rb);
        float acc2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int u = 0; u < 8; u++) {
            uint32_t a0, a4, a0n, a4n, b0, b4, b0n, b4n;
            frags(ra, u, a0, a4, a0n, a4n);
            frags(rb, u, b0, b4, b0n, b4n);
            uint2 x0 = make_uint2(0u, 0u), x1 = make_uint2(0u, 0u);
            if (g < 2) {
                x0 = xf[((2 * u) * 4 + t) * 2 + g];
                x1 = xf[((2 * u + 1) * 4 + t) * 2 + g];
            }
            mma16816(acc, a0, b0, a4, b4, x0.x, x0.y);
            mma16816(acc2, a0n, b0n, a4n, b4n, x1.x, x1.y);
        }
#pragma unroll
        for (int i = 0; i < 4; i++) acc[i] += acc2[i];
    }
};

// Q5_K keeps the reference's fp32 weights (no fp16 rounding: d*sc*q - dmin*m rounded
// once to fp32, as metal/kernels.metal:141-169 computes it). On the tensor cores each
// weight, scaled by a power of two s per row and super-block (largest |w * s| in
// [2^14, 2^15)), is split into fp16 hi + lo (~22 bits; the lo part stays normal), and
// each k-step issues two MMAs (hi, lo) into the same accumulators; the row's partial
// sums are scaled back by 1/s (exact).
template <>
struct TcDot<T_Q5_K> {
    struct Row {
        TcDot<T_Q4_K>::Row q;  // scales, mins and d as Q4_K; q.w = the lane's 8 quant words
        uint32_t h[8];          // the 8 qh words (every lane reads all 32 bytes)
        float s, inv;           // the row's power-of-two weight scale and its inverse
    };

    static FDEV void load_row(const uint8_t *blk, int t, Row &r) {
        // header (d, dmin, 12 scale bytes) has Q4_K's layout; reuse its decode, then
        // replace the quant words (qs at 48 instead of 16)
        TcDot<T_Q4_K>::load_row(blk, t, r.q);
        const uint4 q0 = *reinterpret_cast<const uint4 *>(blk + 48 + 32 * t);
        const uint4 q1 = *reinterpret_cast<const uint4 *>(blk + 64 + 32 * t);
        r.q.w[0] = q0.x; r.q.w[1] = q0.y; r.q.w[2] = q0.z; r.q.w[3] = q0.w;
        r.q.w[4] = q1.x; r.q.w[5] = q1.y; r.q.w[6] = q1.z; r.q.w[7] = q1.w;
        const uint4 h0 = *reinterpret_cast<const uint4 *>(blk + 16);
        const uint4 h1 = *reinterpret_cast<const uint4 *>(blk + 32);
        r.h[0] = h0.x; r.h[1] = h0.y; r.h[2] = h0.z; r.h[3] = h0.w;
        r.h[4] = h1.x; r.h[5] = h1.y; r.h[6] = h1.z; r.h[7] = h1.w;
        // |w| <= d * 63 * 31 + dmin * 63
        const uint32_t hx = *reinterpret_cast<const uint32_t *>(blk);
        const float bound = fmaf(h2f((uint16_t)(hx & 0xFFFF)), 1953.0f, h2f((uint16_t)(hx >> 16)) * 63.0f);
        int eb = (int)((__float_as_uint(bound) >> 23) & 0xFF);
        eb = max(15, min(eb, 254));  // bound in [2^(eb-127), 2^(eb-126))
        r.s = __uint_as_float((uint32_t)(268 - eb) << 23);    // 2^(141 - eb): bound * s < 2^15
        r.inv = __uint_as_float((uint32_t)(eb - 14) << 23);   // 1 / s
    }

    // hi and lo fragments of a pair of fp32 weights scaled by s
    static FDEV void split(float a, float b, float s, uint32_t &hi, uint32_t &lo) {
        const float as = a * s, bs = b * s;
        hi = pack_f16x2(as, bs);
        float ra, rb;
        asm("{\n .reg .f16 l, u, m;\n mov.b32 {l, u}, %2;\n mov.b16 m, 0xBC00;\n"
            " fma.rn.f32.f16 %0, l, m, %3;\n fma.rn.f32.f16 %1, u, m, %4;\n}\n"
            : "=f"(ra), "=f"(rb)
            : "r"(hi), "f"(as), "f"(bs));
        lo = pack_f16x2(ra, rb);
    }

    // word u of the row: hi/lo fragments for k-steps 2u (f0, f2) and 2u + 1 (f1, f3)
    static FDEV void frags(const Row &r, int u, int t, uint32_t (&fh)[4], uint32_t (&fl)[4]) {
        const uint32_t w = r.q.w[u], w8 = w >> 8;
        const uint32_t bl = (r.h[u] >> (2 * t)) & 0x01010101u, bh = (r.h[u] >> (2 * t + 1)) & 0x01010101u;
        constexpr uint32_t M = 0x64006400u;
        // 1024 + q (low nibbles, fifth bit at bit 4) and 1024 + 16 q (high nibbles, at bit 8)
        const uint32_t h0 = lop3_or_and(w, 0x000F000Fu, M | ((bl & 0x00010001u) << 4));
        const uint32_t h1 = lop3_or_and(w8, 0x000F000Fu, M | (((bl >> 8) & 0x00010001u) << 4));
        const uint32_t h2 = lop3_or_and(w, 0x00F000F0u, M | ((bh & 0x00010001u) << 8));
        const uint32_t h3 = lop3_or_and(w8, 0x00F000F0u, M | (((bh >> 8) & 0x00010001u) << 8));
        const uint32_t n0 = hfma2_u(h0, r.q.A_lo, r.q.B_lo), n1 = hfma2_u(h1, r.q.A_lo, r.q.B_lo);
        const uint32_t n2 = hfma2_u(h2, r.q.A_hi, r.q.B_hi), n3 = hfma2_u(h3, r.q.A_hi, r.q.B_hi);
        float a, b;
        mixed_fma2(n0, r.q.d16, r.q.c_lo, a, b);
        split(a, b, r.s, fh[0], fl[0]);
        mixed_fma2(n1, r.q.d16, r.q.c_lo, a, b);
        split(a, b, r.s, fh[1], fl[1]);
        mixed_fma2(n2, r.q.d16, r.q.c_hi, a, b);
        split(a, b, r.s, fh[2], fl[2]);
        mixed_fma2(n3, r.q.d16, r.q.c_hi, a, b);
        split(a, b, r.s, fh[3], fl[3]);
    }

    static FDEV void run(const uint8_t *rowg, const uint8_t *rowg8, const uint2 *xf, int g, int t, float (&acc)[4]) {
        Row ra, rb;
        load_row(rowg, t, ra);
        load_row(rowg8, t, rb);
        float pa[4] = {0.f, 0.f, 0.f, 0.f}, pb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int u = 0; u < 8; u++) {
            uint32_t ah[4], al[4], bh[4], bl[4];
            frags(ra, u, t, ah, al);
            frags(rb, u, t, bh, bl);
            uint2 x0 = make_uint2(0u, 0u), x1 = make_uint2(0u, 0u);
            if (g < 2) {
                x0 = xf[((2 * u) * 4 + t) * 2 + g];
                x1 = xf[((2 * u + 1) * 4 + t) * 2 + g];
            }
            // k-step 2u: a0 = f0 (row g), a1 = f0 (row g + 8), a2 = f2, a3 = f2; 2u + 1: f1, f3
            mma16816(pa, ah[0], bh[0], ah[2], bh[2], x0.x, x0.y);
            mma16816(pb, al[0], bl[0], al[2], bl[2], x0.x, x0.y);
            mma16816(pa, ah[1], bh[1], ah[3], bh[3], x1.x, x1.y);
            mma16816(pb, al[1], bl[1], al[3], bl[3], x1.x, x1.y);
        }
        acc[0] = fmaf(pa[0] + pb[0], ra.inv, acc[0]);
        acc[1] = fmaf(pa[1] + pb[1], ra.inv, acc[1]);
        acc[2] = fmaf(pa[2] + pb[2], rb.inv, acc[2]);
        acc[3] = fmaf(pa[3] + pb[3], rb.inv, acc[3]);
    }
};

template <>
struct TcDot<T_Q6_K> {
    // 16 bytes starting at a 2-byte aligned shared-memory address
    static FDEV uint4 lds16_u2(const uint8_t *p) {
        const uintptr_t a = reinterpret_cast<uintptr_t>(p);
        const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~(uintptr_t)3);
        const uint32_t sh = (uint32_t)(a & 3) * 8;  // 0 or 16
        const uint32_t w0 = w[0], w1 = w[1], w2 = w[2], w3 = w[3], w4 = w[4];
        uint4 r;
        r.x = __funnelshift_r(w0, w1, sh);
        r.y = __funnelshift_r(w1, w2, sh);
        r.z = __funnelshift_r(w2, w3, sh);
        r.w = __funnelshift_r(w3, w4, sh);
        return r;
    }

    struct Row {
        uint4 A, B, H;
        float sc[4];
        uint16_t d16;
        float c;  // -32 * d (exact)
    };

    static FDEV void load_row(const uint8_t *blk, int t, Row &r) {
        const int h = t >> 1, lh = t & 1;
        r.A = lds16_u2(blk + 64 * h + 16 * lh);
        r.B = lds16_u2(blk + 64 * h + 32 + 16 * lh);
        r.H = lds16_u2(blk + 128 + 32 * h + 16 * lh);
        const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192 + 8 * h + lh);
        const uint16_t d16 = *reinterpret_cast<const uint16_t *>(blk + 208);
        const float d = h2f(d16);
#pragma unroll
        for (int k = 0; k < 4; k++) r.sc[k] = (float)sc[2 * k];
        r.d16 = d16;
        r.c = -__fmul_rn(1056.0f, d);  // (1024 + 32) * d: d*(1024+q) - 1056*d = d*(q-32)
    }

    // 4 quant bytes (6-bit values) for word u and plane k
    static FDEV uint32_t q6(const Row &r, int u, int k) {
        const uint32_t a = (&r.A.x)[u], b = (&r.B.x)[u], hh = (&r.H.x)[u];
        switch (k) {
        case 0: return lop3_or_and(a, 0x0F0F0F0Fu, (hh << 4) & 0x30303030u);
        case 1: return lop3_or_and(b, 0x0F0F0F0Fu, (hh << 2) & 0x30303030u);
        case 2: return lop3_or_and(a >> 4, 0x0F0F0F0Fu, hh & 0x30303030u);
        default: return lop3_or_and(b >> 4, 0x0F0F0F0Fu, (hh >> 2) & 0x30303030u);
        }
    }

    static FDEV void frags(const Row &r, int u, int k, uint32_t &fa, uint32_t &fb) {
        const uint32_t q = q6(r, u, k);
        const uint32_t h02 = __byte_perm(q, 0x64646464u, 0x4240);  // (1024+q.b0, 1024+q.b2)
        const uint32_t h13 = __byte_perm(q, 0x64646464u, 0x4341);  // (1024+q.b1, 1024+q.b3)
        float a, b;
        mixed_fma2(h02, r.d16, r.c, a, b);
        fa = pack_f16x2(__fmul_rn(a, r.sc[k]), __fmul_rn(b, r.sc[k]));
        mixed_fma2(h13, r.d16, r.c, a, b);
        fb = pack_f16x2(__fmul_rn(a, r.sc[k]), __fmul_rn(b, r.sc[k]));
    }

    static FDEV void run(const uint8_t *rowg, const uint8_t *rowg8, const uint2 *xf, int g, int t, float (&acc)[4]) {
        Row ra, rb;
        load_row(rowg, t, ra);
        load_row(rowg8, t, rb);
#pragma unroll
        for (int u = 0; u < 4; u++) {
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int s = 4 * u + k;
                uint32_t a0, a4, b0, b4;
                frags(ra, u, k, a0, a4);
                frags(rb, u, k, b0, b4);
                uint2 x = make_uint2(0u, 0u);
                if (g < 2) x = xf[(s * 4 + t) * 2 + g];
                mma16816(acc, a0, b0, a4, b4, x.x, x.y);
            }
        }
    }
};

template <>
struct TcDot<T_F16> {
    static FDEV void run(const uint8_t *rowg, const uint8_t *rowg8, const uint2 *xf, int g, int t, float (&acc)[4]) {
        const uint32_t *ra = reinterpret_cast<const uint32_t *>(rowg);
        const uint32_t *rb = reinterpret_cast<const uint32_t *>(rowg8);
#pragma unroll
        for (int s = 0; s < 16; s++) {
            const uint32_t a0 = ra[8 * s + t], a4 = ra[8 * s + t + 4];
            const uint32_t b0 = rb[8 * s + t], b4 = rb[8 * s + t + 4];
            uint2 x = make_uint2(0u, 0u);
            if (g < 2) x = xf[(s * 4 + t) * 2 + g];
            mma16816(acc, a0, b0, a4, b4, x.x, x.y);
        }
    }
};

// ---- the kernel ------------------------------------------------------------------------

struct TcSeg {
    const uint8_t *w;   // weights of this segment
    const uint8_t *w2;  // second matrix (SwiGLU up), same shape
    int rows;
    int out_off;        // EPI_STORE: output offset of row 0
    int tiles;
};

struct TcParams {
    TcSeg seg[3];
    int nseg;
    int cols;
    int row_bytes;     // bytes of one weight row in HBM
    int stride;        // bytes of one row in shared memory
    int per_row_copy;  // 1: one bulk copy per row into a padded stride; 0: one per tile
    int n_tiles;
    int stages;
    int stage_x;       // 1: keep an fp32 copy of x in shared memory while staging
    const float *x;
    const float *norm_w;
    float eps;
    float *y;
    float *resid;
    float2 *am_part;
    unsigned int *am_count;
    int32_t *am_out;
    int32_t *adv_token, *adv_pos, *rec_tokens, *rec_step;
    int *err;          // set to 3 if a bounded wait gives up
};

FDEV void locate(const TcParams &p, int tile, int &s, int &lt) {
    s = 0;
    lt = tile;
    while (s + 1 < p.nseg && lt >= p.seg[s].tiles) lt -= p.seg[s++].tiles;
}

// One thread: bulk-copy tile `tile` (all NMAT matrices) into buf; completion on bar.
// Bytes that do not fill a whole 16-byte unit at the end are copied with plain loads.
template <int NMAT>
FDEV void issue_tile(const TcParams &p, uint8_t *buf, int tile, uint64_t *bar) {
    int s, lt;
    locate(p, tile, s, lt);
    const TcSeg &sg = p.seg[s];
    const int r0 = lt * TC_M;
    const int nrows = min(TC_M, sg.rows - r0);
    const uint32_t mat_bytes = (uint32_t)nrows * p.row_bytes;
    const uint32_t main_bytes = p.per_row_copy ? mat_bytes : (mat_bytes & ~15u);
    mbar_expect_tx(bar, main_bytes * NMAT);
#pragma unroll
    for (int m = 0; m < NMAT; m++) {
        const uint8_t *src = (m == 0 ? sg.w : sg.w2) + (size_t)r0 * p.row_bytes;
        uint8_t *dst = buf + (size_t)m * TC_M * p.stride;
        if (p.per_row_copy) {
            for (int r = 0; r < nrows; r++)
                bulk_g2s(dst + (size_t)r * p.stride, src + (size_t)r * p.row_bytes, p.row_bytes, bar);
        } else {
            if (main_bytes) bulk_g2s(dst, src, main_bytes, bar);
            for (uint32_t k = main_bytes; k < mat_bytes; k++) dst[k] = src[k];
        }
    }
}

// Stage the input as hi/lo fp16 fragments xf[b][s][t][hi, lo] (uint2 pairs),
// through the RMSNorm when norm_w is set: xn[i] = (x[i] * rrms) * w[i].
// One coalesced pass over x (into xs when the caller has room for it, else x is
// gathered again from L2), one block reduction of (sum x^2, max |x|).
template <int T>
FDEV float stage_xf(const TcParams &p, uint2 *xf, float *xs, float *red) {
    const int n = p.cols;
    float ss = 0.f, mx = 0.f;
    for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4) {
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(p.x + i));
        if (xs) *reinterpret_cast<float4 *>(xs + i) = v;
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
        if (p.norm_w) {
            const float4 w = __ldg(reinterpret_cast<const float4 *>(p.norm_w + i));
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x * w.x), fabsf(v.y * w.y)), fmaxf(fabsf(v.z * w.z), fabsf(v.w * w.w))));
        } else {
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
    }
    // one block reduction of both
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ss += __shfl_xor_sync(0xffffffffu, ss, o);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        red[2 * warp] = ss;
        red[2 * warp + 1] = mx;
    }
    __syncthreads();
    ss = 0.f;
    mx = 0.f;
    for (int w = 0; w < nw; w++) {
        ss += red[2 * w];
        mx = fmaxf(mx, red[2 * w + 1]);
    }
    const float rrms = p.norm_w ? 1.0f / sqrtf(ss / (float)n + p.eps) : 1.0f;
    mx *= rrms;  // max |xn| up to rounding: only picks the power-of-two scale
    // scale so max |x| lands near [2^13, 2^14): exact, keeps x_lo out of fp16 subnormals
    int e = 0;
    if (mx > 0.f) frexpf(mx, &e);
    const int sh = (mx > 0.f && isfinite(mx)) ? (14 - e) : 0;
    const float scale = ldexpf(1.0f, sh);
    const int nb = n >> 8;
    for (int f = threadIdx.x; f < nb * 64; f += blockDim.x) {
        const int b = f >> 6, s = (f >> 2) & 15, t = f & 3;
        __half hi[4], lo[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int k = b * 256 + TcType<T>::elem(t, s, i);
            float v = xs ? xs[k] : __ldcg(p.x + k);
            if (p.norm_w) v = __fmul_rn(__fmul_rn(v, rrms), __ldg(p.norm_w + k));
            v *= scale;
            hi[i] = __float2half_rn(v);
            lo[i] = __float2half_rn(v - __half2float(hi[i]));
        }
        const uint32_t h01 = (uint32_t)__half_as_ushort(hi[0]) | ((uint32_t)__half_as_ushort(hi[1]) << 16);
        const uint32_t h23 = (uint32_t)__half_as_ushort(hi[2]) | ((uint32_t)__half_as_ushort(hi[3]) << 16);
        const uint32_t l01 = (uint32_t)__half_as_ushort(lo[0]) | ((uint32_t)__half_as_ushort(lo[1]) << 16);
        const uint32_t l23 = (uint32_t)__half_as_ushort(lo[2]) | ((uint32_t)__half_as_ushort(lo[3]) << 16);
        xf[2 * f + 0] = make_uint2(h01, h23);
        xf[2 * f + 1] = make_uint2(l01, l23);
    }
    __syncthreads();
    return ldexpf(1.0f, -sh);  // multiply results by this
}

template <int T, int EPI, int NMAT>
__global__ void __launch_bounds__(TC_THREADS) gemv_tc_kernel(const TcParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[4];
    __shared__ float red[TC_WARPS * NMAT * TC_M];
    __shared__ float2 am_warp[TC_WARPS];
    __shared__ unsigned int am_ticket;
    __shared__ int bail;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int nb = p.cols >> 8;
    const size_t tile_bytes = (size_t)NMAT * TC_M * p.stride;
    uint8_t *ring = smem;
    uint2 *xf = reinterpret_cast<uint2 *>(smem + tile_bytes * p.stages);
    float *xs = p.stage_x ? reinterpret_cast<float *>(xf + (size_t)nb * 128) : nullptr;

    const int my_tiles = p.n_tiles > (int)blockIdx.x ? (p.n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    pdl_trigger();
    if (tid == 0) {
        for (int s = 0; s < p.stages; s++) mbar_init(&full[s], 1);
        mbar_fence_init();
        bail = 0;
    }
    __syncthreads();
    if (tid == 0)
        for (int i = 0; i < p.stages && i < my_tiles; i++)
            issue_tile<NMAT>(p, ring + tile_bytes * i, (int)blockIdx.x + i * (int)gridDim.x, &full[i]);

    // everything above touched only weights and this CTA's shared memory; the
    // input (and the residual) are the previous kernel's output
    pdl_wait();
    float resid_in = 0.f;
    if constexpr (EPI == EPI_RESID) {
        if (p.resid && my_tiles == 1 && tid < TC_M) {
            int sg0, lt0;
            locate(p, (int)blockIdx.x, sg0, lt0);
            const int r = lt0 * TC_M + tid;
            if (r < p.seg[sg0].rows) resid_in = __ldcg(p.resid + r);
        }
    }
    const float unscale = stage_xf<T>(p, xf, xs, red);

    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    for (int i = 0; i < my_tiles; i++) {
        const int s = i % p.stages;
        const uint32_t parity = (uint32_t)((i / p.stages) & 1);
        const int tile = (int)blockIdx.x + i * (int)gridDim.x;
        if (!mbar_wait(&full[s], parity)) {
            bail = 1;  // racy write of the same value: fine
            if (p.err) *p.err = 3;
        }
        __syncthreads();
        if (bail) {
            // wait (bounded) for copies still in flight into this CTA's smem, then leave
            for (int k = i; k < i + p.stages && k < my_tiles; k++) mbar_wait(&full[k % p.stages], (uint32_t)((k / p.stages) & 1));
            return;
        }
        const uint8_t *buf = ring + tile_bytes * s;
        int sg, lt;
        locate(p, tile, sg, lt);
        float acc[NMAT][4];
#pragma unroll
        for (int m = 0; m < NMAT; m++) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;
        for (int b = warp; b < nb; b += TC_WARPS) {
            const uint2 *xfb = xf + (size_t)b * 128;
#pragma unroll
            for (int m = 0; m < NMAT; m++) {
                const uint8_t *mb = buf + (size_t)m * TC_M * p.stride + (size_t)b * TcType<T>::BB;
                TcDot<T>::run(mb + (size_t)g * p.stride, mb + (size_t)(g + 8) * p.stride, xfb, g, t, acc[m]);
            }
        }
        if (t == 0) {
#pragma unroll
            for (int m = 0; m < NMAT; m++) {
                red[(warp * NMAT + m) * TC_M + g] = acc[m][0] + acc[m][1];
                red[(warp * NMAT + m) * TC_M + g + 8] = acc[m][2] + acc[m][3];
            }
        }
        __syncthreads();  // tile buffer s fully consumed; partials visible
        if (tid == 0 && i + p.stages < my_tiles)
            issue_tile<NMAT>(p, ring + tile_bytes * s, tile + p.stages * (int)gridDim.x, &full[s]);
        if (tid < TC_M) {
            const int r = lt * TC_M + tid;
            float v[NMAT];
#pragma unroll
            for (int m = 0; m < NMAT; m++) {
                float sum = 0.f;
#pragma unroll
                for (int w = 0; w < TC_WARPS; w++) sum += red[(w * NMAT + m) * TC_M + tid];
                v[m] = sum * unscale;
            }
            if (r < p.seg[sg].rows) {
                if constexpr (EPI == EPI_STORE) {
                    p.y[p.seg[sg].out_off + r] = v[0];
                } else if constexpr (EPI == EPI_RESID) {
                    // in place (y null): resid[r] += v; out of place: y[r] = (resid ? resid[r] : 0) + v
                    float *dst = p.y ? p.y : p.resid;
                    dst[r] = p.resid ? __fadd_rn(my_tiles == 1 ? resid_in : __ldcg(p.resid + r), v[0]) : v[0];
                } else if constexpr (EPI == EPI_SWIGLU) {
                    const float gt = v[0];
                    p.y[r] = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))), v[NMAT - 1]);
                } else {
                    p.y[r] = v[0];
                    if (better(v[0], r, best_v, best_i)) {
                        best_v = v[0];
                        best_i = r;
                    }
                }
            }
        }
        __syncthreads();  // red reused next tile
    }

    if constexpr (EPI == EPI_ARGMAX) {
        // threads 0..15 hold candidates; reduce within warp 0
        if (warp == 0) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
                const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
                if (better(ov, oi, best_v, best_i)) {
                    best_v = ov;
                    best_i = oi;
                }
            }
            if (lane == 0) {
                p.am_part[blockIdx.x] = make_float2(best_v, __int_as_float(best_i));
                __threadfence();
                am_ticket = atomicAdd(p.am_count, 1u);
            }
        }
        __syncthreads();
        if (am_ticket == gridDim.x - 1) {
            __threadfence();
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int i = tid; i < (int)gridDim.x; i += blockDim.x) {
                const float2 e = __ldcg(p.am_part + i);
                const int ei = __float_as_int(e.y);
                if (better(e.x, ei, bv, bi)) {
                    bv = e.x;
                    bi = ei;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (better(ov, oi, bv, bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (lane == 0) am_warp[warp] = make_float2(bv, __int_as_float(bi));
            __syncthreads();
            if (tid == 0) {
                for (int w = 1; w < TC_WARPS; w++) {
                    const int wi = __float_as_int(am_warp[w].y);
                    if (better(am_warp[w].x, wi, bv, bi)) {
                        bv = am_warp[w].x;
                        bi = wi;
                    }
                }
                if (bi == 0x7fffffff) bi = 0;
                *p.am_out = bi;
                if (p.adv_token) *p.adv_token = bi;
                if (p.adv_pos) *p.adv_pos += 1;
                if (p.rec_tokens) {
                    const int st = *p.rec_step;
                    p.rec_tokens[st] = bi;
                    *p.rec_step = st + 1;
                }
                *p.am_count = 0u;
            }
        }
    }
}

}  // namespace fiber
