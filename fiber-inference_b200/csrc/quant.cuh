// quant.cuh — exact decoding of GGUF K-quant weights on the device.
//
// Each decoded weight equals, bit for bit, what the reference's CPU dequantizer
// produces (src/dequant.h:9-58): the products d*sc*q and dmin*m are exact in
// fp32 (at most 22 significant bits), the difference is rounded once to fp32
// and then to fp16. Q5_K follows the reference's only definition, the Metal
// kernel (metal/kernels.metal:141-169), which keeps the fp32 value.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#define FDEV __device__ __forceinline__

namespace fiber {

enum : int { T_F32 = 0, T_F16 = 1, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14 };

// Programmatic dependent launch (every kernel of the decode step uses both):
// pdl_trigger lets the next kernel in the stream start its prologue; pdl_wait
// blocks until the previous kernel has completed and its writes are visible.
// Every kernel waits before it reads or writes any activation, so completion of
// a kernel implies completion of all earlier ones.
FDEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
FDEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

FDEV float h2f(uint32_t bits16) { return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFFu))); }
FDEV float round_f16(float v) { return __half2float(__float2half_rn(v)); }

// 6-bit scale and min of sub-block j (0..7) from the 12-byte field held in three
// little-endian words s0 = bytes 0-3, s1 = bytes 4-7, s2 = bytes 8-11
// (layout of get_scale_min_k4, metal/kernels.metal:10-19).
FDEV void scale_min_k4(int j, uint32_t s0, uint32_t s1, uint32_t s2, int &sc, int &mn) {
    if (j < 4) {
        sc = (s0 >> (8 * j)) & 63;
        mn = (s1 >> (8 * j)) & 63;
    } else {
        const int k = j - 4;
        const uint32_t lo = (s2 >> (8 * k)) & 0xFF;
        sc = (lo & 0xF) | (((s0 >> (8 * k + 6)) & 3) << 4);
        mn = (lo >> 4) | (((s1 >> (8 * k + 6)) & 3) << 4);
    }
}

// weight = fp16( (d*sc)*q - dmin*m ); dsc and dmm are exact products.
FDEV float q4k_weight(float dsc, float dmm, int q) { return round_f16(__fsub_rn(__fmul_rn(dsc, (float)q), dmm)); }
// Metal Q5_K: (d*sc)*(nib + 16*hi) - dmin*m in fp32, no fp16 rounding.
FDEV float q5k_weight(float dsc, float dmm, int q) { return __fsub_rn(__fmul_rn(dsc, (float)q), dmm); }
// Q6_K: fp16( (d*sc)*q ), q in [-32, 31]
FDEV float q6k_weight(float dsc, int q) { return round_f16(__fmul_rn(dsc, (float)q)); }

// Decode element e (0..255) of one super-block; used by the dequant entry point
// and by the embedding lookup. Returns the weight as the GEMV uses it.
template <int T>
FDEV float decode_elem(const uint8_t *__restrict__ blk, int e);

template <>
FDEV float decode_elem<T_Q4_K>(const uint8_t *__restrict__ blk, int e) {
    const uint16_t *h = reinterpret_cast<const uint16_t *>(blk);
    const float d = h2f(h[0]), dmin = h2f(h[1]);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(blk + 4);
    const int g = e >> 6, s = (e >> 5) & 1, l = e & 31;
    int sc, mn;
    scale_min_k4(2 * g + s, w[0], w[1], w[2], sc, mn);
    const uint8_t q = blk[16 + 32 * g + l];
    return q4k_weight(__fmul_rn(d, (float)sc), __fmul_rn(dmin, (float)mn), s ? (q >> 4) : (q & 15));
}

template <>
FDEV float decode_elem<T_Q5_K>(const uint8_t *__restrict__ blk, int e) {
    const uint16_t *h = reinterpret_cast<const uint16_t *>(blk);
    const float d = h2f(h[0]), dmin = h2f(h[1]);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(blk + 4);
    const int g = e >> 6, s = (e >> 5) & 1, l = e & 31;
    int sc, mn;
    scale_min_k4(2 * g + s, w[0], w[1], w[2], sc, mn);
    const uint8_t q = blk[48 + 32 * g + l];
    const int nib = s ? (q >> 4) : (q & 15);
    const int hi = (blk[16 + l] >> (2 * g + s)) & 1;
    return q5k_weight(__fmul_rn(d, (float)sc), __fmul_rn(dmin, (float)mn), nib + 16 * hi);
}

template <>
FDEV float decode_elem<T_Q6_K>(const uint8_t *__restrict__ blk, int e) {
    const float d = h2f((uint32_t)blk[208] | ((uint32_t)blk[209] << 8));
    const int half = e >> 7, r = e & 127, quad = r >> 5, l = r & 31;
    const uint8_t *ql = blk + 64 * half, *qh = blk + 128 + 32 * half;
    const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192 + 8 * half);
    const uint8_t lo = (quad & 1) ? ql[l + 32] : ql[l];
    const int low4 = (quad >= 2) ? (lo >> 4) : (lo & 15);
    const int hi2 = (qh[l] >> (2 * quad)) & 3;
    const int q = (low4 | (hi2 << 4)) - 32;
    return q6k_weight(__fmul_rn(d, (float)sc[l / 16 + 2 * quad]), q);
}

}  // namespace fiber
