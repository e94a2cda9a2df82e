// gemv.cuh — batch-1 dequant-fused matrix-vector kernels (CUDA cores).
//
// One CTA = 8 warps; each warp owns ROWS consecutive output rows and walks
// their super-blocks, each lane decoding 8 weights per block from one 32-bit
// word of quants (coalesced 128-byte warp loads). The input vector is staged in
// shared memory once per CTA, optionally through the RMSNorm the reference runs
// as a separate dispatch (metal/kernels.metal:271-286, src/fiber_proof.m:23-28):
// x_s[i] = (x[i] * rrms) * w[i], rrms = 1 / sqrtf(sum(x^2)/n + eps).
// Epilogues fuse what follows each projection in the reference's step
// (src/gpu_ffn.m:500-610): plain store (QKV), residual add (Wo, W_down:
// residual_add / residual_rmsnorm), SwiGLU of the gate/up pair (silu_gate),
// and greedy argmax over the logits (sampler.c:38-46) for the lm_head.
#pragma once
#include "quant.cuh"

namespace fiber {

constexpr int GEMV_WARPS = 8;
constexpr int GEMV_THREADS = GEMV_WARPS * 32;

// Per-lane partial dot product of one weight row with x_s (shared memory).
template <int T>
struct RowDot;

template <>
struct RowDot<T_Q4_K> {
    static constexpr int BLOCK_BYTES = 144;
    static FDEV float run(const uint8_t *__restrict__ row, const float *__restrict__ xs, int nb, int lane) {
        const int j = lane >> 3, o = (lane & 7) * 4;
        float acc = 0.f;
#pragma unroll 2
        for (int b = 0; b < nb; b++) {
            const uint8_t *blk = row + b * BLOCK_BYTES;
            const uint4 hdr = __ldg(reinterpret_cast<const uint4 *>(blk));
            const uint32_t qw = __ldg(reinterpret_cast<const uint32_t *>(blk + 16) + lane);
            const float d = h2f(hdr.x), dmin = h2f(hdr.x >> 16);
            int s1, m1, s2, m2;
            scale_min_k4(2 * j, hdr.y, hdr.z, hdr.w, s1, m1);
            scale_min_k4(2 * j + 1, hdr.y, hdr.z, hdr.w, s2, m2);
            const float a1 = __fmul_rn(d, (float)s1), b1 = __fmul_rn(dmin, (float)m1);
            const float a2 = __fmul_rn(d, (float)s2), b2 = __fmul_rn(dmin, (float)m2);
            const float *xb = xs + b * 256 + 64 * j + o;
            const float4 xl = *reinterpret_cast<const float4 *>(xb);
            const float4 xh = *reinterpret_cast<const float4 *>(xb + 32);
            acc = fmaf(q4k_weight(a1, b1, (qw >> 0) & 15), xl.x, acc);
            acc = fmaf(q4k_weight(a1, b1, (qw >> 8) & 15), xl.y, acc);
            acc = fmaf(q4k_weight(a1, b1, (qw >> 16) & 15), xl.z, acc);
            acc = fmaf(q4k_weight(a1, b1, (qw >> 24) & 15), xl.w, acc);
            acc = fmaf(q4k_weight(a2, b2, (qw >> 4) & 15), xh.x, acc);
            acc = fmaf(q4k_weight(a2, b2, (qw >> 12) & 15), xh.y, acc);
            acc = fmaf(q4k_weight(a2, b2, (qw >> 20) & 15), xh.z, acc);
            acc = fmaf(q4k_weight(a2, b2, (qw >> 28) & 15), xh.w, acc);
        }
        return acc;
    }
};

template <>
struct RowDot<T_Q5_K> {
    static constexpr int BLOCK_BYTES = 176;
    static FDEV float run(const uint8_t *__restrict__ row, const float *__restrict__ xs, int nb, int lane) {
        const int j = lane >> 3, o = (lane & 7) * 4;
        float acc = 0.f;
#pragma unroll 2
        for (int b = 0; b < nb; b++) {
            const uint8_t *blk = row + b * BLOCK_BYTES;
            const uint4 hdr = __ldg(reinterpret_cast<const uint4 *>(blk));
            const uint32_t hw = __ldg(reinterpret_cast<const uint32_t *>(blk + 16 + o));
            const uint32_t qw = __ldg(reinterpret_cast<const uint32_t *>(blk + 48) + lane);
            const float d = h2f(hdr.x), dmin = h2f(hdr.x >> 16);
            int s1, m1, s2, m2;
            scale_min_k4(2 * j, hdr.y, hdr.z, hdr.w, s1, m1);
            scale_min_k4(2 * j + 1, hdr.y, hdr.z, hdr.w, s2, m2);
            const float a1 = __fmul_rn(d, (float)s1), b1 = __fmul_rn(dmin, (float)m1);
            const float a2 = __fmul_rn(d, (float)s2), b2 = __fmul_rn(dmin, (float)m2);
            const float *xb = xs + b * 256 + 64 * j + o;
            const float4 xl = *reinterpret_cast<const float4 *>(xb);
            const float4 xh = *reinterpret_cast<const float4 *>(xb + 32);
            const float xlv[4] = {xl.x, xl.y, xl.z, xl.w}, xhv[4] = {xh.x, xh.y, xh.z, xh.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int ql = ((qw >> (8 * i)) & 15) | (((hw >> (8 * i + 2 * j)) & 1) << 4);
                const int qh = ((qw >> (8 * i + 4)) & 15) | (((hw >> (8 * i + 2 * j + 1)) & 1) << 4);
                acc = fmaf(q5k_weight(a1, b1, ql), xlv[i], acc);
                acc = fmaf(q5k_weight(a2, b2, qh), xhv[i], acc);
            }
        }
        return acc;
    }
};

template <>
struct RowDot<T_Q6_K> {
    static constexpr int BLOCK_BYTES = 210;
    static FDEV float run(const uint8_t *__restrict__ row, const float *__restrict__ xs, int nb, int lane) {
        float acc = 0.f;
        const int is = lane >> 4;
#pragma unroll 2
        for (int b = 0; b < nb; b++) {
            const uint8_t *blk = row + b * BLOCK_BYTES;
            const float d = h2f((uint32_t)__ldg(blk + 208) | ((uint32_t)__ldg(blk + 209) << 8));
#pragma unroll
            for (int half = 0; half < 2; half++) {
                const uint32_t l0 = __ldg(blk + 64 * half + lane);
                const uint32_t l1 = __ldg(blk + 64 * half + lane + 32);
                const uint32_t hb = __ldg(blk + 128 + 32 * half + lane);
                const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192 + 8 * half);
                const float c0 = __fmul_rn(d, (float)__ldg(sc + is + 0));
                const float c1 = __fmul_rn(d, (float)__ldg(sc + is + 2));
                const float c2 = __fmul_rn(d, (float)__ldg(sc + is + 4));
                const float c3 = __fmul_rn(d, (float)__ldg(sc + is + 6));
                const int q0 = (int)((l0 & 15) | ((hb & 3) << 4)) - 32;
                const int q1 = (int)((l1 & 15) | (((hb >> 2) & 3) << 4)) - 32;
                const int q2 = (int)((l0 >> 4) | (((hb >> 4) & 3) << 4)) - 32;
                const int q3 = (int)((l1 >> 4) | (((hb >> 6) & 3) << 4)) - 32;
                const float *xb = xs + b * 256 + 128 * half + lane;
                acc = fmaf(q6k_weight(c0, q0), xb[0], acc);
                acc = fmaf(q6k_weight(c1, q1), xb[32], acc);
                acc = fmaf(q6k_weight(c2, q2), xb[64], acc);
                acc = fmaf(q6k_weight(c3, q3), xb[96], acc);
            }
        }
        return acc;
    }
};

template <>
struct RowDot<T_F16> {
    static constexpr int BLOCK_BYTES = 512;  // 256 halves per "block"
    static FDEV float run(const uint8_t *__restrict__ row, const float *__restrict__ xs, int nb, int lane) {
        float acc = 0.f;
        const uint4 *r4 = reinterpret_cast<const uint4 *>(row);
        for (int k = lane; k < nb * 32; k += 32) {  // 8 halves per lane step
            const uint4 v = __ldg(r4 + k);
            const float *xb = xs + 8 * k;
            const float4 xa = *reinterpret_cast<const float4 *>(xb);
            const float4 xc = *reinterpret_cast<const float4 *>(xb + 4);
            acc = fmaf(h2f(v.x), xa.x, acc);
            acc = fmaf(h2f(v.x >> 16), xa.y, acc);
            acc = fmaf(h2f(v.y), xa.z, acc);
            acc = fmaf(h2f(v.y >> 16), xa.w, acc);
            acc = fmaf(h2f(v.z), xc.x, acc);
            acc = fmaf(h2f(v.z >> 16), xc.y, acc);
            acc = fmaf(h2f(v.w), xc.z, acc);
            acc = fmaf(h2f(v.w >> 16), xc.w, acc);
        }
        return acc;
    }
};

FDEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

FDEV float block_sum(float v, float *red /* >= 32 floats */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    if (warp == 0) {
        t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
        t = warp_sum(t);
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    return red[0];
}

// Stage x (length n) into shared memory, through RMSNorm when norm_w != nullptr.
FDEV void stage_input(float *xs, const float *__restrict__ x, int n, const float *__restrict__ norm_w, float eps,
                      float *red) {
    if (norm_w == nullptr) {
        for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4)
            *reinterpret_cast<float4 *>(xs + i) = __ldcg(reinterpret_cast<const float4 *>(x + i));
        __syncthreads();
        return;
    }
    float ss = 0.f;
    for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4) {
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(x + i));
        *reinterpret_cast<float4 *>(xs + i) = v;
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
    }
    const float total = block_sum(ss, red);
    const float rrms = 1.0f / sqrtf(total / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) xs[i] = __fmul_rn(__fmul_rn(xs[i], rrms), __ldg(norm_w + i));
    __syncthreads();
}

enum : int { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };

struct GemvSeg {
    const uint8_t *w;
    int type;
    int rows;
    int out_off;
};

struct GemvParams {
    GemvSeg seg[3];
    int nseg;
    int tiles[3];  // CTAs per segment
    int cols;
    const float *x;
    const float *norm_w;
    float eps;
    float *y;                 // STORE: y[out_off + r]; SWIGLU: y[r]; ARGMAX: logits
    float *resid;             // RESID: resid[r] += acc (y null), or y[r] = resid[r] + acc (resid may be null)
    const uint8_t *w_up;      // SWIGLU: up matrix (same type as seg[0])
    // ARGMAX scratch and outputs
    float2 *am_part;          // [gridDim.x] (value, index bits)
    unsigned int *am_count;   // zero between launches
    int32_t *am_out;          // argmax result
    int32_t *adv_token;       // if non-null: next-step token <- argmax
    int32_t *adv_pos;         // if non-null: ++*adv_pos
    int32_t *rec_tokens;      // if non-null: rec_tokens[*rec_step] = argmax, ++*rec_step
    int32_t *rec_step;
};

template <int ROWS>
constexpr int tile_rows() { return ROWS * GEMV_WARPS; }

FDEV bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

template <int T, int EPI, int ROWS>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_kernel(const GemvParams p) {
    extern __shared__ float4 smem4[];
    float *xs = reinterpret_cast<float *>(smem4);
    __shared__ float red[32];
    __shared__ float2 am_warp[GEMV_WARPS];
    __shared__ unsigned int am_ticket;

    pdl_trigger();
    pdl_wait();
    // locate segment and tile
    int tile = blockIdx.x, s = 0;
    while (s + 1 < p.nseg && tile >= p.tiles[s]) tile -= p.tiles[s++];
    const GemvSeg sg = p.seg[s];

    stage_input(xs, p.x, p.cols, p.norm_w, p.eps, red);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = p.cols >> 8;
    const size_t row_bytes = (size_t)nb * RowDot<T>::BLOCK_BYTES;
    const int r0 = tile * tile_rows<ROWS>() + warp * ROWS;

    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
#pragma unroll
    for (int k = 0; k < ROWS; k++) {
        const int r = r0 + k;
        if (r >= sg.rows) break;
        float acc = warp_sum(RowDot<T>::run(sg.w + (size_t)r * row_bytes, xs, nb, lane));
        if constexpr (EPI == EPI_SWIGLU) {
            const float up = warp_sum(RowDot<T>::run(p.w_up + (size_t)r * row_bytes, xs, nb, lane));
            if (lane == 0) {
                const float sg_ = __fdiv_rn(acc, __fadd_rn(1.0f, expf(-acc)));
                p.y[r] = __fmul_rn(sg_, up);
            }
        } else if constexpr (EPI == EPI_RESID) {
            if (lane == 0) {
                // in place (y null): resid[r] += acc; out of place: y[r] = (resid ? resid[r] : 0) + acc
                float *dst = p.y ? p.y : p.resid;
                dst[r] = p.resid ? __fadd_rn(p.resid[r], acc) : acc;
            }
        } else if constexpr (EPI == EPI_ARGMAX) {
            if (lane == 0) p.y[r] = acc;
            if (better(acc, r, best_v, best_i)) {
                best_v = acc;
                best_i = r;
            }
        } else {
            if (lane == 0) p.y[sg.out_off + r] = acc;
        }
    }

    if constexpr (EPI == EPI_ARGMAX) {
        if (lane == 0) am_warp[warp] = make_float2(best_v, __int_as_float(best_i));
        __syncthreads();
        if (threadIdx.x == 0) {
            float bv = am_warp[0].x;
            int bi = __float_as_int(am_warp[0].y);
            for (int w = 1; w < GEMV_WARPS; w++) {
                const int wi = __float_as_int(am_warp[w].y);
                if (better(am_warp[w].x, wi, bv, bi)) {
                    bv = am_warp[w].x;
                    bi = wi;
                }
            }
            p.am_part[blockIdx.x] = make_float2(bv, __int_as_float(bi));
            __threadfence();
            am_ticket = atomicAdd(p.am_count, 1u);
        }
        __syncthreads();
        if (am_ticket == gridDim.x - 1) {  // last CTA reduces the partials
            __threadfence();
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) {
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
            if (threadIdx.x == 0) {
                for (int w = 1; w < GEMV_WARPS; w++) {
                    const int wi = __float_as_int(am_warp[w].y);
                    if (better(am_warp[w].x, wi, bv, bi)) {
                        bv = am_warp[w].x;
                        bi = wi;
                    }
                }
                if (bi == 0x7fffffff) bi = 0;  // all logits NaN: deterministic fallback
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

// Decoded weights for the bit-exactness checks: fp16 bits (Q4_K, Q6_K, F16) or fp32 (Q5_K).
template <int T>
__global__ void dequant_kernel(const uint8_t *__restrict__ w, void *out, int rows, int cols) {
    const int bpr = cols >> 8;
    const size_t total = (size_t)rows * cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / cols;
        const int c = (int)(i % cols);
        if constexpr (T == T_F16) {
            reinterpret_cast<uint16_t *>(out)[i] = reinterpret_cast<const uint16_t *>(w)[i];
        } else {
            constexpr int BB = RowDot<T>::BLOCK_BYTES;
            const uint8_t *blk = w + (r * bpr + (c >> 8)) * BB;
            const float v = decode_elem<T>(blk, c & 255);
            if constexpr (T == T_Q5_K)
                reinterpret_cast<float *>(out)[i] = v;
            else
                reinterpret_cast<uint16_t *>(out)[i] = __half_as_ushort(__float2half_rn(v));
        }
    }
}

}  // namespace fiber
