// attention.cuh — GQA decode attention over the paged fp16 KV cache, with the
// RoPE of q/k and the KV append of the new position fused in.
//
// Reference semantics (metal/kernels.metal:374-504, src/fiber_proof.m:30-51,
// 79-109): half-split RoPE on pairs (i, i + hd/2) with angle pos * theta^(-2i/hd);
// K/V of the new position stored at `pos`; per query head h (kv head
// h * n_kv / n_heads) softmax(q.K_t * 1/sqrt(hd)) over t <= pos, then sum p_t V_t.
//
// Split-K (flash-decoding): CTA (chunk c, kv head g) handles the page of
// positions [c*P, c*P + P) for all G = n_heads / n_kv query heads sharing g, so
// each K/V page is read from HBM once per step. It writes (max, sum, o[hd]) per
// head to scratch; the last CTA of each kv head (atomic ticket) merges the
// chunks into the output. Dot products q.K and the RoPE rotations use the
// reference's operation order with unfused multiplies and adds, so for equal
// inputs the scores are bit-identical to the CPU path.
#pragma once
#include "quant.cuh"

namespace fiber {

struct AttnParams {
    const float *qkv;         // q [n_heads*hd] | k [n_kv*hd] | v [n_kv*hd], unrotated
    const float2 *rope;       // [max_seq][hd/2] (cos, sin), computed on the host like the CPU path
    uint16_t *k_pool;         // fp16 bits, [page][layer][kv_head][P][hd]
    uint16_t *v_pool;
    const int32_t *page_table;  // [max_pages] for this sequence slot
    const int32_t *pos_ptr;   // current position (device)
    float *part;              // [n_kv][max_chunks][G][hd + 2]
    unsigned int *count;      // [n_kv], zero between launches
    float *out;               // [n_heads * hd]
    int layer, n_layers, n_kv, n_heads, max_chunks, max_seq;
    float scale;
    int *err;                 // set to 1 when pos is out of range
};

constexpr int ATTN_THREADS = 256;  // 8 warps
constexpr int ATTN_P = 64;         // positions per page / chunk
constexpr int ATTN_MAX_CHUNKS = 512;

struct SyncThreads {
    FDEV void operator()() const { __syncthreads(); }
};

// Shared memory one attention unit needs (qs, padded K rows, V rows).
template <int HD, int G>
constexpr int attn_smem_bytes() {
    return G * HD * 4 + ATTN_P * (HD + 2) * 2 + ATTN_P * HD * 2;
}

// One (chunk c, kv head g) unit, run by ATTN_THREADS threads synchronised by
// `bar`: warps own query heads (G <= 8: one head per warp, lanes over positions
// for q.K and over head dims for P.V, softmax by shuffles); the chunk-local
// (max, sum, o[hd]) go to scratch and the last unit of the kv head merges all
// chunks, loading every partial it needs at once.
template <int HD, int G, class Bar>
FDEV void attn_unit(const AttnParams &a, int c, int g, int pos, uint8_t *sm, unsigned int *ticket, Bar bar) {
    constexpr int P = ATTN_P;
    constexpr int KST = HD + 2;   // padded K row (halves): lanes walking d stay on distinct banks
    constexpr int DPL = HD / 32;  // head dims per lane in P.V
    float(*qs)[HD] = reinterpret_cast<float(*)[HD]>(sm);
    uint16_t(*ks)[KST] = reinterpret_cast<uint16_t(*)[KST]>(sm + G * HD * 4);
    uint16_t(*vs)[HD] = reinterpret_cast<uint16_t(*)[HD]>(sm + G * HD * 4 + P * KST * 2);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int seq = pos + 1;
    const int nch = (seq + P - 1) / P;
    const int t0 = c * P;
    const int nt = min(P, seq - t0);
    const int kvd = a.n_kv * HD;
    const float2 *rp = a.rope + (size_t)pos * (HD / 2);

    // rotated queries of the G heads of this group (half-split pairs)
    for (int i = tid; i < G * (HD / 2); i += ATTN_THREADS) {
        const int h = i / (HD / 2), j = i % (HD / 2);
        const float *qh = a.qkv + (size_t)(g * G + h) * HD;
        const float x1 = __ldcg(qh + j), x2 = __ldcg(qh + j + HD / 2);
        const float2 cs = __ldg(rp + j);
        qs[h][j] = __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y));
        qs[h][j + HD / 2] = __fadd_rn(__fmul_rn(x1, cs.y), __fmul_rn(x2, cs.x));
    }

    const int page = a.page_table[c];
    const size_t base = (((size_t)page * a.n_layers + a.layer) * a.n_kv + g) * (size_t)P * HD;
    uint16_t *kp = a.k_pool + base, *vp = a.v_pool + base;

    // the chunk holding `pos` appends the new K (rotated) and V, rounded to fp16
    if (c == nch - 1) {
        const int tn = pos - t0;
        const float *kr = a.qkv + (size_t)a.n_heads * HD + (size_t)g * HD;
        const float *vr = a.qkv + (size_t)a.n_heads * HD + kvd + (size_t)g * HD;
        for (int j = tid; j < HD / 2; j += ATTN_THREADS) {
            const float x1 = __ldcg(kr + j), x2 = __ldcg(kr + j + HD / 2);
            const float2 cs = __ldg(rp + j);
            const float y1 = __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y));
            const float y2 = __fadd_rn(__fmul_rn(x1, cs.y), __fmul_rn(x2, cs.x));
            kp[(size_t)tn * HD + j] = __half_as_ushort(__float2half_rn(y1));
            kp[(size_t)tn * HD + j + HD / 2] = __half_as_ushort(__float2half_rn(y2));
        }
        for (int j = tid; j < HD; j += ATTN_THREADS) vp[(size_t)tn * HD + j] = __half_as_ushort(__float2half_rn(__ldcg(vr + j)));
        bar();  // unit-wide visibility of the appended row
    }

    // stage the chunk: K with padded rows, V dense (16-byte loads)
    constexpr int V8 = HD / 8;
    for (int i = tid; i < nt * V8; i += ATTN_THREADS) {
        const int t = i / V8, k8 = i % V8;
        const uint4 kv4 = __ldcg(reinterpret_cast<const uint4 *>(kp + (size_t)t * HD) + k8);
        const uint4 vv4 = __ldcg(reinterpret_cast<const uint4 *>(vp + (size_t)t * HD) + k8);
        uint32_t *kd = reinterpret_cast<uint32_t *>(&ks[t][8 * k8]);
        kd[0] = kv4.x; kd[1] = kv4.y; kd[2] = kv4.z; kd[3] = kv4.w;
        *reinterpret_cast<uint4 *>(&vs[t][8 * k8]) = vv4;
    }
    bar();

    float *pg = a.part + (size_t)g * a.max_chunks * G * (HD + 2);
    for (int h = warp; h < G; h += ATTN_THREADS / 32) {
        // scores for positions lane and lane+32; four interleaved partial sums
        float s[2];
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const int t = lane + 32 * k;
            float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
            if (t < nt) {
#pragma unroll
                for (int d = 0; d < HD; d += 4) {
                    d0 = fmaf(qs[h][d + 0], __half2float(__ushort_as_half(ks[t][d + 0])), d0);
                    d1 = fmaf(qs[h][d + 1], __half2float(__ushort_as_half(ks[t][d + 1])), d1);
                    d2 = fmaf(qs[h][d + 2], __half2float(__ushort_as_half(ks[t][d + 2])), d2);
                    d3 = fmaf(qs[h][d + 3], __half2float(__ushort_as_half(ks[t][d + 3])), d3);
                }
            }
            s[k] = t < nt ? __fmul_rn((d0 + d1) + (d2 + d3), a.scale) : -INFINITY;
        }
        float m = fmaxf(s[0], s[1]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float e0 = lane < nt ? expf(s[0] - m) : 0.f;
        const float e1 = lane + 32 < nt ? expf(s[1] - m) : 0.f;
        float l = e0 + e1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        // P.V: lane owns dims lane + 32*j; position weights come by shuffle
        float o[DPL], o2[DPL];
#pragma unroll
        for (int j = 0; j < DPL; j++) o[j] = o2[j] = 0.f;
        const int n0 = min(nt, 32);
        for (int t = 0; t < n0; t++) {
            const float w = __shfl_sync(0xffffffffu, e0, t);
#pragma unroll
            for (int j = 0; j < DPL; j++) o[j] = fmaf(w, __half2float(__ushort_as_half(vs[t][lane + 32 * j])), o[j]);
        }
        for (int t = 32; t < nt; t++) {
            const float w = __shfl_sync(0xffffffffu, e1, t - 32);
#pragma unroll
            for (int j = 0; j < DPL; j++) o2[j] = fmaf(w, __half2float(__ushort_as_half(vs[t][lane + 32 * j])), o2[j]);
        }
        float *pc = pg + ((size_t)c * G + h) * (HD + 2);
#pragma unroll
        for (int j = 0; j < DPL; j++) pc[2 + lane + 32 * j] = o[j] + o2[j];
        if (lane == 0) {
            pc[0] = m;
            pc[1] = l;
        }
    }
    __threadfence();
    bar();
    if (tid == 0) *ticket = atomicAdd(a.count + g, 1u);
    bar();
    const bool last = *ticket == (unsigned)(nch - 1);
    if (last) {
        // last unit of this kv head: merge the nch chunks of every head (warp per head)
        __threadfence();
        for (int h = warp; h < G; h += ATTN_THREADS / 32) {
            float M = -INFINITY;
            for (int k = lane; k < nch; k += 32) M = fmaxf(M, __ldcg(pg + ((size_t)k * G + h) * (HD + 2)));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            float Lsum = 0.f;
            float O[DPL];
#pragma unroll
            for (int j = 0; j < DPL; j++) O[j] = 0.f;
            for (int k0 = 0; k0 < nch; k0 += 32) {
                const int kk = k0 + lane;
                float w = 0.f;
                if (kk < nch) {
                    const float *e = pg + ((size_t)kk * G + h) * (HD + 2);
                    w = expf(__ldcg(e) - M);
                    Lsum = fmaf(w, __ldcg(e + 1), Lsum);
                }
                const int kn = min(32, nch - k0);
#pragma unroll 4
                for (int k = 0; k < kn; k++) {
                    const float wk = __shfl_sync(0xffffffffu, w, k);
                    const float *e = pg + ((size_t)(k0 + k) * G + h) * (HD + 2) + 2;
#pragma unroll
                    for (int j = 0; j < DPL; j++) O[j] = fmaf(wk, __ldcg(e + lane + 32 * j), O[j]);
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) Lsum += __shfl_xor_sync(0xffffffffu, Lsum, o);
#pragma unroll
            for (int j = 0; j < DPL; j++) a.out[(size_t)(g * G + h) * HD + lane + 32 * j] = O[j] / Lsum;
        }
        if (tid == 0) a.count[g] = 0u;
    }
    bar();  // shared memory and the ticket are reused by the next unit
}

template <int HD, int G>
__global__ void __launch_bounds__(ATTN_THREADS) attn_decode_kernel(const AttnParams a) {
    __shared__ __align__(16) uint8_t sm[attn_smem_bytes<HD, G>()];
    __shared__ unsigned int ticket;
    pdl_trigger();
    pdl_wait();
    const int pos = *a.pos_ptr;
    if (pos < 0 || pos >= a.max_seq) {
        if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *a.err = 1;
        return;
    }
    const int nch = (pos + ATTN_P) / ATTN_P;
    if ((int)blockIdx.x >= nch) return;
    attn_unit<HD, G>(a, blockIdx.x, blockIdx.y, pos, sm, &ticket, SyncThreads());
}

// Embedding row of `*token` (fp16-rounded like the reference's fp16 buf_x,
// src/gpu_ffn.m:466-482) into the fp32 residual stream.
template <int T>
__global__ void embed_kernel(const uint8_t *__restrict__ tab, const int32_t *__restrict__ token, float *x, int dim,
                             int vocab, int *err) {
    pdl_trigger();
    pdl_wait();
    int tok = *token;
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) *err = 2;
        tok = 0;
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x) {
        float v;
        if constexpr (T == T_F16) {
            v = h2f(reinterpret_cast<const uint16_t *>(tab)[(size_t)tok * dim + i]);
        } else if constexpr (T == T_F32) {
            v = round_f16(reinterpret_cast<const float *>(tab)[(size_t)tok * dim + i]);
        } else {
            constexpr int BB = T == T_Q4_K ? 144 : (T == T_Q5_K ? 176 : 210);
            const uint8_t *blk = tab + ((size_t)tok * (dim >> 8) + (i >> 8)) * BB;
            v = round_f16(decode_elem<T>(blk, i & 255));
        }
        x[i] = v;
    }
}

}  // namespace fiber
