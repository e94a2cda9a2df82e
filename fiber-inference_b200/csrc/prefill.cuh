// prefill.cuh — the non-GEMM kernels of a batched layer pass: n tokens in one pass per
// layer, either a prompt chunk of one sequence (positions start .. start + n - 1, one
// KV slot) or one decode step of n sequences (token t at position pos[t] in KV slot
// t). The projections run on the tensor cores (gemm_tc5.cuh); these kernels do the
// per-token parts with the decode path's arithmetic (the RMSNorms are folded into the
// GEMM's input packing):
//   embed_rows_kernel   embedding rows of the n tokens (fp16-rounded, as gpu_embed)
//   rope_kv_kernel      half-split RoPE of q (in place) and k; K/V appended (fp16)
//   attn_prefill_kernel causal GQA attention of each token over the cache
//   swiglu_rows_kernel  h = silu(gate) * up
//   argmax_rows_kernel  greedy token of each logits row (lowest index on ties)
//   batch_advance_kernel  device-resident greedy loop: argmax -> next token, pos + 1
#pragma once
#include "attention.cuh"

namespace fiber {

template <int T>
__global__ void embed_rows_kernel(const uint8_t *__restrict__ tab, const int32_t *__restrict__ tokens, float *X,
                                  int dim, int vocab, int *err) {
    const int t = blockIdx.y;
    int tok = tokens[t];
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
            v = round_f16(decode_elem<T>(tab + ((size_t)tok * (dim >> 8) + (i >> 8)) * BB, i & 255));
        }
        X[(size_t)t * dim + i] = v;
    }
}

// Where token t of a pass sits: position pos[t] (or start + t) of KV slot
// slot + slot_step * t; page tables are [slot][max_pages].
struct TokenPlace {
    int start;             // position of token 0 when pos is null
    const int32_t *pos;    // [n] per-token positions, or null
    int slot, slot_step, max_pages;
    int max_pos;           // positions must stay below this (cache and RoPE table)
    int *err;              // set to 3 for a position outside [0, max_pos)
};

FDEV int place_pos(const TokenPlace &p, int t) { return p.pos ? p.pos[t] : p.start + t; }
FDEV const int32_t *place_pages(const TokenPlace &p, const int32_t *page_table, int t) {
    return page_table + (size_t)(p.slot + p.slot_step * t) * p.max_pages;
}

struct RopeKvParams {
    float *qkv;            // [n][ldq]: q | k | v of each token (q rotated in place)
    int ldq;
    TokenPlace at;
    const float2 *rope;    // [max_seq][hd/2]
    int n_heads, n_kv, hd;
    uint16_t *k_pool, *v_pool;
    const int32_t *page_table;
    int layer, n_layers;
};

// One CTA per token: rotate q and k (the decode path's expressions), store K and V.
__global__ void rope_kv_kernel(const RopeKvParams a) {
    const int t = blockIdx.x, pos = place_pos(a.at, t), hd = a.hd, half = hd / 2;
    if (pos < 0 || pos >= a.at.max_pos) {
        if (threadIdx.x == 0) *a.at.err = 3;
        return;
    }
    float *q = a.qkv + (size_t)t * a.ldq;
    const float *k = q + (size_t)a.n_heads * hd, *v = k + (size_t)a.n_kv * hd;
    const float2 *rp = a.rope + (size_t)pos * half;
    const int32_t *pages = place_pages(a.at, a.page_table, t);
    for (int i = threadIdx.x; i < a.n_heads * half; i += blockDim.x) {
        const int h = i / half, j = i % half;
        const float2 cs = rp[j];
        const float x1 = q[h * hd + j], x2 = q[h * hd + j + half];
        q[h * hd + j] = __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y));
        q[h * hd + j + half] = __fadd_rn(__fmul_rn(x1, cs.y), __fmul_rn(x2, cs.x));
    }
    const int page = pages[pos / ATTN_P], tn = pos % ATTN_P;
    for (int i = threadIdx.x; i < a.n_kv * half; i += blockDim.x) {
        const int g = i / half, j = i % half;
        const float2 cs = rp[j];
        const float x1 = k[g * hd + j], x2 = k[g * hd + j + half];
        uint16_t *kp = a.k_pool + ((((size_t)page * a.n_layers + a.layer) * a.n_kv + g) * ATTN_P + tn) * hd;
        kp[j] = __half_as_ushort(__float2half_rn(__fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y))));
        kp[j + half] = __half_as_ushort(__float2half_rn(__fadd_rn(__fmul_rn(x1, cs.y), __fmul_rn(x2, cs.x))));
    }
    for (int i = threadIdx.x; i < a.n_kv * hd; i += blockDim.x) {
        const int g = i / hd, d = i % hd;
        uint16_t *vp = a.v_pool + ((((size_t)page * a.n_layers + a.layer) * a.n_kv + g) * ATTN_P + tn) * hd;
        vp[d] = __half_as_ushort(__float2half_rn(v[g * hd + d]));
    }
}

struct AttnPrefillParams {
    const float *qkv;      // [n][ldq], q rotated
    int ldq;
    float *out;            // [n][ldo]
    int ldo;
    TokenPlace at;
    const uint16_t *k_pool, *v_pool;
    const int32_t *page_table;
    int layer, n_layers, n_kv, n_heads;
    float scale;
    // page split (gridDim.z = psplit > 1): CTA z takes pages [z P', (z+1) P') of the
    // token's context, P' = ceil(pages / psplit); it writes its softmax state (max, sum,
    // unnormalised output per head) to part, and the last CTA of (token, KV head)
    // (ticket) merges the psplit states in split order
    float *part;            // [n][n_kv][psplit][G][HD + 2]
    unsigned int *tickets;  // [n][n_kv], zero between launches
};

// One page (nt <= 64 positions, staged in ks / vs) for one query vector q (shared
// memory, HD floats), on one warp: scores (lanes over positions, fp32 FMAs over fp16 K),
// page max and sum, P.V, then the online merge into the running (m, l, o) state
// (first: the state starts here).
template <int HD>
FDEV void apf_page(const float *q, const uint16_t (*ks)[HD + 2], const uint16_t (*vs)[HD], int nt, float scale,
                   int lane, bool first, float &m_run, float &l_run, float (&o_run)[HD / 32]) {
    constexpr int DPL = HD / 32;
    float sc2[2];
#pragma unroll
    for (int k = 0; k < 2; k++) {
        const int r = lane + 32 * k;
        float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
        if (r < nt) {
#pragma unroll
            for (int d = 0; d < HD; d += 4) {
                d0 = fmaf(q[d + 0], __half2float(__ushort_as_half(ks[r][d + 0])), d0);
                d1 = fmaf(q[d + 1], __half2float(__ushort_as_half(ks[r][d + 1])), d1);
                d2 = fmaf(q[d + 2], __half2float(__ushort_as_half(ks[r][d + 2])), d2);
                d3 = fmaf(q[d + 3], __half2float(__ushort_as_half(ks[r][d + 3])), d3);
            }
        }
        sc2[k] = r < nt ? __fmul_rn((d0 + d1) + (d2 + d3), scale) : -INFINITY;
    }
    float m = fmaxf(sc2[0], sc2[1]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float e0 = lane < nt ? expf(sc2[0] - m) : 0.f;
    const float e1 = lane + 32 < nt ? expf(sc2[1] - m) : 0.f;
    float l = e0 + e1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    float o1[DPL], o2[DPL];
#pragma unroll
    for (int j = 0; j < DPL; j++) o1[j] = o2[j] = 0.f;
    for (int r = 0; r < min(nt, 32); r++) {
        const float w = __shfl_sync(0xffffffffu, e0, r);
#pragma unroll
        for (int j = 0; j < DPL; j++) o1[j] = fmaf(w, __half2float(__ushort_as_half(vs[r][lane + 32 * j])), o1[j]);
    }
    for (int r = 32; r < nt; r++) {
        const float w = __shfl_sync(0xffffffffu, e1, r - 32);
#pragma unroll
        for (int j = 0; j < DPL; j++) o2[j] = fmaf(w, __half2float(__ushort_as_half(vs[r][lane + 32 * j])), o2[j]);
    }
    if (first) {
        m_run = m;
        l_run = l;
#pragma unroll
        for (int j = 0; j < DPL; j++) o_run[j] = o1[j] + o2[j];
    } else {
        const float M = fmaxf(m_run, m);
        const float al = expf(m_run - M), be = expf(m - M);
        l_run = fmaf(al, l_run, be * l);
#pragma unroll
        for (int j = 0; j < DPL; j++) o_run[j] = fmaf(al, o_run[j], be * (o1[j] + o2[j]));
        m_run = M;
    }
}

// CTA (token t, KV head g[, page split z]): the G query heads of g attend to positions
// 0 .. pos(t) of the token's slot, page by page (64 positions) with the decode path's
// score / softmax / P.V arithmetic, pages combined online.
template <int HD, int G>
__global__ void __launch_bounds__(ATTN_THREADS) attn_prefill_kernel(const AttnPrefillParams a) {
    constexpr int P = ATTN_P, KST = HD + 2, DPL = HD / 32;
    __shared__ __align__(16) float qs[G][HD];
    __shared__ __align__(16) uint16_t ks[P][KST];
    __shared__ __align__(16) uint16_t vs[P][HD];
    const int t = blockIdx.x, g = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int pos = place_pos(a.at, t);
    if (pos < 0 || pos >= a.at.max_pos) return;  // rope_kv_kernel reported it
    const int seqlen = pos + 1, nch = (seqlen + P - 1) / P;
    const int32_t *pages = place_pages(a.at, a.page_table, t);
    const int ps = gridDim.z, z = blockIdx.z, per = (nch + ps - 1) / ps;
    const int cbeg = min(nch, z * per), cend = min(nch, cbeg + per);
    for (int i = tid; i < G * HD; i += ATTN_THREADS)
        qs[i / HD][i % HD] = a.qkv[(size_t)t * a.ldq + (size_t)(g * G + i / HD) * HD + i % HD];
    float m_run = -INFINITY, l_run = 0.f, o_run[DPL];
#pragma unroll
    for (int j = 0; j < DPL; j++) o_run[j] = 0.f;
    __syncthreads();  // qs staged
    for (int c = cbeg; c < cend; c++) {
        __syncthreads();  // previous page consumed
        const int t0 = c * P, nt = min(P, seqlen - t0);
        const size_t base = (((size_t)pages[c] * a.n_layers + a.layer) * a.n_kv + g) * (size_t)P * HD;
        constexpr int V8 = HD / 8;
        for (int i = tid; i < nt * V8; i += ATTN_THREADS) {
            const int r = i / V8, k8 = i % V8;
            const uint4 kv4 = *reinterpret_cast<const uint4 *>(a.k_pool + base + (size_t)r * HD + 8 * k8);
            const uint4 vv4 = *reinterpret_cast<const uint4 *>(a.v_pool + base + (size_t)r * HD + 8 * k8);
            uint32_t *kd = reinterpret_cast<uint32_t *>(&ks[r][8 * k8]);
            kd[0] = kv4.x; kd[1] = kv4.y; kd[2] = kv4.z; kd[3] = kv4.w;
            *reinterpret_cast<uint4 *>(&vs[r][8 * k8]) = vv4;
        }
        __syncthreads();
        for (int h = warp; h < G; h += ATTN_THREADS / 32)  // warp h keeps head h's state
            apf_page<HD>(qs[h], ks, vs, nt, a.scale, lane, c == cbeg, m_run, l_run, o_run);
    }
    if (ps == 1) {
        if (warp < G)
#pragma unroll
            for (int j = 0; j < DPL; j++)
                a.out[(size_t)t * a.ldo + (size_t)(g * G + warp) * HD + lane + 32 * j] = o_run[j] / l_run;
        return;
    }
    constexpr int ST = HD + 2;  // one head's state: max, sum, output
    float *mine = a.part + (((size_t)t * a.n_kv + g) * ps + z) * (G * ST);
    if (warp < G) {
#pragma unroll
        for (int j = 0; j < DPL; j++) mine[warp * ST + 2 + lane + 32 * j] = o_run[j];
        if (lane == 0) {
            mine[warp * ST] = m_run;
            mine[warp * ST + 1] = l_run;
        }
    }
    __syncthreads();
    __shared__ int last;
    unsigned int *ticket = a.tickets + (size_t)t * a.n_kv + g;
    if (tid == 0) {
        __threadfence();
        last = atomicAdd(ticket, 1u) == (unsigned int)(ps - 1);
        if (last) __threadfence();
    }
    __syncthreads();
    if (!last) return;
    if (warp < G) {
        const float *all = a.part + ((size_t)t * a.n_kv + g) * ps * (G * ST) + warp * ST;
        float M = -INFINITY;
        for (int q = 0; q < ps; q++) M = fmaxf(M, __ldcg(all + (size_t)q * G * ST));
        float L = 0.f, o[DPL];
#pragma unroll
        for (int j = 0; j < DPL; j++) o[j] = 0.f;
        for (int q = 0; q < ps; q++) {
            const float *st = all + (size_t)q * G * ST;
            const float mq = __ldcg(st);
            if (mq == -INFINITY) continue;  // a split without pages
            const float w = expf(mq - M);
            L = fmaf(w, __ldcg(st + 1), L);
#pragma unroll
            for (int j = 0; j < DPL; j++) o[j] = fmaf(w, __ldcg(st + 2 + lane + 32 * j), o[j]);
        }
#pragma unroll
        for (int j = 0; j < DPL; j++) a.out[(size_t)t * a.ldo + (size_t)(g * G + warp) * HD + lane + 32 * j] = o[j] / L;
    }
    if (tid == 0) *ticket = 0u;
}

// Prompt chunks (every token of one KV slot, consecutive positions) of models with
// fewer than 8 query heads per KV head: CTA (block of TB consecutive tokens, KV head g). Each page is staged once for the block; the G x TB
// (query head, token) pairs are spread over the 8 warps (pair p: token p / G, head
// p % G; warp w takes pairs w, w + 8, ...), each pair with apf_page's arithmetic in the
// same page order as attn_prefill_kernel, so the outputs are the same bit for bit.
// Tokens per block: 8 / G, so that each warp holds one (head, token) pair (the work per
// warp stays that of attn_prefill_kernel and the freed warps take more tokens), as far as
// the q vectors fit the 48 KB of static shared memory next to one K and one V page.
HDCE int apf_tb(int hd, int g) {
    const int page = ATTN_P * (hd + 2) * 2 + ATTN_P * hd * 2, free_b = 48 * 1024 - page;
    int tb = 8 / g;
    while (tb > 1 && tb * g * hd * 4 > free_b) tb >>= 1;
    return tb;
}

template <int HD, int G, int TB>
__global__ void __launch_bounds__(ATTN_THREADS) attn_prefill_tb_kernel(const AttnPrefillParams a, int n) {
    constexpr int P = ATTN_P, KST = HD + 2, DPL = HD / 32, NW = ATTN_THREADS / 32;
    constexpr int PAIRS = G * TB, PPW = (PAIRS + NW - 1) / NW;
    __shared__ __align__(16) float qs[TB][G][HD];
    __shared__ __align__(16) uint16_t ks[P][KST];
    __shared__ __align__(16) uint16_t vs[P][HD];
    const int t0 = blockIdx.x * TB, g = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nvalid = min(TB, n - t0);
    const int pos0 = place_pos(a.at, t0), posl = pos0 + nvalid - 1;
    if (pos0 < 0 || posl >= a.at.max_pos) return;  // rope_kv_kernel reported it
    const int nch = (posl + 1 + P - 1) / P;
    const int32_t *pages = place_pages(a.at, a.page_table, t0);
    for (int i = tid; i < nvalid * G * HD; i += ATTN_THREADS) {
        const int tt = i / (G * HD), h = (i / HD) % G, d = i % HD;
        qs[tt][h][d] = a.qkv[(size_t)(t0 + tt) * a.ldq + (size_t)(g * G + h) * HD + d];
    }
    float m_run[PPW], l_run[PPW], o_run[PPW][DPL];
#pragma unroll
    for (int q = 0; q < PPW; q++) {
        m_run[q] = -INFINITY;
        l_run[q] = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; j++) o_run[q][j] = 0.f;
    }
    __syncthreads();  // qs staged
    for (int c = 0; c < nch; c++) {
        __syncthreads();  // previous page consumed
        const int p0 = c * P, nt = min(P, posl + 1 - p0);
        const size_t base = (((size_t)pages[c] * a.n_layers + a.layer) * a.n_kv + g) * (size_t)P * HD;
        constexpr int V8 = HD / 8;
        for (int i = tid; i < nt * V8; i += ATTN_THREADS) {
            const int r = i / V8, k8 = i % V8;
            const uint4 kv4 = *reinterpret_cast<const uint4 *>(a.k_pool + base + (size_t)r * HD + 8 * k8);
            const uint4 vv4 = *reinterpret_cast<const uint4 *>(a.v_pool + base + (size_t)r * HD + 8 * k8);
            uint32_t *kd = reinterpret_cast<uint32_t *>(&ks[r][8 * k8]);
            kd[0] = kv4.x; kd[1] = kv4.y; kd[2] = kv4.z; kd[3] = kv4.w;
            *reinterpret_cast<uint4 *>(&vs[r][8 * k8]) = vv4;
        }
        __syncthreads();
#pragma unroll
        for (int q = 0; q < PPW; q++) {
            const int pr = warp + q * NW, tt = pr / G, h = pr % G;
            if (pr >= PAIRS || tt >= nvalid) continue;
            const int ntt = min(P, pos0 + tt + 1 - p0);  // this token's causal limit in the page
            if (ntt <= 0) continue;                      // page entirely after this token
            apf_page<HD>(qs[tt][h], ks, vs, ntt, a.scale, lane, c == 0, m_run[q], l_run[q], o_run[q]);
        }
    }
#pragma unroll
    for (int q = 0; q < PPW; q++) {
        const int pr = warp + q * NW, tt = pr / G, h = pr % G;
        if (pr >= PAIRS || tt >= nvalid) continue;
#pragma unroll
        for (int j = 0; j < DPL; j++)
            a.out[(size_t)(t0 + tt) * a.ldo + (size_t)(g * G + h) * HD + lane + 32 * j] = o_run[q][j] / l_run[q];
    }
}

__global__ void swiglu_rows_kernel(float *hg, const float *__restrict__ hu, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float g = hg[i];
        hg[i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), hu[i]);
    }
}

// One CTA (256 threads) per row: index of the maximum, the lowest index winning ties
// (the strict > scan of the reference sampler, src/sampler.c:38-46). NaN never wins.
__global__ void __launch_bounds__(256) argmax_rows_kernel(const float *__restrict__ logits, int V, int ld,
                                                          int32_t *arg) {
    __shared__ float bv[8];
    __shared__ int bi[8];
    const float *row = logits + (size_t)blockIdx.x * ld;
    float best = -INFINITY;
    int idx = V;  // larger than every index: "none yet"
    for (int i = threadIdx.x; i < V; i += 256) {
        const float v = row[i];
        if (v > best) {  // a thread visits indices in increasing order: ties keep the first
            best = v;
            idx = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > best || (ov == best && oi < idx)) {
            best = ov;
            idx = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        bv[threadIdx.x >> 5] = best;
        bi[threadIdx.x >> 5] = idx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; w++)
            if (bv[w] > best || (bv[w] == best && bi[w] < idx)) {
                best = bv[w];
                idx = bi[w];
            }
        arg[blockIdx.x] = idx < V ? idx : 0;  // all NaN / -inf: token 0
    }
}

// Device-resident greedy loop over n sequences: token[t] <- arg[t], pos[t] + 1, and the
// token recorded at rec[step * n + t]; one CTA, then the step counter advances.
__global__ void batch_advance_kernel(const int32_t *arg, int32_t *tokens, int32_t *pos, int32_t *rec, int *step,
                                     int n) {
    const int s = *step;
    for (int t = threadIdx.x; t < n; t += blockDim.x) {
        const int32_t a = arg[t];
        tokens[t] = a;
        pos[t] += 1;
        rec[(size_t)s * n + t] = a;
    }
    __syncthreads();
    if (threadIdx.x == 0) *step = s + 1;
}

}  // namespace fiber
