// flow.cuh — one decode step as one cooperative kernel whose phases hand their
// results to each other as tagged words instead of meeting at grid barriers.
//
// A phase's output vector (q|k|v, the attention output, the residual stream, the
// SwiGLU activations) is written as 8-byte words (fp32 value in the low half, the
// launch's tag in the high half) with single 64-bit stores; a consumer polls the
// words it needs and takes each one as soon as it carries this launch's tag. So a
// phase waits only for the data it reads (one L2 round trip after the last
// producer's store), never for every CTA of the grid, and needs no separate
// flag, fence or staging copy. Every output word of a step is written exactly
// once per launch (one buffer per layer and kind), so a word can only be stale
// from an earlier launch, whose tag differs.
//
// Per CTA (one per SM, all co-resident: cooperative launch):
//   * warp 8, one lane (producer): streams this CTA's weight tiles of every phase,
//     and the K/V pages of its attention unit, with cp.async.bulk into a byte ring
//     in shared memory (FIFO, full/empty mbarrier pair per slot), in consumption
//     order, so loading runs ahead across phases and waits;
//   * warps 0..7 (consumers), per GEMV phase: poll the input words, RMSNorm them
//     where the phase has one, scale by a power of two (keeps the fp16 hi/lo split
//     in range for any activation size), write the MMA fragments; then per tile
//     every warp decodes and multiplies its super-blocks (TcDot) and writes its
//     partial sums; the last warp to finish a tile (shared-memory ticket) sums the
//     eight partials, applies the epilogue (residual add, SwiGLU, logits + argmax
//     candidate) and stores the output words — no CTA barrier per tile;
//   * attention: one unit per (KV head, page split) with all query heads of the
//     group, so K/V pages are read once per group; split states are merged in
//     split order by the last unit to finish (ticket).
// Every wait is bounded (%globaltimer); on timeout the kernel records error 4,
// stops issuing work and returns once its own copies have landed.
#pragma once
#include <cuda.h>

#include "persistent.cuh"

namespace fiber {

constexpr int FL_WARPS = 8;
constexpr int FL_CONSUMERS = FL_WARPS * 32;
// + a producer warpgroup (warps 8..11): lane 0 of warp 8 streams the ring, warp 9 runs
// the tile epilogues. With 12 warps the launch gives every thread 168 registers (three
// warps share each SM sub-partition's register file); the producer group then drops to
// FL_REG_PRODUCER and the consumer warps rise to FL_REG_CONSUMER (setmaxnreg):
// 4 x 32 x 56 + 8 x 32 x 224 = 12 x 32 x 168, exactly the launch's registers.
constexpr int FL_THREADS = FL_CONSUMERS + 128;
constexpr int FL_EPI_WARP = FL_WARPS + 1;
constexpr int FL_REG_PRODUCER = 56, FL_REG_CONSUMER = 224;
static_assert(4 * 32 * FL_REG_PRODUCER + 8 * 32 * FL_REG_CONSUMER <= FL_THREADS * 168, "register split");
constexpr int FL_NDESC = 16;                   // ring slots
constexpr int FL_MAX_TP = 8;                   // tensor-parallel ranks at most
constexpr unsigned long long FL_WAIT_NS = 2000000000ull;
constexpr int FL_RING_PAD = 1024;              // the ring starts at the first 1024-byte boundary (swizzled copies)
// Optional per-phase, per-CTA timeline (FParams::trace non-null), fields:
//  0 globaltimer (ns) at the phase start   1 cycles polling the input words
//  2 cycles RMSNorm + fragments            3 cycles from the tiles' start to the phase end
//  4 cycles warp 0 waited for ring slots   5 globaltimer (ns) at the phase end
//  6 producer: globaltimer after issuing the phase's last copy   7 producer: cycles waiting for ring space
//  attention units: 1 cycles polling q|k|v   2 RoPE, K/V append, q fragments
//  8 cycles of the page loop   9 cycles merging (warps, then splits: includes polling them)
//  GEMV phases: 10 globaltimer when the last warp had staged its input chunks
//               11 globaltimer after the last tile epilogue of this CTA
//  attention units (warp 0): 12 cycles acquiring pages  13 cycles of q.K  14 cycles of the
//               softmax  15 cycles of P.V
//  GEMV phases: 11 globaltimer after the last tile epilogue of this CTA (epilogue warp)
//               12 cycles warp 0 spent in its tile dot products  13 cycles publishing them
//               15 tiles of warp 0; epilogue warp: 8 cycles waiting for partial sums,
//               9 cycles in epilogues, 14 globaltimer when it started the phase
constexpr int FL_TRACE_FIELDS = 16;

enum : int { FL_QKV = 0, FL_ATTN = 1, FL_RESID = 2, FL_SWIGLU = 3, FL_LM = 4 };

struct __align__(16) FPhase {
    int kind;
    int nseg;
    int nmat;        // 2 for SwiGLU (a tile: 8 rows of gate, then the same 8 rows of up), else 1
    int cols;        // input length
    int layer;
    int n_tiles;
    int embed_in;    // layer 0 QKV: the input is the embedding row of the current token
    int stage_ctas;  // CTAs below this stage the input (they have tiles here, or keep it for the next residual phase)
    float eps;
    int tp_sum;      // tensor parallel, norm phase: the input is x (the residual kept by the last norm
                     // phase) plus every rank's partial sums, `in` = [world][cols] words in rank order
    const uint64_t *in;    // tagged input words (cols of them); null for the embedding input
    const float *norm_w;   // RMSNorm weights of the input, or null
    uint64_t *out;         // tagged output words (QKV: q|k|v, ATTN: attention, RESID: x, SWIGLU: h)
    float *logits;         // LM: fp32 logits
    long long tp_off;      // tensor parallel, residual phase: word offset of its [world][rows] partial
                           // sums in every rank's exchange buffer (the epilogue stores to each rank), or -1
    PSeg seg[3];
};
static_assert(sizeof(FPhase) % 16 == 0 && sizeof(FPhase) / 16 <= 32, "phase descriptors are copied in 16-byte chunks");

struct FParams {
    // K and V pools as 2D tensors [rows = page * layer * kv_head * 64 positions][head_dim] fp16,
    // box 64 x 64 with 128-byte swizzle (attention pages)
    alignas(64) CUtensorMap kmap;
    alignas(64) CUtensorMap vmap;
    const FPhase *phases;  // device array
    int n_phases;
    const uint8_t *embd;
    int embd_type;
    int dim, vocab;
    // attention
    const float2 *rope;          // [max_seq][hd/2] (cos, sin)
    uint16_t *k_pool, *v_pool;   // fp16 bits, [page][layer][kv_head][P][hd]
    const int32_t *page_table;
    int n_layers, n_kv, n_heads, max_seq;
    float att_scale;
    int att_max_split;           // page splits per KV head at most
    uint64_t *att_words;         // tagged split states [n_layers][n_kv][att_max_split][G][hd + 2]
    int hd, G;                   // head_dim, query heads per KV head (the q|k|v word layout)
    // greedy argmax and step state
    unsigned long long *am_key;  // [gridDim.x] per-CTA best (value, index) keys
    unsigned int *am_count;      // ticket, zero between launches
    int32_t *io_token, *io_pos, *io_argmax, *io_err, *io_step;
    int32_t *rec_tokens;
    int loop;                    // 1: feed the argmax back as the next token, advance pos, record it
    unsigned int *epoch;         // tag of the current launch (advanced by the last CTA to exit)
    unsigned int *exit_count;
    int ring_bytes, frag_bytes, xres_floats, xin_floats, nw_floats;
    unsigned long long *trace;   // [n_phases][gridDim.x][FL_TRACE_FIELDS] or null
    // tensor parallelism (tp_world > 1): each rank's exchange buffer, mapped into this
    // rank (peer memory over NVLink; this rank's own is local)
    int tp_world, tp_rank;
    uint64_t *tp_bufs[FL_MAX_TP];
    int lm_shard;                // tensor parallel, no logits wanted: each rank runs its share of the
                                 // lm_head tiles and the ranks exchange their best keys
    long long tp_key_off;        // word offset of the [world][2] key area in the exchange buffers
};

// ---- per-CTA state ----------------------------------------------------------------------
// dynamic: [pad to 1024][ring][fragments frag_bytes][xres xres_floats][xin xin_floats][norm weights nw_floats]
extern __shared__ __align__(128) uint8_t fl_dyn[];
__shared__ __align__(8) uint64_t fl_full[FL_NDESC];
__shared__ __align__(8) uint64_t fl_empty[FL_NDESC];
__shared__ __align__(16) FPhase fl_F[2];
__shared__ __align__(16) FPhase fl_E[2];  // the epilogue warp's own copies (it runs behind the consumers)
__shared__ __align__(16) float fl_red[FL_NDESC][FL_WARPS][TC_M];  // per ring slot: warp partial sums
__shared__ __align__(8) uint64_t fl_done[FL_NDESC];  // per ring slot: the eight warps' partial sums written
__shared__ float fl_stat[2 * FL_WARPS];
__shared__ unsigned long long fl_best;   // this CTA's best logit key
__shared__ int fl_tile_off[FL_NDESC];
__shared__ volatile int fl_abort;
constexpr int FL_MAX_CHUNKS = 64;        // input length / 256 at most (16384 elements)
__shared__ float fl_cinv[FL_MAX_CHUNKS]; // staged input: per-chunk inverse fragment scale
__shared__ float fl_wss[4][FL_WARPS];    // staged input of phase ph: per-warp sums of x^2 (RMSNorm),
                                         // at ph % 4 (the epilogue warp may run a phase or two behind)
__shared__ unsigned long long fl_tmark[1];  // trace: globaltimer when the inputs were staged
__shared__ float2 fl_rope[64];           // RoPE (cos, sin) row of this launch's position

FDEV uint8_t *fl_ring() { return fl_dyn + ((FL_RING_PAD - (smem_u32(fl_dyn) & (FL_RING_PAD - 1))) & (FL_RING_PAD - 1)); }
FDEV uint2 *fl_frag(const FParams &P) { return reinterpret_cast<uint2 *>(fl_dyn + FL_RING_PAD + P.ring_bytes); }
FDEV float *fl_xres(const FParams &P) {
    return reinterpret_cast<float *>(fl_dyn + FL_RING_PAD + P.ring_bytes + P.frag_bytes);
}
FDEV float *fl_xin(const FParams &P) { return fl_xres(P) + P.xres_floats; }
FDEV float *fl_nw(const FParams &P) { return fl_xin(P) + P.xin_floats; }

// ---- tagged words ----------------------------------------------------------------------

FDEV uint64_t ll_word(float v, uint32_t tag) { return ((uint64_t)tag << 32) | __float_as_uint(v); }
FDEV void ll_store(uint64_t *p, float v, uint32_t tag) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(ll_word(v, tag)) : "memory");
}
FDEV ulonglong2 ll_load2(const uint64_t *p) {
    ulonglong2 r;
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(r.x), "=l"(r.y) : "l"(p) : "memory");
    return r;
}

// Tagged words exchanged between GPUs: system-scope stores into a peer's buffer and
// system-scope loads of this GPU's buffer (no multicast, no bulk copies on peer memory).
FDEV void ll_store_sys(uint64_t *p, float v, uint32_t tag) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(ll_word(v, tag)) : "memory");
}
FDEV void ll_store_bits_sys(uint64_t *p, uint32_t bits, uint32_t tag) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(((uint64_t)tag << 32) | bits) : "memory");
}
FDEV ulonglong2 ll_load2_sys(const uint64_t *p) {
    ulonglong2 r;
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(r.x), "=l"(r.y) : "l"(p) : "memory");
    return r;
}

// Tensor parallel: one partial sum to word `off` of every rank's exchange buffer (out of
// line: the single-GPU epilogue carries only the call).
__device__ __noinline__ void fl_tp_store_partial(const FParams &P, long long off, float v, uint32_t tag) {
    for (int q = 0; q < P.tp_world; q++) ll_store_sys(P.tp_bufs[q] + off, v, tag);
}

FDEV void fl_fail(const FParams &P) {
    fl_abort = 1;
    *P.io_err = 4;
}

// Consumer barrier that also returns the OR of v over the 256 consumer threads, so
// every thread takes the same branch after it (a stop decision never splits them).
FDEV bool cbar_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(FL_CONSUMERS)
        : "memory");
    return r != 0;
}

// Copy phase descriptor src into shared memory with 16-byte async copies (lanes of
// one warp); complete after cp_async_wait_all + a barrier.
FDEV void fl_fetch_phase(FPhase *dst, const FPhase *src, int lane) {
    constexpr int CH = (int)(sizeof(FPhase) / 16);
    if (lane < CH) cp_async16(reinterpret_cast<uint4 *>(dst) + lane, reinterpret_cast<const uint4 *>(src) + lane);
}

FDEV void fl_locate(const FPhase &F, int tile, int &s, int &lt) {
    s = 0;
    lt = tile;
    while (s + 1 < F.nseg && lt >= F.seg[s].tiles) lt -= F.seg[s++].tiles;
}

// Poll n tagged words (n even, src 16-byte aligned) into dst[0..n) (shared memory).
// All consumer threads; each issues up to eight 16-byte loads before it waits, then
// reloads only the words without this launch's tag. Returns false on timeout.
FDEV bool fl_poll(const FParams &P, const uint64_t *src, float *dst, int n, uint32_t tag) {
    const int nch = n >> 1;
    for (int base = threadIdx.x; base < nch; base += 8 * FL_CONSUMERS) {
        ulonglong2 w[8];
        uint32_t pend = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int c = base + i * FL_CONSUMERS;
            if (c < nch) {
                w[i] = ll_load2(src + 2 * c);
                pend |= 1u << i;
            }
        }
        unsigned long long t0 = 0;
        for (long long it = 0;; it++) {
#pragma unroll
            for (int i = 0; i < 8; i++) {
                if ((pend >> i) & 1u) {
                    if ((uint32_t)(w[i].x >> 32) == tag && (uint32_t)(w[i].y >> 32) == tag) {
                        const int c = base + i * FL_CONSUMERS;
                        dst[2 * c] = __uint_as_float((uint32_t)w[i].x);
                        dst[2 * c + 1] = __uint_as_float((uint32_t)w[i].y);
                        pend &= ~(1u << i);
                    }
                }
            }
            if (!pend) break;
            if (it == 0) {
                t0 = gtimer();
            } else if ((it & 15) == 0 && (fl_abort || gtimer() - t0 > FL_WAIT_NS)) {
                fl_fail(P);
                return false;
            }
#pragma unroll
            for (int i = 0; i < 8; i++)
                if ((pend >> i) & 1u) w[i] = ll_load2(src + 2 * (base + i * FL_CONSUMERS));
        }
    }
    return true;
}

// Bounded wait on a ring slot by one lane.
FDEV bool fl_mbar_wait(uint64_t *bar, uint32_t parity) {
    if (pk_mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = gtimer();
    for (;;) {
        if (pk_mbar_try_wait(bar, parity)) return true;
        if (fl_abort || gtimer() - t0 > FL_WAIT_NS) return false;
    }
}

// Bounded wait for a warp that has nothing else to do (the producer on ring space, the
// epilogue warp on partial sums): each try suspends the thread until the phase completes
// or the hint (ns) runs out, so the wait takes no issue slots from the compute warps
// that share its SM sub-partition.
FDEV bool fl_mbar_wait_idle(uint64_t *bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    const unsigned long long t0 = gtimer();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(a), "r"(parity), "r"(20000u)
            : "memory");
        if (ok) return true;
        if (fl_abort || gtimer() - t0 > FL_WAIT_NS) return false;
    }
}

// Warp-level acquire of ring item `seq`: lane 0 waits, the warp agrees.
FDEV const uint8_t *fl_acquire(const FParams &P, long long seq, long long &wcycles) {
    const int d = (int)(seq % FL_NDESC);
    int ok = 1;
    if ((threadIdx.x & 31) == 0) {
        const long long c0 = clock64();
        ok = fl_mbar_wait(&fl_full[d], (uint32_t)((seq / FL_NDESC) & 1));
        if (!ok) fl_fail(P);
        wcycles += clock64() - c0;
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    return ok ? fl_ring() + fl_tile_off[d] : nullptr;
}

// Block-wide reduction over the consumer threads of two values (sum, max), fixed order.
FDEV void fl_reduce2(float &sum, float &mx) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (lane == 0) {
        fl_stat[warp] = sum;
        fl_stat[FL_WARPS + warp] = mx;
    }
    cbar();
    sum = 0.f;
    mx = 0.f;
#pragma unroll
    for (int w = 0; w < FL_WARPS; w++) {
        sum += fl_stat[w];
        mx = fmaxf(mx, fl_stat[FL_WARPS + w]);
    }
    cbar();  // fl_stat reused
}

// Power-of-two scale that puts the largest staged magnitude m in [2^13, 2^14):
// the fp16 hi part stays far below 65504 and the lo part stays normal.
FDEV void fl_set_scale(float m, float &scale, float &inv) {
    int eb = (int)((__float_as_uint(m) >> 23) & 0xFF);
    eb = max(14, min(eb, 254));
    scale = __uint_as_float((uint32_t)(267 - eb) << 23);
    inv = __uint_as_float((uint32_t)(eb - 13) << 23);
}

template <int HD, int G>
struct FlowAttn;

// v - (fp16 value in the low half of h), exact in fp32 (v's fp16 rounding error)
FDEV float fl_rem(uint32_t h, float v) {
    float r;
    asm("{\n .reg .f16 l, u, m;\n mov.b32 {l, u}, %1;\n mov.b16 m, 0xBC00;\n fma.rn.f32.f16 %0, l, m, %2;\n}\n"
        : "=f"(r)
        : "r"(h), "f"(v));
    return r;
}

// Fragments of chunk b (elements 256b .. 256b+255) of the staged input for weight
// type T (the k-slot order TcDot<T> reads, TcType<T>::elem): per group f the fp16 hi
// parts of its four elements, then the lo parts (hi + lo carries ~22 bits), v = x * w *
// scale where the phase has an RMSNorm (w its weights; rrms is applied to the dot
// products), else x * scale. Lanes of one warp, two groups each.
template <int T>
FDEV void fl_frags_chunk(int b, const float *xs, const float *nw, float scale, uint2 *xf) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const int f = b * 64 + lane + 32 * j, s = (f >> 2) & 15, t = f & 3;
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int k = b * 256 + TcType<T>::elem(t, s, i);
            float x = xs[k];
            if (nw) x = __fmul_rn(x, nw[k]);
            v[i] = x * scale;
        }
        const uint32_t h01 = pack_f16x2(v[0], v[1]), h23 = pack_f16x2(v[2], v[3]);
        const uint32_t l01 = pack_f16x2(fl_rem(h01, v[0]), fl_rem(h01 >> 16, v[1]));
        const uint32_t l23 = pack_f16x2(fl_rem(h23, v[2]), fl_rem(h23 >> 16, v[3]));
        xf[2 * f + 0] = make_uint2(h01, h23);
        xf[2 * f + 1] = make_uint2(l01, l23);
    }
}

// ---- GEMV phase -----------------------------------------------------------------------

// Chunk b of the embedding row of token tok, rounded to fp16 as the reference's
// gpu_embed writes it, into xs (lanes of one warp). Only the first layer runs it, so
// it is kept out of line (instruction-cache footprint of the per-layer path).
__device__ __noinline__ void fl_embed_chunk(const FParams &P, int tok, int b, float *xs) {
    const int lane = threadIdx.x & 31, n = P.dim, nb = n >> 8;
    for (int e = lane; e < 256; e += 32) {
        const int i = b * 256 + e;
        float v;
        switch (P.embd_type) {
        case T_F16: v = h2f(reinterpret_cast<const uint16_t *>(P.embd)[(size_t)tok * n + i]); break;
        case T_F32: v = round_f16(reinterpret_cast<const float *>(P.embd)[(size_t)tok * n + i]); break;
        case T_Q4_K: v = round_f16(decode_elem<T_Q4_K>(P.embd + ((size_t)tok * nb + b) * 144, e)); break;
        case T_Q5_K: v = round_f16(decode_elem<T_Q5_K>(P.embd + ((size_t)tok * nb + b) * 176, e)); break;
        default: v = round_f16(decode_elem<T_Q6_K>(P.embd + ((size_t)tok * nb + b) * 210, e)); break;
        }
        xs[i] = v;
    }
}

// Tensor parallel: chunk b of x = (residual kept in xs) + the ranks' partial sums, added
// in rank order, so every rank computes the same x bit for bit. `in` holds [world][cols]
// tagged words, polled one rank at a time (four 16-byte loads per lane: polling two ranks
// at once held enough registers to make ptxas spill in the tile loops and the attention unit).
// Lanes of one warp; returns false (warp-uniform) when stopped.
FDEV bool fl_stage_tp_chunk(const FParams &P, const FPhase &F, int b, uint32_t tag, float *xs) {
    const int lane = threadIdx.x & 31, n = F.cols;
    float x[8];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float2 v = *reinterpret_cast<const float2 *>(xs + b * 256 + 2 * (lane + 32 * k));
        x[2 * k] = v.x;
        x[2 * k + 1] = v.y;
    }
    for (int r = 0; r < P.tp_world; r++) {
        const uint64_t *src = F.in + (size_t)r * n + b * 256;
        ulonglong2 w[4];
        uint32_t pend = 15u;
#pragma unroll
        for (int k = 0; k < 4; k++) w[k] = ll_load2_sys(src + 2 * (lane + 32 * k));
        unsigned long long t0 = 0;
        for (long long it = 0;; it++) {
#pragma unroll
            for (int k = 0; k < 4; k++)
                if (((pend >> k) & 1u) && (uint32_t)(w[k].x >> 32) == tag && (uint32_t)(w[k].y >> 32) == tag)
                    pend &= ~(1u << k);
            if (__all_sync(0xffffffffu, pend == 0)) break;
            if (it == 0) {
                t0 = gtimer();
            } else if ((it & 15) == 0) {
                int stop = fl_abort || gtimer() - t0 > FL_WAIT_NS;
                if (__any_sync(0xffffffffu, stop)) {
                    if (lane == 0) fl_fail(P);
                    return false;
                }
            }
#pragma unroll
            for (int k = 0; k < 4; k++)
                if ((pend >> k) & 1u) w[k] = ll_load2_sys(src + 2 * (lane + 32 * k));
        }
#pragma unroll
        for (int k = 0; k < 4; k++) {
            x[2 * k] = __fadd_rn(x[2 * k], __uint_as_float((uint32_t)w[k].x));
            x[2 * k + 1] = __fadd_rn(x[2 * k + 1], __uint_as_float((uint32_t)w[k].y));
        }
    }
#pragma unroll
    for (int k = 0; k < 4; k++)
        *reinterpret_cast<float2 *>(xs + b * 256 + 2 * (lane + 32 * k)) = make_float2(x[2 * k], x[2 * k + 1]);
    return true;
}

// Stage this warp's chunks of the phase input: chunk b (256 elements) is staged by warp
// b % 8, the warp that multiplies super-block column b of every tile, so no other warp
// waits for it. Per chunk: poll its tagged words (or decode the embedding row), keep
// the fp32 values (the residual of the next residual phase), add x^2 in a fixed order
// to this warp's RMSNorm sum (fl_wss[warp], read by the epilogues), choose the power of
// two s_b that puts the chunk's largest |x * w| into [2^13, 2^14) (fl_cinv[b] = 1 / s_b, applied to
// the chunk's dot products) and write its fragments for each weight type of the phase.
// Two chunks at a time (eight 16-byte loads in flight per lane). Warp-level; returns
// false (warp-uniform) when stopped.
// TP: the tensor-parallel instance (norm phases add the ranks' partial sums).
template <bool TP>
__device__ __noinline__ bool fl_stage_warp(const FParams &P, const FPhase &F, int ph, uint32_t tag, int token,
                                           unsigned long long *tr) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = F.cols, nb = n >> 8;
    const bool norm = F.norm_w != nullptr;
    float *xs = norm ? fl_xres(P) : fl_xin(P);
    float *nw = fl_nw(P);
    int type_b = -1;
    for (int k = 1; k < F.nseg; k++)
        if (F.seg[k].type != F.seg[0].type && type_b < 0) type_b = F.seg[k].type;
    uint2 *xf0 = fl_frag(P), *xf1 = xf0 + (size_t)nb * 128;
    int tok = token;
    if (F.embed_in && (tok < 0 || tok >= P.vocab)) {
        if (threadIdx.x == 0 && blockIdx.x == 0) *P.io_err = 2;
        tok = 0;
    }
    float ss = 0.f;
    long long cpoll = 0, cstage = 0;
    for (int b0 = warp; b0 < nb; b0 += 2 * FL_WARPS) {
        const int nc = b0 + FL_WARPS < nb ? 2 : 1;  // chunks b0 and b0 + 8
        long long c0 = clock64();
        if (norm)
            for (int c = 0; c < nc; c++) {
                const int b = b0 + c * FL_WARPS;
                cp_async16(nw + b * 256 + 4 * lane, F.norm_w + b * 256 + 4 * lane);
                cp_async16(nw + b * 256 + 128 + 4 * lane, F.norm_w + b * 256 + 128 + 4 * lane);
            }
        if (F.embed_in) {  // every CTA decodes the embedding row itself (src/gpu_ffn.m:466-482)
            for (int c = 0; c < nc; c++) fl_embed_chunk(P, tok, b0 + c * FL_WARPS, xs);
        } else if (TP && F.tp_sum) {
            for (int c = 0; c < nc; c++)
                if (!fl_stage_tp_chunk(P, F, b0 + c * FL_WARPS, tag, xs)) {
                    cp_async_wait_all();
                    return false;
                }
        } else {
            // pair k of the group: chunk b0 + 8 (k / 4), words 2 (lane + 32 (k % 4)) + {0, 1}
            ulonglong2 w[8];
            uint32_t pend = 0;
#pragma unroll
            for (int k = 0; k < 8; k++) {
                if (k < 4 * nc) {
                    const int b = b0 + (k >> 2) * FL_WARPS;
                    w[k] = ll_load2(F.in + b * 256 + 2 * (lane + 32 * (k & 3)));
                    pend |= 1u << k;
                }
            }
            unsigned long long t0 = 0;
            for (long long it = 0;; it++) {
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    if ((pend >> k) & 1u) {
                        if ((uint32_t)(w[k].x >> 32) == tag && (uint32_t)(w[k].y >> 32) == tag) {
                            const int b = b0 + (k >> 2) * FL_WARPS;
                            const float v0 = __uint_as_float((uint32_t)w[k].x), v1 = __uint_as_float((uint32_t)w[k].y);
                            *reinterpret_cast<float2 *>(xs + b * 256 + 2 * (lane + 32 * (k & 3))) = make_float2(v0, v1);
                            pend &= ~(1u << k);
                        }
                    }
                }
                if (__all_sync(0xffffffffu, pend == 0)) break;
                if (it == 0) {
                    t0 = gtimer();
                } else if ((it & 15) == 0) {
                    int stop = fl_abort || gtimer() - t0 > FL_WAIT_NS;
                    stop = __any_sync(0xffffffffu, stop);
                    if (stop) {
                        if (lane == 0) fl_fail(P);
                        cp_async_wait_all();
                        return false;
                    }
                }
#pragma unroll
                for (int k = 0; k < 8; k++)
                    if ((pend >> k) & 1u) {
                        const int b = b0 + (k >> 2) * FL_WARPS;
                        w[k] = ll_load2(F.in + b * 256 + 2 * (lane + 32 * (k & 3)));
                    }
            }
        }
        cp_async_wait_all();
        __syncwarp();
        const long long c1 = clock64();
        cpoll += c1 - c0;
        for (int c = 0; c < nc; c++) {
            const int b = b0 + c * FL_WARPS;
            float mx = 0.f;
#pragma unroll
            for (int e = 0; e < 8; e++) {  // fixed order: the sums do not depend on arrival order
                const int i = b * 256 + lane + 32 * e;
                const float x = xs[i];
                ss = fmaf(x, x, ss);
                mx = fmaxf(mx, fabsf(norm ? x * nw[i] : x));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (!(mx < 3.0e38f)) {  // non-finite activations
                if (lane == 0) *P.io_err = 5;
                mx = 1.0f;
            }
            float scale, inv;
            fl_set_scale(mx, scale, inv);
            if (lane == 0) fl_cinv[b] = inv;
            for (int pass = 0; pass < (type_b >= 0 ? 2 : 1); pass++) {
                uint2 *dst = pass ? xf1 : xf0;
                switch (pass ? type_b : F.seg[0].type) {
                case T_Q4_K: fl_frags_chunk<T_Q4_K>(b, xs, norm ? nw : nullptr, scale, dst); break;
                case T_Q6_K: fl_frags_chunk<T_Q6_K>(b, xs, norm ? nw : nullptr, scale, dst); break;
                case T_Q5_K: fl_frags_chunk<T_Q5_K>(b, xs, norm ? nw : nullptr, scale, dst); break;
                default: fl_frags_chunk<T_F16>(b, xs, norm ? nw : nullptr, scale, dst); break;
                }
            }
        }
        __syncwarp();
        cstage += clock64() - c1;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) {
        fl_wss[ph & 3][warp] = ss;
        if (P.trace) atomicMax(&fl_tmark[0], gtimer());
    }
    __syncwarp();
    if (tr) {
        tr[1] = (unsigned long long)cpoll;
        tr[2] = (unsigned long long)cstage;
    }
    return true;
}

// RMSNorm factor of phase ph's staged input from the eight warps' sums (fixed order).
FDEV float fl_rrms(const FPhase &F, int ph) {
    float ss = 0.f;
#pragma unroll
    for (int w = 0; w < FL_WARPS; w++) ss += fl_wss[ph & 3][w];
    return 1.0f / sqrtf(ss / (float)F.cols + F.eps);
}

// Order-preserving key of a logit: larger value first, then lower index; NaN below
// everything (the reference's strict '>' never picks it), -0 as +0.
FDEV unsigned long long fl_key(float v, int idx) {
    uint32_t b = __float_as_uint(v + 0.0f);
    b = (v != v) ? 0u : ((b & 0x80000000u) ? ~b : (b | 0x80000000u));
    return ((unsigned long long)b << 32) | (0xFFFFFFFFu - (uint32_t)idx);
}

// Epilogue of one tile (the last warp to finish it): lanes 0..15 own its rows; in a
// SwiGLU tile lane j < 8 owns output row 8 lt + j (gate in MMA row j, up in row j + 8).
template <bool TP>
FDEV void fl_epilogue(const FParams &P, const FPhase &F, const PSeg &S, int lt, int d, uint32_t tag, float rrms) {
    const int lane = threadIdx.x & 31;
    const bool pair = F.kind == FL_SWIGLU;
    if (lane < (pair ? TC_M / 2 : TC_M)) {
        const int r = lt * (pair ? TC_M / 2 : TC_M) + lane;
        float v0 = 0.f, v1 = 0.f;
#pragma unroll
        for (int w = 0; w < FL_WARPS; w++) v0 += fl_red[d][w][lane];
        if (pair) {
#pragma unroll
            for (int w = 0; w < FL_WARPS; w++) v1 += fl_red[d][w][lane + TC_M / 2];
        }
        if (F.norm_w) {  // y = rrms * W (x * w)
            v0 *= rrms;
            v1 *= rrms;
        }
        if (r < S.rows) {
            switch (F.kind) {
            case FL_QKV: {  // q|k|v grouped by KV head: [g][G query heads | k | v] x hd
                const int o = S.out_off + r;
                const int qd = P.n_heads * P.hd, kd = P.n_kv * P.hd;
                int gi, slot;
                if (o < qd) {
                    gi = o / (P.G * P.hd);
                    slot = o % (P.G * P.hd);
                } else if (o < qd + kd) {
                    gi = (o - qd) / P.hd;
                    slot = P.G * P.hd + (o - qd) % P.hd;
                } else {
                    gi = (o - qd - kd) / P.hd;
                    slot = (P.G + 1) * P.hd + (o - qd - kd) % P.hd;
                }
                ll_store(F.out + (size_t)gi * (P.G + 2) * P.hd + slot, v0, tag);
                break;
            }
            case FL_RESID:
                if (TP && F.tp_off >= 0) {  // this rank's partial sum, to every rank (the next phase adds them)
                    fl_tp_store_partial(P, F.tp_off + (long long)P.tp_rank * S.rows + r, v0, tag);
                } else {
                    ll_store(F.out + r, __fadd_rn(fl_xres(P)[r], v0), tag);
                }
                break;
            case FL_SWIGLU: {
                const float h = __fmul_rn(__fdiv_rn(v0, __fadd_rn(1.0f, expf(-v0))), v1);
                ll_store(F.out + r, h, tag);
                break;
            }
            default:  // FL_LM
                F.logits[r] = v0;
                atomicMax(&fl_best, fl_key(v0, r));
                break;
            }
        }
    }
}

// Release of a ring slot by one warp: a relaxed arrival (the warp's reads of the slot have
// all returned, their values are consumed, so no release ordering is needed; a release
// would also wait for the epilogue's global stores).
FDEV void fl_release_slot(uint64_t *bar) {
    asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One tile of the phase, warp-level: decode + multiply this warp's super-blocks and
// publish the partial sums (fl_done[d]); the epilogue warp sums the eight and runs the
// epilogue, then frees the slot with the last of its nine arrivals (the partial sums
// live with the slot until it is refilled).
template <int T>
FDEV void fl_tile(const FParams &P, const FPhase &F, const PSeg &S, int lt, const uint8_t *buf, const uint2 *xf,
                  int d, uint32_t tag, unsigned long long *tr, long long (&tacc)[4]) {
    const long long c0 = tr ? clock64() : 0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int nb = F.cols >> 8;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int b = warp; b < nb; b += FL_WARPS) {
        const float inv = fl_cinv[b];  // the chunk's fragment scale, undone per chunk
        const uint8_t *mb = buf + (size_t)b * TcType<T>::BB;
        float part[4] = {0.f, 0.f, 0.f, 0.f};
        TcDot<T>::run(mb + (size_t)g * S.stride, mb + (size_t)(g + 8) * S.stride, xf + (size_t)b * 128, g, t, part);
#pragma unroll
        for (int i = 0; i < 4; i++) acc[i] = fmaf(part[i], inv, acc[i]);
    }
    const long long c1 = tr ? clock64() : 0;
    if (t == 0) {
        fl_red[d][warp][g] = acc[0] + acc[1];
        fl_red[d][warp][g + 8] = acc[2] + acc[3];
    }
    __syncwarp();  // the warp's partial sums are written before lane 0 releases them
    if (lane == 0) {
        mbar_arrive(&fl_done[d]);        // release: the epilogue warp reads the sums
        fl_release_slot(&fl_empty[d]);  // this warp's reads of the slot are done
    }
    if (tr) {  // registers here; the trace is written once per phase
        tacc[0] += c1 - c0;
        tacc[1] += clock64() - c1;
        tacc[3] += 1;
    }
}

// Tiles [t0, t1) of phase F on this GPU: all of them, except the lm_head of a sharded
// greedy step, where each rank takes an equal share (the ranks exchange their best keys).
template <bool TP>
FDEV void fl_tile_range(const FParams &P, const FPhase &F, int &t0, int &t1) {
    t0 = 0;
    t1 = F.n_tiles;
    if (TP && F.kind == FL_LM && P.lm_shard) {
        const int per = (F.n_tiles + P.tp_world - 1) / P.tp_world;
        t0 = min(F.n_tiles, P.tp_rank * per);
        t1 = min(F.n_tiles, t0 + per);
    }
}

// The CTA's tiles of one GEMV phase (tile = blockIdx.x + k * gridDim.x), warp-level.
template <bool TP>
FDEV bool fl_tiles(const FParams &P, const FPhase &F, long long &seq, uint32_t tag, long long &wcycles,
                   unsigned long long *tr) {
    const int nb = F.cols >> 8;
    const uint2 *xf0 = fl_frag(P), *xf1 = xf0 + (size_t)nb * 128;
    long long tacc[4] = {0, 0, 0, 0};
    int t0, t1;
    fl_tile_range<TP>(P, F, t0, t1);
    for (int tile = t0 + blockIdx.x; tile < t1; tile += gridDim.x) {
        int sidx, lt;
        fl_locate(F, tile, sidx, lt);
        const PSeg &S = F.seg[sidx];
        const uint8_t *buf = fl_acquire(P, seq, wcycles);
        if (!buf) return false;
        const int d = (int)(seq % FL_NDESC);
        const uint2 *xf = (S.type == F.seg[0].type) ? xf0 : xf1;
        switch (S.type) {
        case T_Q4_K: fl_tile<T_Q4_K>(P, F, S, lt, buf, xf, d, tag, tr, tacc); break;
        case T_Q6_K: fl_tile<T_Q6_K>(P, F, S, lt, buf, xf, d, tag, tr, tacc); break;
        case T_Q5_K: fl_tile<T_Q5_K>(P, F, S, lt, buf, xf, d, tag, tr, tacc); break;
        default: fl_tile<T_F16>(P, F, S, lt, buf, xf, d, tag, tr, tacc); break;
        }
        seq++;
    }
    if (tr)
        for (int i = 0; i < 4; i++) tr[12 + i] = (unsigned long long)tacc[i];
    return true;
}

// ---- attention ------------------------------------------------------------------------

// Units of the attention phase at position pos: n_kv * S, S page splits per KV head
// (about eight pages per unit, one per warp, so a unit's pages arrive while the QKV
// phase runs and are processed in parallel; at most att_max_split); unit u = g * S + j runs on CTA gridDim.x - 1 - u,
// pages [j * nch / S, (j + 1) * nch / S).
constexpr int FL_PAGES_PER_UNIT = 8;  // one page per consumer warp
FDEV int fl_att_splits(const FParams &P, int nch) {
    return max(1, min((nch + FL_PAGES_PER_UNIT - 1) / FL_PAGES_PER_UNIT, P.att_max_split));
}

// fragments / copies for the attention unit
FDEV void mma16808(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(b0));
}
FDEV void ldsm_x4_trans(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
FDEV uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
// 2D tensor copy (no multicast) of one box into shared memory, completion on bar
FDEV void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
FDEV uint32_t pack_hi_lo(float a, float b, uint32_t &lo) {  // fp16 hi parts of (a, b); lo parts returned in lo
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(a - hf.x, b - hf.y);
    lo = *reinterpret_cast<const uint32_t *>(&l);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Attention unit on the tensor cores. K/V pages arrive by tensor copies in the
// 128-byte swizzled layout: a page of K (or V) is HD/64 column halves of
// [64 rows][128 bytes], 16-byte chunk c of row r stored at chunk c ^ (r & 7), so
// the fragment loads below hit 32 distinct banks.
template <int HD, int G>
struct FlowAttn {
    static constexpr int PG = ATTN_P;
    static constexpr int KS = HD / 16;   // k-steps of q.k
    static constexpr int NT = HD / 8;    // 8-dim tiles of P.V
    static constexpr int HALF = 64 * 128;  // bytes of one 64-dim column half of a page
    static constexpr int PAGE = PG * HD * 2;
    static_assert(G == 1 || G == 2 || G == 4 || G == 8, "query heads per KV head");
    static_assert(HD == 64 || HD == 128, "head_dim 64 or 128");
    static_assert(PG == 64 && FL_WARPS == 8, "eight warps x eight positions per page");

    // shared scratch (in the xin region): q [G][HD] fp32, nk/nv [HD] fp16 each,
    // warp states [8][G][HD + 2], the polled q | k | v [(G + 2) * HD]; then the other
    // splits' states [att_max_split - 1][G][HD + 2] (sized by the host)
    static constexpr int SCRATCH_FLOATS = G * HD + HD + FL_WARPS * G * (HD + 2) + (G + 2) * HD;

    // byte offset of (row r, dims 8c .. 8c+7) in a swizzled page
    static FDEV uint32_t swz(int r, int c) { return (uint32_t)((c >> 3) * HALF + r * 128 + (((c & 7) ^ (r & 7)) << 4)); }

    static __device__ __noinline__ bool unit(const FParams &P, const FPhase &F, int g, int j, int S, int pos, int nch,
                                             long long &seq, uint32_t tag, long long &wcycles, unsigned long long *tr) {
        const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gl = lane >> 2, t = lane & 3;
        long long ck = clock64();
        auto mark = [&](int field) {
            if (tr) {
                const long long n = clock64();
                tr[field] = (unsigned long long)(n - ck);
                ck = n;
            }
        };
        float *sm = fl_xin(P);
        float *qs = sm;                                             // [G][HD]
        uint16_t *nk = reinterpret_cast<uint16_t *>(sm + G * HD);   // [HD]
        uint16_t *nv = nk + HD;                                     // [HD]
        float *wm = sm + G * HD + HD;                               // [FL_WARPS][G][HD + 2]
        float *raw = wm + FL_WARPS * G * (HD + 2);                  // [(G + 2) * HD] q | k | v as polled
        float *others = raw + (G + 2) * HD;                         // [S - 1][G][HD + 2] other splits' states
        const bool got = fl_poll(P, F.in + (size_t)g * (G + 2) * HD, raw, (G + 2) * HD, tag);
        if (cbar_any(!got || fl_abort)) return false;
        mark(1);
        const int tn = pos - (nch - 1) * PG;  // row of the new position in the last page
        const bool writer = j == S - 1;       // the unit holding the last page appends the new K/V row
        const size_t base = (((size_t)P.page_table[nch - 1] * P.n_layers + F.layer) * P.n_kv + g) * (size_t)PG * HD;
        const float2 *rp = fl_rope;
        float qmax = 0.f;
        for (int i = tid; i < (G + 1) * (HD / 2); i += FL_CONSUMERS) {  // RoPE (src/fiber_proof.m:30-51)
            const int h = i / (HD / 2), jj = i % (HD / 2);
            const float2 cs = rp[jj];
            const float x1 = raw[h * HD + jj], x2 = raw[h * HD + jj + HD / 2];
            const float y1 = __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y));
            const float y2 = __fadd_rn(__fmul_rn(x1, cs.y), __fmul_rn(x2, cs.x));
            if (h < G) {
                qs[h * HD + jj] = y1;
                qs[h * HD + jj + HD / 2] = y2;
                qmax = fmaxf(qmax, fmaxf(fabsf(y1), fabsf(y2)));
            } else {
                const uint16_t b1 = __half_as_ushort(__float2half_rn(y1)), b2 = __half_as_ushort(__float2half_rn(y2));
                nk[jj] = b1;
                nk[jj + HD / 2] = b2;
                if (writer) {
                    P.k_pool[base + (size_t)tn * HD + jj] = b1;
                    P.k_pool[base + (size_t)tn * HD + jj + HD / 2] = b2;
                }
            }
        }
        for (int i = tid; i < HD; i += FL_CONSUMERS) {
            const uint16_t b = __half_as_ushort(__float2half_rn(raw[G * HD + HD + i]));
            nv[i] = b;
            if (writer) P.v_pool[base + (size_t)tn * HD + i] = b;
        }
        float dummy = 0.f;
        fl_reduce2(dummy, qmax);  // barriers: qs, nk, nv complete
        if (!(qmax < 3.0e38f)) {
            if (tid == 0) *P.io_err = 5;
            qmax = 1.0f;
        }
        float qscale, qinv;
        fl_set_scale(qmax, qscale, qinv);
        const float sscale = __fmul_rn(qinv, P.att_scale);  // exact power of two times 1/sqrt(hd)

        // q as the A operand: row gl = head gl (hi part), row gl + 8 = its lo part; rows of
        // missing heads are zero
        uint32_t qa[KS][4];
#pragma unroll
        for (int ks = 0; ks < KS; ks++) {
            if (gl < G) {
                const float *qr = qs + gl * HD + 16 * ks + 2 * t;
                uint32_t lo0, lo1;
                qa[ks][0] = pack_hi_lo(qr[0] * qscale, qr[1] * qscale, lo0);
                qa[ks][2] = pack_hi_lo(qr[8] * qscale, qr[9] * qscale, lo1);
                qa[ks][1] = lo0;
                qa[ks][3] = lo1;
            } else {
                qa[ks][0] = qa[ks][1] = qa[ks][2] = qa[ks][3] = 0u;
            }
        }
        mark(2);
        // this warp: whole pages p0 + warp, p0 + warp + 8, ... (all G heads; lane: head gl);
        // every warp steps through every item of the ring, the owner frees it
        float m_run = -INFINITY, l_run = 0.f, o[NT][4];
#pragma unroll
        for (int n = 0; n < NT; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
        const uint32_t nk_a = smem_u32(nk), nv_a = smem_u32(nv);
        const int p0 = (int)((long long)j * nch / S), p1 = (int)((long long)(j + 1) * nch / S);
        bool ok = true;
        long long tacc[4] = {0, 0, 0, 0};  // trace: acquire, q.K, softmax, P.V cycles
        for (int pg = p0; pg < p1; pg++) {
            if ((pg - p0) % FL_WARPS != warp) {
                seq++;
                continue;
            }
            long long ct = clock64();
            auto tmark = [&](int field) {
                if (tr) {
                    const long long n2 = clock64();
                    tacc[field - 12] += n2 - ct;
                    ct = n2;
                }
            };
            const uint8_t *tile = fl_acquire(P, seq, wcycles);
            if (!tile) {
                ok = false;
                break;
            }
            tmark(12);
            const int d = (int)(seq % FL_NDESC);
            seq++;
            const bool last = pg == nch - 1;
            const int nvalid = last ? tn + 1 : PG;  // valid positions of the page
            const uint32_t kb = smem_u32(tile), vb = kb + PAGE;
            // scores of the page: n-tile nt = positions 8 nt .. 8 nt + 7; this lane loads K row 8 nt + gl
            float sc[8][4];
#pragma unroll
            for (int nt = 0; nt < 8; nt++) {
                sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
                const int r = 8 * nt + gl;
                const bool fresh = last && r == tn;
#pragma unroll
                for (int ks = 0; ks < KS; ks++) {
                    const uint32_t a0 = fresh ? nk_a + (16 * ks + 2 * t) * 2 : kb + swz(r, 2 * ks) + 4 * t;
                    const uint32_t a1 = fresh ? nk_a + (16 * ks + 8 + 2 * t) * 2 : kb + swz(r, 2 * ks + 1) + 4 * t;
                    mma16816(sc[nt], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], lds32(a0), lds32(a1));
                }
            }
            tmark(13);
            // lane (gl, t): positions 8 nt + 2t, 8 nt + 2t + 1 of head gl
            float mx = -INFINITY;
#pragma unroll
            for (int nt = 0; nt < 8; nt++) {
                const int pa = 8 * nt + 2 * t;
                sc[nt][0] = pa < nvalid ? __fmul_rn(sc[nt][0] + sc[nt][2], sscale) : -INFINITY;
                sc[nt][1] = pa + 1 < nvalid ? __fmul_rn(sc[nt][1] + sc[nt][3], sscale) : -INFINITY;
                mx = fmaxf(mx, fmaxf(sc[nt][0], sc[nt][1]));
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float M = fmaxf(m_run, mx);
            float al = 1.f, psum = 0.f;
            const bool live = M != -INFINITY && gl < G;
            if (live) {
                al = m_run == -INFINITY ? 0.f : expf(m_run - M);
                m_run = M;
            }
#pragma unroll
            for (int nt = 0; nt < 8; nt++) {
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const float v = sc[nt][e];
                    sc[nt][e] = (live && v != -INFINITY) ? expf(v - M) : 0.f;
                    psum += sc[nt][e];
                }
            }
            l_run = fmaf(al, l_run, psum);
#pragma unroll
            for (int n = 0; n < NT; n++) {
                o[n][0] *= al;
                o[n][1] *= al;
                o[n][2] *= al;
                o[n][3] *= al;
            }
            tmark(14);
            // P.V: k-tile kt = positions 8 kt .. 8 kt + 7 (P as the m16n8k8 A operand: row gl hi
            // parts, row gl + 8 lo parts); V by ldmatrix.trans, matrix mi = dims 8 (4 q4 + mi) ..
#pragma unroll
            for (int kt = 0; kt < 8; kt++) {
                uint32_t plo;
                const uint32_t phi = pack_hi_lo(sc[kt][0], sc[kt][1], plo);
                const int vr = 8 * kt + (lane & 7), mi = lane >> 3;
                const bool vfresh = last && vr == tn;
#pragma unroll
                for (int q4 = 0; q4 < NT / 4; q4++) {
                    const int c = 4 * q4 + mi;
                    const uint32_t va = vfresh ? nv_a + c * 16 : vb + swz(vr, c);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_trans(va, b0, b1, b2, b3);
                    mma16808(o[4 * q4 + 0], phi, plo, b0);
                    mma16808(o[4 * q4 + 1], phi, plo, b1);
                    mma16808(o[4 * q4 + 2], phi, plo, b2);
                    mma16808(o[4 * q4 + 3], phi, plo, b3);
                }
            }
            tmark(15);
            __syncwarp();
            if (lane == 0) mbar_arrive_n(&fl_empty[d], FL_WARPS + 1);  // the page's only reader frees it
        }
        if (tr)
            for (int i = 0; i < 4; i++) tr[12 + i] = (unsigned long long)tacc[i];
        // warp state of head gl -> shared memory
        l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
        l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
        if (gl < G) {
            float *wr = wm + (warp * G + gl) * (HD + 2);
#pragma unroll
            for (int n = 0; n < NT; n++) {
                wr[2 + 8 * n + 2 * t] = o[n][0] + o[n][2];
                wr[2 + 8 * n + 2 * t + 1] = o[n][1] + o[n][3];
            }
            if (t == 0) {
                wr[0] = m_run;
                wr[1] = l_run;
            }
        }
        if (cbar_any(!ok || fl_abort)) return false;
        mark(8);
        // merge the eight warps of each head (warp order) into this split's state
        uint64_t *mine = P.att_words + (((size_t)F.layer * P.n_kv + g) * P.att_max_split + j) * G * (HD + 2);
        // per head h: M = the warps' largest running max, f[h][w] = exp(m_w - M) (0 for a
        // warp without valid positions), kept in the q scratch (q is in registers now)
        float *fw = qs, *Mh = qs + G * FL_WARPS;
        if (tid < G * FL_WARPS) {
            const int h = tid / FL_WARPS, w = tid % FL_WARPS;
            float M = -INFINITY;
#pragma unroll
            for (int v = 0; v < FL_WARPS; v++) M = fmaxf(M, wm[(v * G + h) * (HD + 2)]);
            const float m = wm[(w * G + h) * (HD + 2)];
            fw[tid] = m == -INFINITY ? 0.f : expf(m - M);
            if (w == 0) Mh[h] = M;
        }
        cbar();
        for (int i = tid; i < G * (HD + 2); i += FL_CONSUMERS) {
            const int h = i / (HD + 2), e = i % (HD + 2);
            const float M = Mh[h];
            float acc = 0.f, L = 0.f;
#pragma unroll
            for (int w = 0; w < FL_WARPS; w++) {  // warp order
                const float *st = wm + (w * G + h) * (HD + 2);
                const float f = fw[h * FL_WARPS + w];
                L = fmaf(f, st[1], L);
                if (e >= 2) acc = fmaf(f, st[e], acc);
            }
            const float v = e == 0 ? M : (e == 1 ? L : acc);
            if (S == 1) {
                if (e >= 2) ll_store(F.out + (size_t)(g * G + h) * HD + (e - 2), acc / L, tag);
            } else if (j > 0) {
                ll_store(mine + i, v, tag);  // split j's state, taken by split 0
            } else {
                raw[i] = v;  // split 0 keeps its own state here (raw is no longer needed)
            }
        }
        if (S == 1 || j > 0) {
            mark(9);
            return true;
        }
        // split 0: take the other splits' states as they arrive, merge all S in split order
        const bool got2 = fl_poll(P, mine + G * (HD + 2), others, (S - 1) * G * (HD + 2), tag);
        if (cbar_any(!got2 || fl_abort)) return false;
        for (int i = tid; i < G * HD; i += FL_CONSUMERS) {
            const int h = i / HD, e = i % HD;
            auto st = [&](int jj) { return jj == 0 ? raw + h * (HD + 2) : others + ((jj - 1) * G + h) * (HD + 2); };
            float M = -INFINITY;
            for (int jj = 0; jj < S; jj++) M = fmaxf(M, st(jj)[0]);
            float L = 0.f, O = 0.f;
            for (int jj = 0; jj < S; jj++) {
                const float *q = st(jj);
                if (q[0] == -INFINITY) continue;
                const float f = expf(q[0] - M);
                L = fmaf(f, q[1], L);
                O = fmaf(f, q[2 + e], O);
            }
            ll_store(F.out + (size_t)(g * G + h) * HD + e, O / L, tag);
        }
        mark(9);
        return true;
    }
};

// ---- argmax, exit -------------------------------------------------------------------------

// After the lm_head phase, by the epilogue warp once it ran this CTA's last lm_head
// epilogue: publish the CTA's best key; the last CTA reduces all of them, writes the token
// and (loop mode) advances the step state.
template <bool TP>
FDEV void fl_argmax_finish(const FParams &P, uint32_t tag) {
    const int lane = threadIdx.x & 31;
    unsigned int ticket = 0;
    if (lane == 0) {
        P.am_key[blockIdx.x] = fl_best;
        __threadfence();
        ticket = atomicAdd(P.am_count, 1u);
    }
    ticket = __shfl_sync(0xffffffffu, ticket, 0);
    if (ticket != gridDim.x - 1) return;
    __threadfence();
    unsigned long long best = 0ull;
    for (int i = lane; i < (int)gridDim.x; i += 32) best = max(best, __ldcg(P.am_key + i));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if (TP && P.lm_shard) {
        // this rank's best key to every rank (two tagged words), then the largest of all
        // ranks' keys: every rank picks the same token
        if (lane < P.tp_world) {
            uint64_t *dst = P.tp_bufs[lane] + P.tp_key_off + 2 * P.tp_rank;
            ll_store_bits_sys(dst, (uint32_t)(best >> 32), tag);
            ll_store_bits_sys(dst + 1, (uint32_t)best, tag);
        }
        unsigned long long k = 0ull;
        int ok = 1;
        if (lane < P.tp_world) {
            const uint64_t *src = P.tp_bufs[P.tp_rank] + P.tp_key_off + 2 * lane;
            const unsigned long long t0 = gtimer();
            for (;;) {
                const ulonglong2 w = ll_load2_sys(src);
                if ((uint32_t)(w.x >> 32) == tag && (uint32_t)(w.y >> 32) == tag) {
                    k = ((unsigned long long)(uint32_t)w.x << 32) | (uint32_t)w.y;
                    break;
                }
                if (fl_abort || gtimer() - t0 > FL_WAIT_NS) {
                    ok = 0;
                    break;
                }
            }
        }
        if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) {
                fl_fail(P);
                *P.am_count = 0u;
            }
            return;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) k = max(k, __shfl_xor_sync(0xffffffffu, k, o));
        best = k;
    }
    if (lane == 0) {
        const int bi = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFu));
        *P.io_argmax = bi;
        if (P.loop) {
            *P.io_token = bi;
            *P.io_pos = *P.io_pos + 1;
            const int st = *P.io_step;
            P.rec_tokens[st] = bi;
            *P.io_step = st + 1;
        }
        *P.am_count = 0u;
    }
}

// The epilogue warp: walks the phases as the consumer warps do (descriptors read from
// global memory), and for each of this CTA's GEMV tiles waits until the eight warps have
// published their partial sums, runs the epilogue (residual add, SwiGLU, q|k|v store,
// logits + argmax candidate) and frees the ring slot. Attention pages take ring slots
// without an epilogue (their reader frees them). Every wait is bounded.
template <bool TP>
__device__ __noinline__ void fl_epilogue_warp(const FParams &P, int nch, int S, uint32_t tag) {
    const int lane = threadIdx.x & 31;
    const int units = P.n_kv * S, u = (int)gridDim.x - 1 - (int)blockIdx.x;
    long long seq = 0;
    uint32_t done_phase = 0;  // parity of each slot's fl_done barrier, one bit per slot
    fl_fetch_phase(&fl_E[0], P.phases, lane);
    for (int ph = 0; ph < P.n_phases; ph++) {
        cp_async_wait_all();  // descriptor ph is in fl_E[ph & 1]; fetch the next one behind it
        __syncwarp();
        if (ph + 1 < P.n_phases) fl_fetch_phase(&fl_E[(ph + 1) & 1], P.phases + ph + 1, lane);
        const FPhase &F = fl_E[ph & 1];
        const int kind = F.kind;
        if (kind == FL_ATTN) {
            if (nch > 0 && u < units) {
                const int j = u % S;
                seq += (int)((long long)(j + 1) * nch / S) - (int)((long long)j * nch / S);
            }
            continue;
        }
        float rrms = 1.0f;
        bool have_rrms = F.norm_w == nullptr;
        long long cw = 0, ce = 0;  // trace: cycles waiting for partial sums, in epilogues
        const unsigned long long t_ph = P.trace ? gtimer() : 0ull;
        if ((int)blockIdx.x < F.stage_ctas) {
            int t0, t1;
            fl_tile_range<TP>(P, F, t0, t1);
            for (int tile = t0 + blockIdx.x; tile < t1; tile += gridDim.x) {
                int sidx, lt;
                fl_locate(F, tile, sidx, lt);
                const int d = (int)(seq % FL_NDESC);
                int ok = 1;
                const long long c0 = clock64();
                if (lane == 0) {
                    ok = fl_mbar_wait_idle(&fl_done[d], (done_phase >> d) & 1u);
                    if (!ok) fl_fail(P);
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) {
                    cp_async_wait_all();  // the next descriptor's copy lands before the warp leaves
                    return;
                }
                const long long c1 = clock64();
                cw += c1 - c0;
                done_phase ^= 1u << d;
                if (!have_rrms) {  // the eight warps wrote their sums before their first tile
                    rrms = fl_rrms(F, ph);
                    have_rrms = true;
                }
                fl_epilogue<TP>(P, F, F.seg[sidx], lt, d, tag, rrms);
                __syncwarp();
                if (lane == 0) fl_release_slot(&fl_empty[d]);
                ce += clock64() - c1;
                seq++;
            }
        }
        if (kind == FL_LM) {
            __syncwarp();
            fl_argmax_finish<TP>(P, tag);
        }
        if (P.trace && lane == 0) {
            unsigned long long *tr = P.trace + ((size_t)ph * gridDim.x + blockIdx.x) * FL_TRACE_FIELDS;
            tr[8] = (unsigned long long)cw;
            tr[9] = (unsigned long long)ce;
            tr[11] = gtimer();
            tr[14] = t_ph;
        }
    }
}

// ---- producer ---------------------------------------------------------------------------

template <int HD, bool TP>
__device__ __noinline__ void fl_producer(const FParams &P, int pos, int nch, int S) {
    uint8_t *ring = fl_ring();
    int head = 0, used = 0, need[FL_NDESC];
    long long seq = 0, oldest = 0, pwait = 0;
    auto reserve = [&](int size, int align, int &d) -> uint8_t * {
        int skip, start;
        bool wrap;
        for (;;) {
            if (seq == oldest) head = 0;  // ring empty: restart at the front
            // an item that does not fit before the end starts at the front; the bytes up to
            // its (aligned) start, or up to the end, are charged to it
            start = (head + align - 1) & ~(align - 1);
            wrap = start + size > P.ring_bytes;
            if (wrap) start = 0;
            skip = wrap ? P.ring_bytes - head : start - head;
            if (seq - oldest < FL_NDESC && used + skip + size <= P.ring_bytes) break;
            const int od = (int)(oldest % FL_NDESC);
            const long long w0 = clock64();
            const bool got = fl_mbar_wait_idle(&fl_empty[od], (uint32_t)((oldest / FL_NDESC) & 1));
            pwait += clock64() - w0;
            if (!got) {
                fl_fail(P);
                return nullptr;
            }
            used -= need[od];
            oldest++;
        }
        uint8_t *dst = ring + start;
        head = start + size;
        d = (int)(seq % FL_NDESC);
        need[d] = skip + size;
        used += skip + size;
        fl_tile_off[d] = (int)(dst - ring);
        return dst;
    };
    const int units = P.n_kv * S;
    const int u = (int)gridDim.x - 1 - (int)blockIdx.x;  // this CTA's attention unit, if u < units
    for (int ph = 0; ph < P.n_phases && !fl_abort; ph++) {
        const FPhase &F = P.phases[ph];
        pwait = 0;
        if (F.kind == FL_ATTN) {
            constexpr uint32_t PAGE = ATTN_P * HD * 2;
            if (nch > 0 && u < units) {
                const int g = u / S, j = u % S;
                const int p0 = (int)((long long)j * nch / S), p1 = (int)((long long)(j + 1) * nch / S);
                for (int pg = p0; pg < p1 && !fl_abort; pg++) {
                    int d;
                    uint8_t *dst = reserve(2 * PAGE, 1024, d);  // swizzled boxes: 1024-byte aligned
                    if (!dst) break;
                    const int row = ((P.page_table[pg] * P.n_layers + F.layer) * P.n_kv + g) * ATTN_P;
                    mbar_expect_tx(&fl_full[d], 2 * PAGE);
#pragma unroll
                    for (int h = 0; h < HD / 64; h++) {
                        tma_load_2d(dst + h * 64 * 128, &P.kmap, 64 * h, row, &fl_full[d]);
                        tma_load_2d(dst + PAGE + h * 64 * 128, &P.vmap, 64 * h, row, &fl_full[d]);
                    }
                    seq++;
                }
            }
        } else {
            int t0, t1;
            fl_tile_range<TP>(P, F, t0, t1);
            for (int tile = t0 + blockIdx.x; tile < t1 && !fl_abort; tile += gridDim.x) {
                int s, lt;
                fl_locate(F, tile, s, lt);
                const PSeg &Sg = F.seg[s];
                int d;
                uint8_t *dst = reserve(TC_M * Sg.stride, 16, d);
                if (!dst) break;
                // a SwiGLU tile holds rows 8 lt .. 8 lt + 7 of gate (ring rows 0..7) and of up
                // (ring rows 8..15); other tiles rows 16 lt .. 16 lt + 15 of one matrix
                const int nm = F.kind == FL_SWIGLU ? 2 : 1, rpt = TC_M / nm;
                const int r0 = lt * rpt, nrows = min(rpt, Sg.rows - r0);
                const uint32_t mat_bytes = (uint32_t)nrows * Sg.row_bytes;
                const uint32_t main_bytes = Sg.per_row ? mat_bytes : (mat_bytes & ~15u);
                // plain-copied tail first, then the arrive (release), then the bulk copies
                for (int m = 0; m < nm; m++) {
                    const uint8_t *src = (m == 0 ? Sg.w : Sg.w2) + (size_t)r0 * Sg.row_bytes;
                    uint8_t *mdst = dst + (size_t)m * rpt * Sg.stride;
                    for (uint32_t k = main_bytes; k < mat_bytes; k++) mdst[k] = src[k];
                }
                mbar_expect_tx(&fl_full[d], main_bytes * nm);
                for (int m = 0; m < nm; m++) {
                    const uint8_t *src = (m == 0 ? Sg.w : Sg.w2) + (size_t)r0 * Sg.row_bytes;
                    uint8_t *mdst = dst + (size_t)m * rpt * Sg.stride;
                    if (Sg.per_row) {
                        for (int r = 0; r < nrows; r++)
                            bulk_g2s(mdst + (size_t)r * Sg.stride, src + (size_t)r * Sg.row_bytes, Sg.row_bytes,
                                     &fl_full[d]);
                    } else if (main_bytes) {
                        bulk_g2s(mdst, src, main_bytes, &fl_full[d]);
                    }
                }
                seq++;
            }
        }
        if (P.trace) {
            unsigned long long *tr = P.trace + ((size_t)ph * gridDim.x + blockIdx.x) * FL_TRACE_FIELDS;
            tr[6] = gtimer();
            tr[7] = (unsigned long long)pwait;
        }
    }
    // copies still in flight land before the CTA exits: the consumers wait on every
    // item; after an abort, wait (bounded) here for the issued ones
    if (fl_abort)
        for (long long k = oldest; k < seq; k++) mbar_wait(&fl_full[k % FL_NDESC], (uint32_t)((k / FL_NDESC) & 1));
}

// ---- the kernel -------------------------------------------------------------------------

// TP: the tensor-parallel instance (its norm phases add the ranks' partial sums while
// staging). The single-GPU instance references none of that staging code: with it in the
// same kernel, ptxas spilled registers in the tile loops and the attention unit (1,227 ->
// 1,060 tok/s on one GPU).
template <int HD, int G, bool TP>
__global__ void __launch_bounds__(FL_THREADS, 1) decode_flow_kernel(const __grid_constant__ FParams P) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int d = 0; d < FL_NDESC; d++) {
            mbar_init(&fl_full[d], 1);
            mbar_init(&fl_empty[d], FL_WARPS + 1);  // each consumer warp + the epilogue warp
            mbar_init(&fl_done[d], FL_WARPS);       // each consumer warp's partial sums
        }
        mbar_fence_init();
        fl_abort = 0;
        fl_best = 0ull;
        fl_tmark[0] = 0ull;
    }
    if (warp == 0) fl_fetch_phase(&fl_F[0], P.phases, lane);
    cp_async_wait_all();
    const uint32_t tag = *(volatile unsigned int *)P.epoch;
    const int pos = *P.io_pos;
    const int token0 = *P.io_token;
    __syncthreads();  // the only full-CTA barrier

    const bool pos_ok = pos >= 0 && pos < P.max_seq;
    const int nch = pos_ok ? pos / ATTN_P + 1 : 0;
    if (pos_ok && tid < HD / 2) fl_rope[tid] = __ldg(P.rope + (size_t)pos * (HD / 2) + tid);
    const int S = fl_att_splits(P, nch);
    if (!pos_ok && tid == 0 && blockIdx.x == 0) *P.io_err = 1;

    if (warp >= FL_WARPS) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(FL_REG_PRODUCER));
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(FL_REG_CONSUMER));
    }
    if (!pos_ok) {
        // nothing to decode (the host checks positions before launching; this is the
        // device-side guard): every phase is skipped, the tag still advances
    } else if (warp >= FL_WARPS) {
        if (tid == FL_CONSUMERS) fl_producer<HD, TP>(P, pos, nch, S);
        if (warp == FL_EPI_WARP) fl_epilogue_warp<TP>(P, nch, S, tag);
    } else {
        long long seq = 0;
        const int units = P.n_kv * S;
        const int u = (int)gridDim.x - 1 - (int)blockIdx.x;
        for (int ph = 0; ph < P.n_phases; ph++) {
            const FPhase &F = fl_F[ph & 1];
            unsigned long long *tr = (P.trace && tid == 0)
                                         ? P.trace + ((size_t)ph * gridDim.x + blockIdx.x) * FL_TRACE_FIELDS
                                         : nullptr;
            long long wcycles = 0;
            // every warp is past the previous phase (its epilogues included): the
            // descriptor buffer of phase ph + 1 and the staging areas are free
            if (cbar_any(fl_abort)) break;
            if (warp == 0 && ph + 1 < P.n_phases) fl_fetch_phase(&fl_F[(ph + 1) & 1], P.phases + ph + 1, lane);
            if (tr) tr[0] = gtimer();
            const long long c0 = clock64();
            bool ok = true;
            if (F.kind == FL_ATTN) {
                if (nch > 0 && u < units) ok = FlowAttn<HD, G>::unit(P, F, u / S, u % S, S, pos, nch, seq, tag, wcycles, tr);
            } else if ((int)blockIdx.x < F.stage_ctas) {
                ok = fl_stage_warp<TP>(P, F, ph, tag, token0, tr);
                if (ok) ok = fl_tiles<TP>(P, F, seq, tag, wcycles, tr);
                ok = !cbar_any(!ok || fl_abort);  // all warps past their tiles (the epilogue warp follows)
            }
            cp_async_wait_all();
            if (tr) {
                tr[3] = (unsigned long long)(clock64() - c0);
                tr[4] = (unsigned long long)wcycles;
                tr[5] = gtimer();
                if (F.kind != FL_ATTN) tr[10] = fl_tmark[0];
                fl_tmark[0] = 0ull;  // the next phase starts after a barrier
            }
            if (!ok) break;
        }
        cp_async_wait_all();
    }
    // the last CTA to exit advances the launch tag (also after an abort, so the next
    // launch never mistakes this launch's words for its own)
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(P.exit_count, 1u) == gridDim.x - 1) {
            *P.exit_count = 0u;
            *P.epoch = tag + 1u;
        }
    }
}

}  // namespace fiber
