// persistent.cuh — one decode step as one cooperative kernel.
//
// Why: a batch-1 step of the 1.1B model moves ~640 MB through ~110 dependent
// phases; launched as separate kernels, each phase pays launch, first-byte
// latency and an x-staging/epilogue chain (~5-10 us) for ~0.5-2 us of data.
// Here every SM runs one CTA for the whole step:
//   * warp 8 (producer, one lane) walks the CTA's weight tiles of ALL phases in
//     consumption order, and the K/V pages of its attention units, and streams
//     them with cp.async.bulk into a shared-memory byte ring (FIFO, an mbarrier
//     full/empty pair per tile in flight), so loading runs ahead across phase
//     boundaries and barrier waits;
//   * warps 0..7 (consumers) wait for the phase's input (grid barrier), copy it
//     in as fp16 hi/lo MMA fragments, decode + multiply each tile on the tensor
//     cores (TcDot) and run the phase's epilogue, which writes the next phase's
//     input fragments (times the next RMSNorm weights) and per-CTA sums of
//     squares, so the RMSNorm scale is applied to the next phase's dot products;
//     consumers synchronise among themselves with named barrier 1, never with
//     the producer;
//   * between phases a grid barrier: one arrive counter per phase in global
//     memory (zeroed before each launch), polled with bounded spins.
// Phases per token: per layer QKV (layer 0 stages the embedding row itself),
// attention (RoPE, KV append, per-unit partial softmax over prefetched pages),
// attention merged by the last unit of each KV head into Wo's input, Wo (+residual), gate/up
// (+RMSNorm, SwiGLU), down (+residual); then lm_head (+RMSNorm, greedy argmax).
// Each phase body is a separate non-inlined function so that its registers are
// allocated on its own; the per-CTA state lives in shared memory.
// Every wait is bounded: on timeout the kernel records an error code (4) in the
// step state, stops issuing work and returns once its own copies have landed.
#pragma once
#include "attention.cuh"
#include "gemv_tc.cuh"

namespace fiber {

constexpr int PK_CONSUMERS = 256;               // 8 warps
constexpr int PK_WARPS = PK_CONSUMERS / 32;
constexpr int PK_THREADS = PK_CONSUMERS + 32;   // + producer warp
constexpr int PK_NDESC = 16;                    // tiles in flight per CTA
constexpr int PK_RPRE = 8;                      // residual rows prefetched for this many tiles
constexpr long long PK_SPIN_LIMIT = 1ll << 24;  // grid-barrier polls (also limited to PK_WAIT_NS)
// Optional per-phase, per-CTA timeline (PParams::trace non-null), fields:
//  0 globaltimer (ns) when the phase's grid barrier released the CTA
//  1 SM cycles from the phase start to that release     2 cycles staging the input vector
//  3 cycles in the tile loop (or attention units)   4 of those waiting for tiles to land
//  5 cycles from the end of the tile loop to the arrive
//  6 producer: globaltimer (ns) after issuing the phase's last tile   7 producer: cycles waiting for ring space
//  8, 9 attention: cycles until q/k/v are staged, cycles of the page loop (first head of the CTA)
constexpr int PK_TRACE_FIELDS = 10;

enum : int { PH_QKV = 0, PH_ATTN = 1, PH_RESID = 2, PH_SWIGLU = 3, PH_LM = 4 };

struct PSeg {
    const uint8_t *w, *w2;
    int type;
    int rows;
    int out_off;
    int tiles;
    int row_bytes;  // bytes of one weight row in HBM
    int stride;     // bytes of one row in the ring
    int per_row;    // 1: one bulk copy per row; 0: one per tile (plus a plain-copied tail)
};

struct __align__(16) PPhase {
    int kind;
    int nseg;
    int nmat;       // 2 for SwiGLU (gate + up), else 1
    int cols;
    int layer;
    int n_tiles;
    int embed_in;   // 1: the input is the embedding row of the current token
    float eps;
    const float *x;
    const float *norm_w;
    float *y;
    float *resid;
    // input of the phase as MMA fragments (written by the previous phase): one
    // layout per weight type of the phase, 4 * cols bytes each; null for the
    // embedding input, which the phase stages itself
    const uint2 *gf_in;
    const float *ss_in;     // per-CTA sums of squares of the input (RMSNorm), or null
    // outputs that feed the next phase: its input fragments (value * nw_out) and
    // per-CTA sums of squares (ss_out), when this phase's outputs are its input
    uint16_t *gf_out;
    const float *nw_out;    // RMSNorm weights of the next phase, or null
    float *ss_out;          // [gridDim.x] partial sums of squares, or null
    int out_types[2];       // weight types of the next phase's layouts (-1: none)
    int n_out;              // elements of the next phase's input
    int pad_;
    PSeg seg[3];
};
static_assert(sizeof(PPhase) % 16 == 0 && sizeof(PPhase) / 16 <= 32, "phase descriptors are copied in 16-byte chunks");

// Largest activation magnitude the fp16 hi/lo fragments represent; beyond it
// the step reports error 5 instead of computing with an overflowed input.
constexpr float PK_FRAG_MAX = 65504.0f;

struct PParams {
    const PPhase *phases;  // device array
    int n_phases;
    unsigned int *bar;     // [n_phases] arrive counters, zero at launch
    const uint8_t *embd;
    int embd_type;
    int dim, vocab;
    float *x;              // residual stream
    AttnParams attn;
    float2 *am_part;       // [gridDim.x]
    unsigned int *am_count;
    int32_t *io_token, *io_pos, *io_argmax, *io_err, *io_step;
    int32_t *rec_tokens;
    int loop;              // 1: feed argmax back as next token, advance pos, record it
    int ring_bytes;
    int xf_bytes;          // fragment region (one or two staged types)
    int xs_floats;         // fp32 staging copy of x
    int nw_floats;         // RMSNorm weights of the phase (prefetched)
    unsigned long long *trace;  // [n_phases][gridDim.x][PK_TRACE_FIELDS] or null
};

// ---- per-CTA state (shared memory) -------------------------------------------------
// dynamic: [ring ring_bytes][fragments xf_bytes][xs xs_floats][norm weights nw_floats]
extern __shared__ __align__(128) uint8_t pk_dyn[];
__shared__ __align__(8) uint64_t pk_full[PK_NDESC];
__shared__ __align__(8) uint64_t pk_empty[PK_NDESC];
__shared__ __align__(16) PPhase pk_F[2];         // descriptors of the current and the next phase
__shared__ __align__(16) float pk_rpre[PK_RPRE * TC_M];   // residual rows of this CTA's first tiles
__shared__ __align__(16) float pk_nwpre[PK_RPRE * TC_M];  // next phase's norm weights for those rows
__shared__ __align__(16) float pk_ssin[256];              // per-CTA sums of squares of the input
__shared__ float pk_red[PK_WARPS * 2 * TC_M];
__shared__ float2 pk_cand[PK_WARPS];
__shared__ float pk_stat[2 * PK_WARPS];
__shared__ unsigned int pk_ticket;
__shared__ volatile int pk_abort;                // set by any thread that gives up (producer included)
__shared__ int pk_stop;                          // consumers' uniform copy, written by thread 0 before a barrier
__shared__ int pk_gstop;                         // the same for the grid-barrier wait
__shared__ int pk_tile_off[PK_NDESC];            // ring offset of each tile in flight (producer -> consumers)

FDEV uint8_t *pk_ring() { return pk_dyn; }
FDEV uint2 *pk_xf(const PParams &P) { return reinterpret_cast<uint2 *>(pk_dyn + P.ring_bytes); }
FDEV float *pk_xs(const PParams &P) { return reinterpret_cast<float *>(pk_dyn + P.ring_bytes + P.xf_bytes); }
FDEV float *pk_nws(const PParams &P) { return pk_xs(P) + P.xs_floats; }

FDEV unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

FDEV void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(PK_CONSUMERS) : "memory"); }
FDEV void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// n arrivals at once (a ring slot's empty barrier expects one per consumer warp)
FDEV void mbar_arrive_n(uint64_t *bar, uint32_t n) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(n) : "memory");
}

FDEV int tile_bytes_of(const PSeg &s, int nmat) { return nmat * TC_M * s.stride; }

FDEV void locate_p(const PPhase &F, int tile, int &s, int &lt) {
    s = 0;
    lt = tile;
    while (s + 1 < F.nseg && lt >= F.seg[s].tiles) lt -= F.seg[s++].tiles;
}

FDEV uint32_t ld_acquire_u32(const unsigned int *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

FDEV void cp_async16(void *sdst, const void *gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(sdst)), "l"(gsrc) : "memory");
}
FDEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Copy phase descriptor `src` into shared memory with 16-byte async copies
// (lanes of one warp); complete after cp_async_wait_all + a barrier.
FDEV void pk_fetch_phase(PPhase *dst, const PPhase *src, int lane) {
    constexpr int CH = (int)(sizeof(PPhase) / 16);
    if (lane < CH) cp_async16(reinterpret_cast<uint4 *>(dst) + lane, reinterpret_cast<const uint4 *>(src) + lane);
}

// mbarrier wait that suspends the thread (up to hint_ns) instead of spinning, so
// a waiting thread takes no issue slots from the warps that share its scheduler.
constexpr unsigned long long PK_WAIT_NS = 2000000000ull;  // a ring wait gives up after 2 s

// Bounded mbarrier wait (time-limited) that also gives up when another thread
// has aborted.
FDEV bool pk_mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
FDEV bool pk_mbar_wait(uint64_t *bar, uint32_t parity) {
    if (pk_mbar_try_wait(bar, parity)) return true;  // usual case: no timer read
    const unsigned long long t0 = gtimer();
    for (;;) {
        if (pk_mbar_try_wait(bar, parity)) return true;
        if (pk_abort || gtimer() - t0 > PK_WAIT_NS) return false;
    }
}

// Per-thread trace marks (thread 0 of the consumers; tr is null otherwise).
struct PkTrace {
    unsigned long long *tr;
    long long ck;
    FDEV void mark(int field) {
        if (tr) {
            const long long n = clock64();
            tr[field] = (unsigned long long)(n - ck);
            ck = n;
        }
    }
    FDEV void put(int field, unsigned long long v) {
        if (tr) tr[field] = v;
    }
};

// ---- consumer side of the ring -------------------------------------------------------
// Every consumer thread calls acquire/release in the same order; thread 0 alone
// waits on the mbarrier (bounded) and publishes the stop decision before the
// barrier, so all threads agree. acquire returns null when the step stops.
FDEV const uint8_t *ring_acquire(const PParams &P, int seq, long long &wfull) {
    const int d = seq % PK_NDESC;
    if (threadIdx.x == 0) {
        const long long w0 = clock64();
        if (!pk_mbar_wait(&pk_full[d], (uint32_t)((seq / PK_NDESC) & 1))) {
            pk_abort = 1;
            *P.io_err = 4;
        }
        wfull += clock64() - w0;
        pk_stop = pk_abort;
    }
    cbar();
    return pk_stop ? nullptr : pk_ring() + pk_tile_off[d];
}
FDEV void ring_release(int seq) {
    cbar();
    if (threadIdx.x == 0) mbar_arrive_n(&pk_empty[seq % PK_NDESC], PK_WARPS);  // for all eight warps
}

// Wait until every CTA has finished phase ph - 1 (all consumer threads; thread 0
// polls the arrive counter with bounded spins and publishes the stop decision
// before the barrier). Also completes this thread's async copies.
FDEV bool pk_grid_wait(const PParams &P, int ph) {
    if (threadIdx.x == 0) {
        if (ph > 0) {
            bool ok = false;
            const unsigned int *cnt = P.bar + (ph - 1);
            const unsigned long long t0 = gtimer();
            for (long long i = 0; i < PK_SPIN_LIMIT; i++) {  // each poll is an L2 round trip
                if (ld_acquire_u32(cnt) >= gridDim.x) {
                    ok = true;
                    break;
                }
                if ((i & 63) == 63 && (pk_abort || gtimer() - t0 > PK_WAIT_NS)) break;
            }
            if (!ok) {
                pk_abort = 1;
                *P.io_err = 4;
            }
        }
        pk_gstop = pk_abort;
    }
    cp_async_wait_all();
    cbar();
    return !pk_gstop;
}

// ---- GEMV pieces ---------------------------------------------------------------------

// Fragments of the staged input for weight type T: fp16 hi/lo pairs of
// scale * x[k] (times rrms * norm[k] where the phase has an RMSNorm), in the
// k-slot order TcDot<T> consumes (TcType<T>::elem). Reads x and the norm
// weights from shared memory.
template <int T>
FDEV void pk_stage(int nb, const float *xs, const float *nws, float rrms, float scale, uint2 *xf) {
    for (int f = threadIdx.x; f < nb * 64; f += PK_CONSUMERS) {
        const int b = f >> 6, s = (f >> 2) & 15, t = f & 3;
        __half hi[4], lo[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int k = b * 256 + TcType<T>::elem(t, s, i);
            float v = xs[k];
            if (nws) v = __fmul_rn(__fmul_rn(v, rrms), nws[k]);
            v *= scale;
            hi[i] = __float2half_rn(v);
            lo[i] = __float2half_rn(v - __half2float(hi[i]));
        }
        xf[2 * f + 0] = make_uint2((uint32_t)__half_as_ushort(hi[0]) | ((uint32_t)__half_as_ushort(hi[1]) << 16),
                                   (uint32_t)__half_as_ushort(hi[2]) | ((uint32_t)__half_as_ushort(hi[3]) << 16));
        xf[2 * f + 1] = make_uint2((uint32_t)__half_as_ushort(lo[0]) | ((uint32_t)__half_as_ushort(lo[1]) << 16),
                                   (uint32_t)__half_as_ushort(lo[2]) | ((uint32_t)__half_as_ushort(lo[3]) << 16));
    }
}

// Input element k (of a phase whose weights are of type T) as fp16 hi/lo pair
// into fragment layout gf: group f = (k/256)*64 + s*4 + t holds 8 halves, the
// four hi slots then the four lo slots (the order pk_stage writes and TcDot reads).
template <int T>
FDEV void pk_frag_put(uint16_t *gf, int k, float v) {
    int t = 0, s = 0, i = 0;
    TcType<T>::pos(k & 255, t, s, i);
    const int f = (k >> 8) * 64 + s * 4 + t;
    const __half hi = __float2half_rn(v);
    const __half lo = __float2half_rn(v - __half2float(hi));
    gf[8 * f + i] = __half_as_ushort(hi);
    gf[8 * f + 4 + i] = __half_as_ushort(lo);
}

// Write v as element k of the next phase's input, in each of its layouts.
// Returns false (nothing written) when v is outside the fragment range.
FDEV bool pk_frag_out(const PPhase &F, int k, float v) {
    if (!(fabsf(v) < PK_FRAG_MAX)) return false;
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const int ty = F.out_types[j];
        if (ty < 0) break;
        uint16_t *gf = F.gf_out + (size_t)j * 2 * F.n_out;
        switch (ty) {
        case T_Q4_K: pk_frag_put<T_Q4_K>(gf, k, v); break;
        case T_Q6_K: pk_frag_put<T_Q6_K>(gf, k, v); break;
        default: pk_frag_put<T_F16>(gf, k, v); break;
        }
    }
    return true;
}

// One tile (16 rows of each of NMAT matrices) against the staged fragments:
// warp w takes super-blocks w, w + 8, ...; its per-row partial sums go to pk_red.
template <int T, int NMAT>
FDEV void pk_dot(const uint8_t *buf, int stride, const uint2 *xf, int nb) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    float acc[NMAT][4];
#pragma unroll
    for (int m = 0; m < NMAT; m++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[m][i] = 0.f;
    for (int b = warp; b < nb; b += PK_WARPS) {
        const uint2 *xfb = xf + (size_t)b * 128;
#pragma unroll
        for (int m = 0; m < NMAT; m++) {
            const uint8_t *mb = buf + (size_t)m * TC_M * stride + (size_t)b * TcType<T>::BB;
            TcDot<T>::run(mb + (size_t)g * stride, mb + (size_t)(g + 8) * stride, xfb, g, t, acc[m]);
        }
    }
    if (t == 0) {
#pragma unroll
        for (int m = 0; m < NMAT; m++) {
            pk_red[(warp * 2 + m) * TC_M + g] = acc[m][0] + acc[m][1];
            pk_red[(warp * 2 + m) * TC_M + g + 8] = acc[m][2] + acc[m][3];
        }
    }
}

// ---- attention -----------------------------------------------------------------------

// One query head h of the attention phase, on one CTA. Threads 0..HD/2-1 rotate
// q and the new position's k (RoPE), the next HD threads round the new v row, at
// the same time; the CTA holding query head g*G (g = h's KV head) appends the new
// K/V row (fp16) to the cache. The KV head's pages come through the ring (the
// producer prefetched them, in page order) and every warp works on every page:
// warp w takes the page's positions 8w .. 8w+7, four lanes per position, each
// lane a quarter of the head dims (q in registers; K words read in a per-lane
// rotated order, so the 32 lanes read 32 distinct banks), then the softmax
// weights of those positions and their P.V (lane = head dims lane, lane + 32, ..),
// combined online across pages (max, sum, o). A page's ring slot is free when all
// eight warps have arrived on its empty barrier. The position being decoded is
// taken from the fresh rows (nk, nv), not from the page copy, which may predate
// the append. The eight warp results are merged in shared memory in warp order and
// the head's output is written as Wo's input fragments (elements h*hd .. h*hd +
// hd - 1). Returns false when the step stopped.
template <int HD, int G>
FDEV bool pk_attn_head(const PParams &P, const PPhase &F, int h, int pos, int nch, int &seq, long long &wfull,
                       unsigned long long *tr) {
    const long long c0 = clock64();
    constexpr int PG = ATTN_P;
    constexpr int W = HD / 2;          // 32-bit words of a K/V row
    constexpr int DPL = HD / 32;       // head dims per lane in P.V
    constexpr int PW = PG / PK_WARPS;  // positions of a page per warp
    constexpr int QW = W / 4;          // K words per lane (a quarter of the row)
    static_assert(PW == 8 && (QW == 8 || QW == 16), "eight warps, head_dim 64 or 128");
    const AttnParams &a = P.attn;
    uint8_t *sm = reinterpret_cast<uint8_t *>(pk_xf(P));
    float *qs = reinterpret_cast<float *>(sm);                       // [HD] rotated q
    uint16_t *nk = reinterpret_cast<uint16_t *>(sm + HD * 4);        // [HD] new K row (fp16)
    uint16_t *nv = nk + HD;                                          // [HD] new V row (fp16)
    float *wm = reinterpret_cast<float *>(sm + HD * 4 + HD * 4);     // [PK_WARPS][HD + 2] warp results
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = h / G, seqlen = pos + 1, tn = pos - (nch - 1) * PG;
    const bool writer = h % G == 0;  // appends the new K/V row of KV head g
    const size_t base = (((size_t)a.page_table[nch - 1] * a.n_layers + F.layer) * a.n_kv + g) * (size_t)PG * HD;
    if (tid < HD / 2) {
        const int j = tid;
        const float2 cs = __ldg(a.rope + (size_t)pos * (HD / 2) + j);
        const float *qh = a.qkv + (size_t)h * HD;
        const float *kr = a.qkv + (size_t)a.n_heads * HD + (size_t)g * HD;
        const float x1 = __ldcg(qh + j), x2 = __ldcg(qh + j + HD / 2);
        const float k1 = __ldcg(kr + j), k2 = __ldcg(kr + j + HD / 2);
        qs[j] = __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y));
        qs[j + HD / 2] = __fadd_rn(__fmul_rn(x1, cs.y), __fmul_rn(x2, cs.x));
        const uint16_t y1 = __half_as_ushort(__float2half_rn(__fsub_rn(__fmul_rn(k1, cs.x), __fmul_rn(k2, cs.y))));
        const uint16_t y2 = __half_as_ushort(__float2half_rn(__fadd_rn(__fmul_rn(k1, cs.y), __fmul_rn(k2, cs.x))));
        nk[j] = y1;
        nk[j + HD / 2] = y2;
        if (writer) {
            a.k_pool[base + (size_t)tn * HD + j] = y1;
            a.k_pool[base + (size_t)tn * HD + j + HD / 2] = y2;
        }
    } else if (tid < HD / 2 + HD) {
        const int j = tid - HD / 2;
        const float *vr = a.qkv + (size_t)a.n_heads * HD + (size_t)(a.n_kv + g) * HD;
        const uint16_t h16 = __half_as_ushort(__float2half_rn(__ldcg(vr + j)));
        nv[j] = h16;
        if (writer) a.v_pool[base + (size_t)tn * HD + j] = h16;
    }
    cbar();  // qs, nk, nv ready
    const long long c1 = clock64();

    // lane roles: position pi of the warp's eight, quarter qq of the head dims
    const int pi = lane >> 2, qq = lane & 3;
    const int rot = QW == 8 ? pi : 2 * pi + (qq >> 1);  // word rotation (bank = qq*QW + rotated word, mod 32)
    float qr[2 * QW];
#pragma unroll
    for (int i = 0; i < QW; i++) {
        const float2 v = *reinterpret_cast<const float2 *>(qs + qq * 2 * QW + 2 * ((i + rot) & (QW - 1)));
        qr[2 * i] = v.x;
        qr[2 * i + 1] = v.y;
    }
    const int tw = warp * PW;  // this warp's first position in a page
    float m_run = -INFINITY, l_run = 0.f, o_run[DPL];
#pragma unroll
    for (int j = 0; j < DPL; j++) o_run[j] = 0.f;
    bool stopped = false;
    for (int pg = 0; pg < nch; pg++) {
        const long long sq = seq + pg;
        const int d = (int)(sq % PK_NDESC);
        int got = 1;
        if (lane == 0) {
            const long long w0 = clock64();
            got = pk_mbar_wait(&pk_full[d], (uint32_t)((sq / PK_NDESC) & 1));
            if (!got) {
                pk_abort = 1;
                *P.io_err = 4;
            }
            if (tid == 0) wfull += clock64() - w0;
        }
        if (!__shfl_sync(0xffffffffu, got, 0)) {
            stopped = true;
            break;
        }
        const uint8_t *tile = pk_ring() + pk_tile_off[d];
        const int nt = min(PG, seqlen - pg * PG);  // valid positions of the page
        const bool last = pg == nch - 1;
        const int t = tw + pi;
        // score of position t: this lane's quarter, then the four quarters
        float d0 = 0.f, d1 = 0.f;
        if (t < nt) {
            const uint32_t *krow = ((last && t == tn) ? reinterpret_cast<const uint32_t *>(nk)
                                                      : reinterpret_cast<const uint32_t *>(tile) + (size_t)t * W) +
                                   qq * QW;
#pragma unroll
            for (int i = 0; i < QW; i++) {
                const float2 kf = __half22float2(*reinterpret_cast<const __half2 *>(krow + ((i + rot) & (QW - 1))));
                d0 = fmaf(qr[2 * i], kf.x, d0);
                d1 = fmaf(qr[2 * i + 1], kf.y, d1);
            }
        }
        float s = d0 + d1;
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        s = t < nt ? __fmul_rn(s, a.scale) : -INFINITY;
        const int nvw = min(PW, nt - tw);  // valid positions of this warp (warp-uniform)
        if (nvw > 0) {
            float m = fmaxf(s, __shfl_xor_sync(0xffffffffu, s, 4));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
            const float M = fmaxf(m_run, m);
            const float p = t < nt ? expf(s - M) : 0.f;
            const float al = m_run == -INFINITY ? 0.f : expf(m_run - M);
            // running sum per lane (this lane's position); the lanes are summed after the pages
            l_run = fmaf(al, l_run, p);
            const uint16_t *vpg = reinterpret_cast<const uint16_t *>(tile) + (size_t)PG * HD;
            // P.V over the warp's positions: every row of the page copy is in bounds, so the
            // loads are unconditional and invalid positions are zeroed by a select
            float vv[PW][DPL], pw[PW];
#pragma unroll
            for (int u = 0; u < PW; u++) {
                pw[u] = __shfl_sync(0xffffffffu, p, 4 * u);
                const uint16_t *vrow = (last && tw + u == tn) ? nv : vpg + (size_t)(tw + u) * HD;
#pragma unroll
                for (int j = 0; j < DPL; j++) {
                    const float v = __half2float(__ushort_as_half(vrow[lane + 32 * j]));
                    vv[u][j] = u < nvw ? v : 0.f;
                }
            }
#pragma unroll
            for (int j = 0; j < DPL; j++) {
                float ov = 0.f;
#pragma unroll
                for (int u = 0; u < PW; u++) ov = fmaf(pw[u], vv[u][j], ov);
                o_run[j] = fmaf(al, o_run[j], ov);
            }
            m_run = M;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&pk_empty[d]);  // this warp is done with the page
    }
    // the warp's sum over its eight positions (lanes of one quarter; all quarters agree)
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 4);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 8);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 16);
    // warp results -> shared memory, merged in warp order (trace: 8 = q/k/v ready, 9 = page loop)
    float *wr = wm + warp * (HD + 2);
#pragma unroll
    for (int j = 0; j < DPL; j++) wr[2 + lane + 32 * j] = o_run[j];
    if (lane == 0) {
        wr[0] = stopped ? -INFINITY : m_run;
        wr[1] = l_run;
    }
    cbar();
    if (tid == 0) pk_stop = pk_abort;
    if (tr) {
        tr[8] = (unsigned long long)(c1 - c0);
        tr[9] = (unsigned long long)(clock64() - c1);
    }
    seq += nch;
    bool ok = true;
    for (int dd = tid; dd < HD; dd += PK_CONSUMERS) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < PK_WARPS; w++) M = fmaxf(M, wm[w * (HD + 2)]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < PK_WARPS; w++) {
            const float mw = wm[w * (HD + 2)];
            if (mw == -INFINITY) continue;  // a warp without positions
            const float e = expf(mw - M);
            L = fmaf(e, wm[w * (HD + 2) + 1], L);
            O = fmaf(e, wm[w * (HD + 2) + 2 + dd], O);
        }
        ok &= pk_frag_out(F, h * HD + dd, O / L);
    }
    if (!ok) *P.io_err = 5;
    cbar();  // pk_stop published; shared memory reused by the next head
    return !pk_stop;
}

// Attention phase: this CTA's query heads. Returns false when stopped.
template <int HD, int G>
__device__ __noinline__ bool pk_attn_phase(const PParams &P, const PPhase &F, int pos, int nch, int &seq,
                                           long long &wfull, unsigned long long *tr) {
    if (pos < 0 || pos >= P.attn.max_seq) {
        if (threadIdx.x == 0 && blockIdx.x == 0) *P.io_err = 1;
        return true;
    }
    for (int h = blockIdx.x; h < P.attn.n_heads; h += gridDim.x)
        if (!pk_attn_head<HD, G>(P, F, h, pos, nch, seq, wfull, h == (int)blockIdx.x ? tr : nullptr)) return false;
    return true;
}

// ---- GEMV phase ----------------------------------------------------------------------

// Layer 0: every CTA decodes the embedding row of the current token, sums its
// squares and stages x * norm as fragments itself; returns the RMSNorm scale.
__device__ __noinline__ float pk_stage_embed(const PParams &P, const PPhase &F, int token0, int type_a, int type_b) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n = F.cols, nb = n >> 8;
    uint2 *xf0 = pk_xf(P), *xf1 = xf0 + (size_t)nb * 128;
    float rrms = 1.0f;
    // embedding row of the current token: every CTA decodes it, sums its
    // squares and stages x * norm itself
    const float *nw = F.norm_w ? pk_nws(P) : nullptr;
    float *xs = pk_xs(P);
    int tok = token0;
    if (tok < 0 || tok >= P.vocab) {
        if (tid == 0 && blockIdx.x == 0) *P.io_err = 2;
        tok = 0;
    }
    float ss = 0.f;
    for (int i = tid; i < n; i += PK_CONSUMERS) {
        float v;
        switch (P.embd_type) {
        case T_F16: v = h2f(reinterpret_cast<const uint16_t *>(P.embd)[(size_t)tok * n + i]); break;
        case T_F32: v = round_f16(reinterpret_cast<const float *>(P.embd)[(size_t)tok * n + i]); break;
        case T_Q4_K: v = round_f16(decode_elem<T_Q4_K>(P.embd + ((size_t)tok * (n >> 8) + (i >> 8)) * 144, i & 255)); break;
        case T_Q5_K: v = round_f16(decode_elem<T_Q5_K>(P.embd + ((size_t)tok * (n >> 8) + (i >> 8)) * 176, i & 255)); break;
        default: v = round_f16(decode_elem<T_Q6_K>(P.embd + ((size_t)tok * (n >> 8) + (i >> 8)) * 210, i & 255)); break;
        }
        xs[i] = v;
        if (blockIdx.x == 0) P.x[i] = v;  // the residual stream starts as the embedding
        ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) pk_stat[warp] = ss;
    cbar();
    ss = 0.f;
#pragma unroll
    for (int w = 0; w < PK_WARPS; w++) ss += pk_stat[w];
    if (nw) rrms = 1.0f / sqrtf(ss / (float)n + F.eps);
    for (int pass = 0; pass < (type_b >= 0 ? 2 : 1); pass++) {
        uint2 *dst = pass ? xf1 : xf0;
        switch (pass ? type_b : type_a) {
        case T_Q4_K: pk_stage<T_Q4_K>(nb, xs, nw, 1.0f, 1.0f, dst); break;
        case T_Q6_K: pk_stage<T_Q6_K>(nb, xs, nw, 1.0f, 1.0f, dst); break;
        default: pk_stage<T_F16>(nb, xs, nw, 1.0f, 1.0f, dst); break;
        }
    }
    cbar();
    return rrms;
}

// One GEMV phase of this CTA: stage the input fragments (written by the previous
// phase, or the embedding row staged here), then decode + multiply its tiles
// from the ring and apply the epilogue, which also writes the next phase's
// input fragments. Returns false when the step stopped.
template <int HD, int G>
__device__ __noinline__ bool pk_gemv_phase(const PParams &P, const PPhase &F, int ph, int token0, int &seq,
                                           long long &wfull, float &best_v, int &best_i, PkTrace &T) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n = F.cols, nb = n >> 8;
    if (!pk_grid_wait(P, ph)) return false;
    T.put(0, gtimer());
    T.mark(1);

    // layouts: one per weight type of the phase (at most two: QKV may mix Q4_K and Q6_K)
    const int type_a = F.seg[0].type;
    int type_b = -1;
    for (int k = 1; k < F.nseg; k++)
        if (F.seg[k].type != type_a && type_b < 0) type_b = F.seg[k].type;
    uint2 *xf0 = pk_xf(P), *xf1 = xf0 + (size_t)nb * 128;  // second layout follows the first
    float rrms = 1.0f;
    if (F.embed_in) {
        rrms = pk_stage_embed(P, F, token0, type_a, type_b);
    } else {
        // fragments and per-CTA sums of squares written by the previous phase
        const int chunks = (type_b >= 0 ? 2 : 1) * (n >> 2);  // 16-byte chunks, 4n bytes per layout
        for (int c = tid; c < chunks; c += PK_CONSUMERS) cp_async16(xf0 + 2 * c, F.gf_in + 2 * c);
        if (F.ss_in)
            for (int c = tid; c < ((int)gridDim.x + 3) / 4; c += PK_CONSUMERS) cp_async16(pk_ssin + 4 * c, F.ss_in + 4 * c);
        cp_async_wait_all();
        cbar();
        if (F.ss_in && warp == 0) {
            // sum of the per-CTA partials: fixed per-lane strides, then a fixed tree
            float ss = 0.f;
            for (int i = lane; i < (int)gridDim.x; i += 32) ss += pk_ssin[i];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            rrms = 1.0f / sqrtf(ss / (float)n + F.eps);
        }
    }
    T.mark(2);

    // ---- tiles of this CTA
    const int my_tiles = (F.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    float ssacc = 0.f;
    bool ok = true;
    for (int k = 0; k < my_tiles; k++) {
        const int tile = (int)blockIdx.x + k * (int)gridDim.x;
        int sidx, lt;
        locate_p(F, tile, sidx, lt);
        const PSeg &S = F.seg[sidx];
        const uint8_t *buf = ring_acquire(P, seq, wfull);
        if (!buf) return false;
        const uint2 *xf = (S.type == type_a) ? xf0 : xf1;
        if (F.nmat == 2) {
            switch (S.type) {
            case T_Q4_K: pk_dot<T_Q4_K, 2>(buf, S.stride, xf, nb); break;
            case T_Q6_K: pk_dot<T_Q6_K, 2>(buf, S.stride, xf, nb); break;
            default: pk_dot<T_F16, 2>(buf, S.stride, xf, nb); break;
            }
        } else {
            switch (S.type) {
            case T_Q4_K: pk_dot<T_Q4_K, 1>(buf, S.stride, xf, nb); break;
            case T_Q6_K: pk_dot<T_Q6_K, 1>(buf, S.stride, xf, nb); break;
            default: pk_dot<T_F16, 1>(buf, S.stride, xf, nb); break;
            }
        }
        ring_release(seq);  // tile consumed, partials visible
        if (tid < TC_M) {
            const int r = lt * TC_M + tid;
            float v0 = 0.f, v1 = 0.f;
#pragma unroll
            for (int w = 0; w < PK_WARPS; w++) v0 += pk_red[(w * 2) * TC_M + tid];
            v0 *= rrms;
            if (F.nmat == 2) {
#pragma unroll
                for (int w = 0; w < PK_WARPS; w++) v1 += pk_red[(w * 2 + 1) * TC_M + tid];
                v1 *= rrms;
            }
            if (r < S.rows) {
                if (F.kind == PH_QKV) {
                    F.y[S.out_off + r] = v0;
                } else if (F.kind == PH_RESID) {
                    const bool pre = k < PK_RPRE && (r & ~3) + 4 <= S.rows;  // fetched before the barrier
                    const float xv = __fadd_rn(pre ? pk_rpre[k * TC_M + tid] : __ldcg(F.resid + r), v0);
                    F.resid[r] = xv;
                    if (F.ss_out) ssacc = fmaf(xv, xv, ssacc);
                    if (F.gf_out) {
                        const float nwv = F.nw_out ? (pre ? pk_nwpre[k * TC_M + tid] : __ldg(F.nw_out + r)) : 1.0f;
                        ok &= pk_frag_out(F, r, F.nw_out ? __fmul_rn(xv, nwv) : xv);
                    }
                } else if (F.kind == PH_SWIGLU) {
                    const float h = __fmul_rn(__fdiv_rn(v0, __fadd_rn(1.0f, expf(-v0))), v1);
                    F.y[r] = h;
                    if (F.gf_out) ok &= pk_frag_out(F, r, h);
                } else {  // PH_LM
                    F.y[r] = v0;
                    if (better(v0, r, best_v, best_i)) {
                        best_v = v0;
                        best_i = r;
                    }
                }
            }
        }
        cbar();  // pk_red reused by the next tile
        seq++;
    }
    if (F.ss_out && warp == 0) {
        // this CTA's sum of squares of its output rows (threads 0..15 hold them)
        float v = tid < TC_M ? ssacc : 0.f;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) F.ss_out[blockIdx.x] = v;
    }
    if (!ok) *P.io_err = 5;
    return true;
}

// Greedy argmax after the lm_head phase: CTA candidate, then the last CTA reduces
// all candidates, publishes the token and (loop mode) advances the step state.
FDEV void pk_argmax_finish(const PParams &P, float best_v, int best_i) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
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
            P.am_part[blockIdx.x] = make_float2(best_v, __int_as_float(best_i));
            __threadfence();
            pk_ticket = atomicAdd(P.am_count, 1u);
        }
    }
    cbar();
    if (pk_ticket != gridDim.x - 1) return;
    __threadfence();
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < (int)gridDim.x; i += PK_CONSUMERS) {
        const float2 e2 = __ldcg(P.am_part + i);
        const int ei = __float_as_int(e2.y);
        if (better(e2.x, ei, bv, bi)) {
            bv = e2.x;
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
    if (lane == 0) pk_cand[warp] = make_float2(bv, __int_as_float(bi));
    cbar();
    if (tid == 0) {
        for (int w = 1; w < PK_WARPS; w++) {
            const int wi = __float_as_int(pk_cand[w].y);
            if (better(pk_cand[w].x, wi, bv, bi)) {
                bv = pk_cand[w].x;
                bi = wi;
            }
        }
        if (bi == 0x7fffffff) bi = 0;
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

// ---- producer ------------------------------------------------------------------------

// Single-thread producer: ring space for the next tile is a slot and `size`
// contiguous bytes (the ring's end is skipped when the tile would straddle it).
template <int HD>
__device__ __noinline__ void pk_producer(const PParams &P, int pos, int nch) {
    uint8_t *ring = pk_ring();
    int head = 0, used = 0, need[PK_NDESC];
    long long seq = 0, oldest = 0, pwait = 0;
    auto reserve = [&](int size, int &d) -> uint8_t * {
        int skip;
        bool wrap;
        for (;;) {
            if (seq == oldest) head = 0;  // ring empty: restart at the front
            // a tile that does not fit before the end starts at the front; the bytes up to
            // the end (none when the last tile ended exactly there) are charged to it
            wrap = head + size > P.ring_bytes;
            skip = wrap ? P.ring_bytes - head : 0;
            if (seq - oldest < PK_NDESC && used + skip + size <= P.ring_bytes) break;
            const int od = (int)(oldest % PK_NDESC);
            const long long w0 = clock64();
            const bool got = pk_mbar_wait(&pk_empty[od], (uint32_t)((oldest / PK_NDESC) & 1));
            pwait += clock64() - w0;
            if (!got) {
                pk_abort = 1;
                *P.io_err = 4;
                return nullptr;
            }
            used -= need[od];
            oldest++;
        }
        if (wrap) head = 0;  // also when skip is 0: head == ring_bytes is past the ring
        uint8_t *dst = ring + head;
        head += size;
        d = (int)(seq % PK_NDESC);
        need[d] = skip + size;
        used += skip + size;
        pk_tile_off[d] = (int)(dst - ring);
        return dst;
    };
    const bool pos_ok = pos >= 0 && pos < P.attn.max_seq;
    for (int ph = 0; ph < P.n_phases && !pk_abort; ph++) {
        const PPhase &F = P.phases[ph];
        pwait = 0;
        if (F.kind == PH_ATTN) {
            // the K and V pages of the KV head of each of this CTA's query heads, in page order
            constexpr uint32_t PAGE = ATTN_P * HD * 2;
            const int G = P.attn.n_heads / P.attn.n_kv;
            for (int h = blockIdx.x; pos_ok && h < P.attn.n_heads && !pk_abort; h += gridDim.x) {
                const int g = h / G;
                for (int pg = 0; pg < nch; pg++) {
                    int d;
                    uint8_t *dst = reserve(2 * PAGE, d);
                    if (!dst) break;
                    const size_t base =
                        (((size_t)P.attn.page_table[pg] * P.attn.n_layers + F.layer) * P.attn.n_kv + g) * (size_t)ATTN_P * HD;
                    mbar_expect_tx(&pk_full[d], 2 * PAGE);
                    bulk_g2s(dst, P.attn.k_pool + base, PAGE, &pk_full[d]);
                    bulk_g2s(dst + PAGE, P.attn.v_pool + base, PAGE, &pk_full[d]);
                    seq++;
                }
            }
        } else {
            for (int tile = blockIdx.x; tile < F.n_tiles && !pk_abort; tile += gridDim.x) {
                int s, lt;
                locate_p(F, tile, s, lt);
                const PSeg &S = F.seg[s];
                int d;
                uint8_t *dst = reserve(tile_bytes_of(S, F.nmat), d);
                if (!dst) break;
                // issue: plain-copied tail first, then the arrive (release), then the bulk copies
                const int r0 = lt * TC_M, nrows = min(TC_M, S.rows - r0);
                const uint32_t mat_bytes = (uint32_t)nrows * S.row_bytes;
                const uint32_t main_bytes = S.per_row ? mat_bytes : (mat_bytes & ~15u);
                for (int m = 0; m < F.nmat; m++) {
                    const uint8_t *src = (m == 0 ? S.w : S.w2) + (size_t)r0 * S.row_bytes;
                    uint8_t *mdst = dst + (size_t)m * TC_M * S.stride;
                    for (uint32_t k = main_bytes; k < mat_bytes; k++) mdst[k] = src[k];
                }
                mbar_expect_tx(&pk_full[d], main_bytes * F.nmat);
                for (int m = 0; m < F.nmat; m++) {
                    const uint8_t *src = (m == 0 ? S.w : S.w2) + (size_t)r0 * S.row_bytes;
                    uint8_t *mdst = dst + (size_t)m * TC_M * S.stride;
                    if (S.per_row) {
                        for (int r = 0; r < nrows; r++)
                            bulk_g2s(mdst + (size_t)r * S.stride, src + (size_t)r * S.row_bytes, S.row_bytes, &pk_full[d]);
                    } else if (main_bytes) {
                        bulk_g2s(mdst, src, main_bytes, &pk_full[d]);
                    }
                }
                seq++;
            }
        }
        if (P.trace) {
            unsigned long long *tr = P.trace + ((size_t)ph * gridDim.x + blockIdx.x) * PK_TRACE_FIELDS;
            tr[6] = gtimer();
            tr[7] = (unsigned long long)pwait;
        }
    }
    // copies still in flight land before the CTA can exit: the consumers wait
    // on every tile; after an abort, wait (bounded) here for the issued ones.
    if (pk_abort)
        for (long long k = oldest; k < seq; k++) mbar_wait(&pk_full[k % PK_NDESC], (uint32_t)((k / PK_NDESC) & 1));
}

// ---- the kernel ----------------------------------------------------------------------

template <int HD, int G>
__global__ void __launch_bounds__(PK_THREADS, 1) decode_persistent_kernel(const __grid_constant__ PParams P) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int d = 0; d < PK_NDESC; d++) {
            mbar_init(&pk_full[d], 1);
            mbar_init(&pk_empty[d], PK_WARPS);  // one arrival per consumer warp
        }
        mbar_fence_init();
        pk_abort = 0;
        pk_stop = 0;
    }
    if (warp == 0) pk_fetch_phase(&pk_F[0], P.phases, lane);
    cp_async_wait_all();
    __syncthreads();  // the only full-CTA barrier

    // attention pages of this step (pos is final for the whole launch)
    const int pos = *P.attn.pos_ptr;
    const int nch = (pos >= 0 && pos < P.attn.max_seq) ? pos / ATTN_P + 1 : 0;

    if (warp == PK_WARPS) {
        if (lane == 0) pk_producer<HD>(P, pos, nch);
        return;
    }

    // ------------------------------------------------------------------ consumers
    const int token0 = *P.io_token;
    int seq = 0;
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    PkTrace T{nullptr, clock64()};
    long long wfull = 0;
    float *nws = pk_nws(P);

    for (int ph = 0; ph < P.n_phases; ph++) {
        const PPhase &F = pk_F[ph & 1];  // fetched during the previous phase
        wfull = 0;
        // the next phase's descriptor, into the other buffer (last read in phase
        // ph - 1; complete at this phase's arrive barrier)
        if (warp == 0 && ph + 1 < P.n_phases) pk_fetch_phase(&pk_F[(ph + 1) & 1], P.phases + ph + 1, lane);
        T.tr = (P.trace && tid == 0) ? P.trace + ((size_t)ph * gridDim.x + blockIdx.x) * PK_TRACE_FIELDS : nullptr;
        const bool gemv = F.kind != PH_ATTN && (int)blockIdx.x < F.n_tiles;
        // inputs that do not depend on the previous phase, fetched before its barrier:
        // the embedding phase's RMSNorm weights; the residual rows (final since two
        // barriers ago) and the next phase's norm weights for this CTA's first tiles
        if (gemv && F.embed_in && F.norm_w)
            for (int i = tid; i < (F.cols >> 2); i += PK_CONSUMERS) cp_async16(nws + 4 * i, F.norm_w + 4 * i);
        if (gemv && F.kind == PH_RESID) {
            const int my_tiles = (F.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
            const int cnt = min(my_tiles, PK_RPRE);
            for (int i = tid; i < cnt * 4; i += PK_CONSUMERS) {
                const int r0 = ((int)blockIdx.x + (i >> 2) * (int)gridDim.x) * TC_M + 4 * (i & 3);
                if (r0 + 4 <= F.seg[0].rows) {
                    cp_async16(pk_rpre + 4 * i, F.resid + r0);
                    if (F.nw_out) cp_async16(pk_nwpre + 4 * i, F.nw_out + r0);
                }
            }
        }
        if (!gemv && F.kind != PH_ATTN && F.ss_out && tid == 0) F.ss_out[blockIdx.x] = 0.f;  // no rows here
        bool ok = true;
        if (gemv) {
            ok = pk_gemv_phase<HD, G>(P, F, ph, token0, seq, wfull, best_v, best_i, T);  // waits for phase ph - 1 itself
        } else {
            if (!pk_grid_wait(P, ph)) break;
            T.put(0, gtimer());
            T.mark(1);
            if (F.kind == PH_ATTN) ok = pk_attn_phase<HD, G>(P, F, pos, nch, seq, wfull, T.tr);
        }
        if (!ok) break;
        T.mark(3);
        T.put(4, (unsigned long long)wfull);

        if (F.kind == PH_LM) {
            pk_argmax_finish(P, best_v, best_i);
        } else {
            // arrive: this CTA's outputs of the phase are written; the next
            // descriptor has landed
            cp_async_wait_all();
            cbar();
            if (tid == 0)  // release: the CTA's writes (ordered before it by the barrier) first
                asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(P.bar + ph) : "memory");
        }
        T.mark(5);
    }
    cp_async_wait_all();
}

}  // namespace fiber
