// persistent.cuh — one decode step as one cooperative kernel.
//
// Why: a batch-1 step of the 1.1B model moves ~640 MB through ~110 dependent
// phases; launched as separate kernels, each phase pays launch, first-byte
// latency and an x-staging/epilogue chain (~5-10 us) for ~0.5-2 us of data.
// Here every SM runs one CTA for the whole step:
//   * warp 8 (producer, one lane) walks the CTA's weight tiles of ALL phases in
//     consumption order and streams them with cp.async.bulk into a shared-memory
//     byte ring (FIFO, an mbarrier full/empty pair per tile in flight), so weight
//     loading runs ahead across phase boundaries and barrier waits;
//   * warps 0..7 (consumers) wait for the phase's input (grid barrier), stage x
//     as fp16 hi/lo fragments (through the RMSNorm where the reference has one),
//     decode + multiply each tile on the tensor cores (TcDot) and run the
//     phase's epilogue; consumers synchronise among themselves with named
//     barrier 1, never with the producer;
//   * between phases a grid barrier: one arrive counter per phase in global
//     memory (zeroed before each launch), polled with bounded spins.
// Phases per token: per layer QKV (layer 0 stages the embedding row itself),
// attention (RoPE, KV append, split-K chunks merged by the last CTA of each KV
// head), Wo (+residual), gate/up (+RMSNorm, SwiGLU), down (+residual); then
// lm_head (+RMSNorm, greedy argmax).
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
constexpr long long PK_SPIN_LIMIT = 1ll << 22;  // grid-barrier polls (with ~100 ns sleeps)

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

struct PPhase {
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
    PSeg seg[3];
};

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
};

FDEV void cbar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
struct ConsumerBar {
    FDEV void operator()() const { cbar(); }
};
FDEV void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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

// Staging for the persistent kernel (256 consumer threads, named barrier).
template <int T>
FDEV float pk_stage(const PPhase &F, const float *xsrc, bool xsrc_smem, float rrms, float scale, uint2 *xf) {
    const int nb = F.cols >> 8;
    for (int f = threadIdx.x; f < nb * 64; f += PK_CONSUMERS) {
        const int b = f >> 6, s = (f >> 2) & 15, t = f & 3;
        __half hi[4], lo[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int k = b * 256 + TcType<T>::elem(t, s, i);
            float v = xsrc_smem ? xsrc[k] : __ldcg(xsrc + k);
            if (F.norm_w) v = __fmul_rn(__fmul_rn(v, rrms), __ldg(F.norm_w + k));
            v *= scale;
            hi[i] = __float2half_rn(v);
            lo[i] = __float2half_rn(v - __half2float(hi[i]));
        }
        xf[2 * f + 0] = make_uint2((uint32_t)__half_as_ushort(hi[0]) | ((uint32_t)__half_as_ushort(hi[1]) << 16),
                                   (uint32_t)__half_as_ushort(hi[2]) | ((uint32_t)__half_as_ushort(hi[3]) << 16));
        xf[2 * f + 1] = make_uint2((uint32_t)__half_as_ushort(lo[0]) | ((uint32_t)__half_as_ushort(lo[1]) << 16),
                                   (uint32_t)__half_as_ushort(lo[2]) | ((uint32_t)__half_as_ushort(lo[3]) << 16));
    }
    return 0.f;
}

// Bounded mbarrier wait that also gives up when another thread has aborted.
FDEV bool pk_mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    for (long long i = 0; i < TC_WAIT_LIMIT; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 255 && *abort_flag) return false;
    }
    return false;
}

template <int HD, int G>
__global__ void __launch_bounds__(PK_THREADS, 1) decode_persistent_kernel(const PParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[PK_NDESC], empty[PK_NDESC];
    __shared__ float red[PK_WARPS * 2 * TC_M];
    __shared__ float2 cand[PK_WARPS];
    __shared__ float stat[2 * PK_WARPS];
    __shared__ unsigned int ticket;
    __shared__ volatile int abort_flag;  // set by any thread that gives up (producer included)
    __shared__ int stop;                 // consumers' uniform copy: written by thread 0 before a barrier
    __shared__ int tile_off[PK_NDESC];  // ring offset of each tile in flight (producer -> consumers)

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint8_t *ring = smem;
    uint2 *xf0 = reinterpret_cast<uint2 *>(smem + P.ring_bytes);
    float *xs = reinterpret_cast<float *>(smem + P.ring_bytes + P.xf_bytes);

    if (tid == 0) {
        for (int d = 0; d < PK_NDESC; d++) {
            mbar_init(&full[d], 1);
            mbar_init(&empty[d], 1);
        }
        mbar_fence_init();
        abort_flag = 0;
        stop = 0;
    }
    __syncthreads();  // the only full-CTA barrier

    // ------------------------------------------------------------------ producer
    if (warp == PK_WARPS) {
        if (lane != 0) return;
        int head = 0, used = 0, need[PK_NDESC];
        long long seq = 0, oldest = 0;
        for (int ph = 0; ph < P.n_phases && !abort_flag; ph++) {
            const PPhase &F = P.phases[ph];
            if (F.kind == PH_ATTN) continue;
            for (int tile = blockIdx.x; tile < F.n_tiles && !abort_flag; tile += gridDim.x) {
                int s, lt;
                locate_p(F, tile, s, lt);
                const PSeg &S = F.seg[s];
                const int size = tile_bytes_of(S, F.nmat);
                // wait for ring space: a slot, and `size` contiguous bytes (skipping
                // the ring's end when the tile would straddle it)
                int skip;
                for (;;) {
                    if (seq == oldest) head = 0;  // ring empty: restart at the front
                    skip = head + size > P.ring_bytes ? P.ring_bytes - head : 0;
                    if (seq - oldest < PK_NDESC && used + skip + size <= P.ring_bytes) break;
                    const int od = (int)(oldest % PK_NDESC);
                    if (!pk_mbar_wait(&empty[od], (uint32_t)((oldest / PK_NDESC) & 1), &abort_flag)) {
                        abort_flag = 1;
                        *P.io_err = 4;
                        break;
                    }
                    used -= need[od];
                    oldest++;
                }
                if (abort_flag) break;
                if (skip) head = 0;
                uint8_t *dst = ring + head;
                head += size;
                const int d = (int)(seq % PK_NDESC);
                need[d] = skip + size;
                used += skip + size;
                tile_off[d] = (int)(dst - ring);
                // issue: plain-copied tail first, then the arrive (release), then the bulk copies
                const int r0 = lt * TC_M, nrows = min(TC_M, S.rows - r0);
                const uint32_t mat_bytes = (uint32_t)nrows * S.row_bytes;
                const uint32_t main_bytes = S.per_row ? mat_bytes : (mat_bytes & ~15u);
                for (int m = 0; m < F.nmat; m++) {
                    const uint8_t *src = (m == 0 ? S.w : S.w2) + (size_t)r0 * S.row_bytes;
                    uint8_t *mdst = dst + (size_t)m * TC_M * S.stride;
                    for (uint32_t k = main_bytes; k < mat_bytes; k++) mdst[k] = src[k];
                }
                mbar_expect_tx(&full[d], main_bytes * F.nmat);
                for (int m = 0; m < F.nmat; m++) {
                    const uint8_t *src = (m == 0 ? S.w : S.w2) + (size_t)r0 * S.row_bytes;
                    uint8_t *mdst = dst + (size_t)m * TC_M * S.stride;
                    if (S.per_row) {
                        for (int r = 0; r < nrows; r++)
                            bulk_g2s(mdst + (size_t)r * S.stride, src + (size_t)r * S.row_bytes, S.row_bytes, &full[d]);
                    } else if (main_bytes) {
                        bulk_g2s(mdst, src, main_bytes, &full[d]);
                    }
                }
                seq++;
            }
        }
        // copies still in flight land before the CTA can exit: the consumers wait
        // on every tile; after an abort, wait (bounded) here for the issued ones.
        if (abort_flag)
            for (long long k = oldest; k < seq; k++)
                mbar_wait(&full[k % PK_NDESC], (uint32_t)((k / PK_NDESC) & 1));
        return;
    }

    // ------------------------------------------------------------------ consumers
    const int g = lane >> 2, t = lane & 3;
    long long seq = 0;
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    const int token0 = *P.io_token;

    for (int ph = 0; ph < P.n_phases; ph++) {
        const PPhase &F = P.phases[ph];
        // wait until every CTA finished the previous phase (thread 0 polls; the
        // stop decision is published before the barrier so all consumers agree)
        if (ph > 0) {
            if (tid == 0) {
                bool ok = false;
                const unsigned int *cnt = P.bar + (ph - 1);
                for (long long i = 0; i < PK_SPIN_LIMIT; i++) {
                    if (ld_acquire_u32(cnt) >= gridDim.x) {
                        ok = true;
                        break;
                    }
                    if ((i & 63) == 63 && abort_flag) break;
                    __nanosleep(64);
                }
                if (ok) {
                    __threadfence();  // order this CTA's reads of the phase inputs after the barrier
                } else {
                    abort_flag = 1;
                    *P.io_err = 4;
                }
                stop = abort_flag;
            }
            cbar();
            if (stop) break;
        }

        if (F.kind == PH_ATTN) {
            const int pos = *P.attn.pos_ptr;
            if (pos < 0 || pos >= P.attn.max_seq) {
                if (tid == 0 && blockIdx.x == 0) *P.io_err = 1;
            } else {
                AttnParams a = P.attn;
                a.layer = F.layer;
                const int nch = (pos + ATTN_P) / ATTN_P, units = nch * a.n_kv;
                for (int u = blockIdx.x; u < units; u += gridDim.x)
                    attn_unit<HD, G>(a, u / a.n_kv, u % a.n_kv, pos, reinterpret_cast<uint8_t *>(xf0), &ticket,
                                     ConsumerBar());
            }
        } else if ((int)blockIdx.x < F.n_tiles) {
            // ---- stage the input vector
            const int n = F.cols, nb = n >> 8;
            const float *xin = F.x;
            bool in_smem = false;
            if (F.embed_in) {
                // embedding row of the current token, computed by every CTA into xs
                int tok = token0;
                if (tok < 0 || tok >= P.vocab) {
                    if (tid == 0 && blockIdx.x == 0) *P.io_err = 2;
                    tok = 0;
                }
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
                }
                cbar();
                xin = xs;
                in_smem = true;
            } else if (P.xs_floats >= n) {
                for (int i = tid * 4; i < n; i += PK_CONSUMERS * 4)
                    *reinterpret_cast<float4 *>(xs + i) = __ldcg(reinterpret_cast<const float4 *>(F.x + i));
                cbar();
                xin = xs;
                in_smem = true;
            }
            // sum of squares and max |x| (scale choice), one reduction
            float ss = 0.f, mx = 0.f;
            for (int i = tid; i < n; i += PK_CONSUMERS) {
                const float v = in_smem ? xin[i] : __ldcg(xin + i);
                ss = fmaf(v, v, ss);
                mx = fmaxf(mx, fabsf(F.norm_w ? v * __ldg(F.norm_w + i) : v));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                ss += __shfl_xor_sync(0xffffffffu, ss, o);
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            }
            if (lane == 0) {
                stat[2 * warp] = ss;
                stat[2 * warp + 1] = mx;
            }
            cbar();
            ss = 0.f;
            mx = 0.f;
            for (int w = 0; w < PK_WARPS; w++) {
                ss += stat[2 * w];
                mx = fmaxf(mx, stat[2 * w + 1]);
            }
            const float rrms = F.norm_w ? 1.0f / sqrtf(ss / (float)n + F.eps) : 1.0f;
            mx *= rrms;
            int e = 0;
            if (mx > 0.f) frexpf(mx, &e);
            const int sh = (mx > 0.f && isfinite(mx)) ? (14 - e) : 0;
            const float scale = ldexpf(1.0f, sh), unscale = ldexpf(1.0f, -sh);
            // fragments for each weight type of the phase (at most two: QKV may mix Q4_K and Q6_K)
            const int type_a = F.seg[0].type;
            int type_b = -1;
            for (int k = 1; k < F.nseg; k++)
                if (F.seg[k].type != type_a) type_b = F.seg[k].type;
            auto stage = [&](int ty, uint2 *dst) {
                switch (ty) {
                case T_Q4_K: pk_stage<T_Q4_K>(F, xin, in_smem, rrms, scale, dst); break;
                case T_Q6_K: pk_stage<T_Q6_K>(F, xin, in_smem, rrms, scale, dst); break;
                default: pk_stage<T_F16>(F, xin, in_smem, rrms, scale, dst); break;
                }
            };
            uint2 *xf1 = xf0 + (size_t)nb * 128;  // second type's fragments follow the first's
            stage(type_a, xf0);
            if (type_b >= 0) stage(type_b, xf1);
            cbar();

            // ---- tiles of this CTA
            for (int tile = blockIdx.x; tile < F.n_tiles; tile += gridDim.x) {
                int sidx, lt;
                locate_p(F, tile, sidx, lt);
                const PSeg &S = F.seg[sidx];
                const int d = (int)(seq % PK_NDESC);
                if (tid == 0) {
                    if (!pk_mbar_wait(&full[d], (uint32_t)((seq / PK_NDESC) & 1), &abort_flag)) {
                        abort_flag = 1;
                        *P.io_err = 4;
                    }
                    stop = abort_flag;
                }
                cbar();  // tile landed (thread 0 observed the mbarrier) and `stop` is published
                if (stop) break;
                const uint8_t *buf = ring + tile_off[d];
                const uint2 *xf = (S.type == type_a) ? xf0 : xf1;
                const int bb = S.type == T_Q4_K ? 144 : (S.type == T_Q6_K ? 210 : 512);
                float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
                for (int b = warp; b < nb; b += PK_WARPS) {
                    const uint2 *xfb = xf + (size_t)b * 128;
                    for (int m = 0; m < F.nmat; m++) {
                        const uint8_t *mb = buf + (size_t)m * TC_M * S.stride + (size_t)b * bb;
                        const uint8_t *rg = mb + (size_t)g * S.stride, *rg8 = mb + (size_t)(g + 8) * S.stride;
                        switch (S.type) {
                        case T_Q4_K: TcDot<T_Q4_K>::run(rg, rg8, xfb, g, t, acc[m]); break;
                        case T_Q6_K: TcDot<T_Q6_K>::run(rg, rg8, xfb, g, t, acc[m]); break;
                        default: TcDot<T_F16>::run(rg, rg8, xfb, g, t, acc[m]); break;
                        }
                    }
                }
                if (t == 0) {
                    for (int m = 0; m < F.nmat; m++) {
                        red[(warp * 2 + m) * TC_M + g] = acc[m][0] + acc[m][1];
                        red[(warp * 2 + m) * TC_M + g + 8] = acc[m][2] + acc[m][3];
                    }
                }
                cbar();  // tile consumed, partials visible
                if (tid == 0) mbar_arrive(&empty[d]);
                if (tid < TC_M) {
                    const int r = lt * TC_M + tid;
                    float v[2] = {0.f, 0.f};
                    for (int m = 0; m < F.nmat; m++) {
                        float sum = 0.f;
#pragma unroll
                        for (int w = 0; w < PK_WARPS; w++) sum += red[(w * 2 + m) * TC_M + tid];
                        v[m] = sum * unscale;
                    }
                    if (r < S.rows) {
                        if (F.kind == PH_QKV) {
                            F.y[S.out_off + r] = v[0];
                        } else if (F.kind == PH_RESID) {
                            F.resid[r] = __fadd_rn(__ldcg(F.resid + r), v[0]);
                        } else if (F.kind == PH_SWIGLU) {
                            F.y[r] = __fmul_rn(__fdiv_rn(v[0], __fadd_rn(1.0f, expf(-v[0]))), v[1]);
                        } else {  // PH_LM
                            F.y[r] = v[0];
                            if (better(v[0], r, best_v, best_i)) {
                                best_v = v[0];
                                best_i = r;
                            }
                        }
                    }
                }
                cbar();  // red reused by the next tile
                seq++;
            }
            if (stop) break;
        }

        if (F.kind == PH_LM) {
            // greedy argmax: CTA candidate, then the last CTA reduces all of them
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
                    ticket = atomicAdd(P.am_count, 1u);
                }
            }
            cbar();
            if (ticket == gridDim.x - 1) {
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
                if (lane == 0) cand[warp] = make_float2(bv, __int_as_float(bi));
                cbar();
                if (tid == 0) {
                    for (int w = 1; w < PK_WARPS; w++) {
                        const int wi = __float_as_int(cand[w].y);
                        if (better(cand[w].x, wi, bv, bi)) {
                            bv = cand[w].x;
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
        } else {
            // arrive: this CTA's outputs of the phase are written
            cbar();
            if (tid == 0) {
                __threadfence();
                atomicAdd(P.bar + ph, 1u);
            }
        }
    }
}

}  // namespace fiber
