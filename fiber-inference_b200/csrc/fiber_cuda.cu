// fiber_cuda.cu — host side of libfiber_cuda.so: model upload, paged KV cache,
// decode-step enqueue, CUDA-graph capture and the extern "C" entry points of
// include/gpu_ffn.h, include/kv_cache.h and include/fiber_cuda.h.
//
// One decode step (src/gpu_ffn.m:488-617 of the reference) is 2 + 5 * n_layers
// kernels on the context's stream:
//   embed(token)                                   gpu_embed, on the device
//   per layer: RMSNorm+[Wq;Wk;Wv]                  rmsnorm + 3 matvecs
//              RoPE+KV append+GQA attention        rope_qk, kv_store_kv, attention_decode
//              Wo (+residual)                      matvec + residual_rmsnorm's add
//              RMSNorm+[W1,W3]+SwiGLU              rmsnorm + 2 matvecs + silu_gate
//              W2 (+residual)                      matvec + residual_add
//   RMSNorm+lm_head+argmax                         rmsnorm + matvec_f32 + sampler argmax
// The step reads token and position from device memory, so it is captured once
// into a CUDA graph and replayed for every token.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <math.h>
#include <nccl.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "attention.cuh"
#include "fiber_cuda.h"
#include "gemv.cuh"
#include "gemv_tc.cuh"
#include "launch.cuh"
#include "persistent.cuh"
#include "flow.cuh"
#include "gemm_tc5.cuh"
#include "prefill.cuh"
#include "sample.cuh"
#include "allreduce.cuh"

using namespace fiber;

// ---- errors --------------------------------------------------------------------

static thread_local char g_err[512] = "";

static int set_err(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

#define CK(call)                                                                                  \
    do {                                                                                          \
        cudaError_t e_ = (call);                                                                  \
        if (e_ != cudaSuccess)                                                                    \
            return set_err(FIBER_ECUDA, "%s:%d %s: %s", __FILE__, __LINE__, #call, cudaGetErrorString(e_)); \
    } while (0)

extern "C" const char *fiber_last_error(void) { return g_err; }

// lets the other translation units of this library report through fiber_last_error()
__attribute__((visibility("hidden"))) void fiber_set_error_message(const char *msg) {
    snprintf(g_err, sizeof(g_err), "%s", msg);
}

extern "C" int fiber_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

// ---- small helpers ----------------------------------------------------------------

static int block_bytes(int t) {
    switch (t) {
    case T_Q4_K: return 144;
    case T_Q5_K: return 176;
    case T_Q6_K: return 210;
    case T_F16: return 512;
    default: return 0;
    }
}

static const char *tname(int t) {
    switch (t) {
    case T_F32: return "F32";
    case T_F16: return "F16";
    case T_Q4_K: return "Q4_K";
    case T_Q5_K: return "Q5_K";
    case T_Q6_K: return "Q6_K";
    default: return "unsupported";
    }
}

static bool matrix_type_ok(int t) { return t == T_Q4_K || t == T_Q5_K || t == T_Q6_K || t == T_F16; }

constexpr int GEMV_ROWS = 2;
constexpr int GEMV_TILE = GEMV_ROWS * GEMV_WARPS;

template <int T, int EPI>
static cudaError_t launch_gemv_t(const GemvParams &p, int grid, cudaStream_t st) {
    const size_t smem = (size_t)p.cols * sizeof(float);
    auto k = gemv_kernel<T, EPI, GEMV_ROWS>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return launch_pdl(k, dim3(grid), dim3(GEMV_THREADS), smem, st, p);
}

static int sm_count() {
    static int cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

// v2 launch (gemv_tc.cuh): tiles of 16 rows; one tile per CTA while the grid fits
// about four CTAs per SM, else a persistent grid of 2 CTAs per SM with a ring of
// up to 4 tiles each.
template <int T, int EPI, int NMAT>
static cudaError_t launch_tc_t(TcParams p, cudaStream_t st) {
    const int sms = sm_count();
    const int nb = p.cols / 256;
    p.row_bytes = nb * TcType<T>::BB;
    p.per_row_copy = (p.row_bytes % 16) == 0;
    p.stride = p.per_row_copy ? p.row_bytes + (16 - p.row_bytes % 128 + 128) % 128 : p.row_bytes;
    p.n_tiles = 0;
    for (int s = 0; s < p.nseg; s++) {
        p.seg[s].tiles = (p.seg[s].rows + TC_M - 1) / TC_M;
        p.n_tiles += p.seg[s].tiles;
    }
    const size_t tile_bytes = (size_t)NMAT * TC_M * p.stride;
    size_t fixed = (size_t)nb * 1024;
    int grid;
    if (p.n_tiles <= 4 * sms) {
        grid = p.n_tiles;
        p.stages = 1;
    } else {
        grid = 2 * sms;
        const long long fit = ((long long)112 * 1024 - (long long)fixed) / (long long)tile_bytes;
        p.stages = (int)(fit < 1 ? 1 : (fit > 4 ? 4 : fit));
    }
    size_t smem = p.stages * tile_bytes + fixed;
    p.stage_x = smem + (size_t)p.cols * 4 <= 227 * 1024;  // fp32 copy of x while staging, if it fits
    if (p.stage_x) smem += (size_t)p.cols * 4;
    if (smem > 227 * 1024) return cudaErrorNotSupported;  // caller falls back to the v1 kernel
    auto k = gemv_tc_kernel<T, EPI, NMAT>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return launch_pdl(k, dim3(grid), dim3(TC_THREADS), smem, st, p);
}

static TcParams to_tc(const GemvParams &g) {
    TcParams p;
    memset(&p, 0, sizeof(p));
    p.nseg = g.nseg;
    for (int s = 0; s < g.nseg; s++) {
        p.seg[s].w = g.seg[s].w;
        p.seg[s].w2 = g.w_up;
        p.seg[s].rows = g.seg[s].rows;
        p.seg[s].out_off = g.seg[s].out_off;
    }
    p.cols = g.cols;
    p.x = g.x;
    p.norm_w = g.norm_w;
    p.eps = g.eps;
    p.y = g.y;
    p.resid = g.resid;
    p.am_part = g.am_part;
    p.am_count = g.am_count;
    p.am_out = g.am_out;
    p.adv_token = g.adv_token;
    p.adv_pos = g.adv_pos;
    p.rec_tokens = g.rec_tokens;
    p.rec_step = g.rec_step;
    return p;
}

template <int EPI>
static cudaError_t launch_gemv(int type, const GemvParams &p, int grid, cudaStream_t st) {
    constexpr int NM = EPI == EPI_SWIGLU ? 2 : 1;
    cudaError_t e = cudaErrorNotSupported;
    switch (type) {
    case T_Q4_K: e = launch_tc_t<T_Q4_K, EPI, NM>(to_tc(p), st); break;
    case T_Q6_K: e = launch_tc_t<T_Q6_K, EPI, NM>(to_tc(p), st); break;
    case T_F16: e = launch_tc_t<T_F16, EPI, NM>(to_tc(p), st); break;
    default: break;
    }
    if (e != cudaErrorNotSupported) return e;
    // Q5_K, or a tile that does not fit in shared memory: the v1 kernel
    switch (type) {
    case T_Q4_K: return launch_gemv_t<T_Q4_K, EPI>(p, grid, st);
    case T_Q5_K: return launch_gemv_t<T_Q5_K, EPI>(p, grid, st);
    case T_Q6_K: return launch_gemv_t<T_Q6_K, EPI>(p, grid, st);
    case T_F16: return launch_gemv_t<T_F16, EPI>(p, grid, st);
    default: return cudaErrorInvalidValue;
    }
}

// All segments of one launch must share a type (the kernel is specialised on
// it); a QKV projection with mixed types is split into per-type launches.
static GemvParams one_seg(const uint8_t *w, int type, int rows, int out_off, int cols) {
    GemvParams p;
    memset(&p, 0, sizeof(p));
    p.seg[0] = {w, type, rows, out_off};
    p.nseg = 1;
    p.tiles[0] = (rows + GEMV_TILE - 1) / GEMV_TILE;
    p.cols = cols;
    return p;
}

static int grid_of(const GemvParams &p) {
    int g = 0;
    for (int s = 0; s < p.nseg; s++) g += p.tiles[s];
    return g;
}

// ---- KV cache ------------------------------------------------------------------------

extern "C" void kv_cache_free(kv_cache_t *kv) {
    if (!kv) return;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(kv->device);
    cudaFree(kv->k_pool);
    cudaFree(kv->v_pool);
    cudaFree(kv->page_table);
    if (prev >= 0) cudaSetDevice(prev);
    free(kv);
}

extern "C" kv_cache_t *kv_cache_init_paged(int device, int n_layers, int n_kv_heads, int head_dim, int max_seq,
                                           int max_batch, int page_size) {
    if (n_layers <= 0 || n_kv_heads <= 0 || head_dim <= 0 || head_dim % 8 || max_seq <= 0 || max_batch <= 0 ||
        page_size != ATTN_P) {
        set_err(FIBER_EARG, "kv_cache_init: bad shape (layers=%d kv_heads=%d head_dim=%d max_seq=%d batch=%d page=%d; page must be %d)",
                n_layers, n_kv_heads, head_dim, max_seq, max_batch, page_size, ATTN_P);
        return nullptr;
    }
    if (cudaSetDevice(device) != cudaSuccess) {
        set_err(FIBER_ECUDA, "kv_cache_init: cannot select device %d", device);
        return nullptr;
    }
    kv_cache_t *kv = (kv_cache_t *)calloc(1, sizeof(kv_cache_t));
    kv->n_layers = n_layers;
    kv->n_kv_heads = n_kv_heads;
    kv->head_dim = head_dim;
    kv->max_seq = max_seq;
    kv->device = device;
    kv->max_batch = max_batch;
    kv->page_size = page_size;
    kv->max_pages_per_seq = (max_seq + page_size - 1) / page_size;
    kv->n_pages = kv->max_pages_per_seq * max_batch;
    const size_t elems = (size_t)kv->n_pages * n_layers * n_kv_heads * page_size * head_dim;
    std::vector<int32_t> pt((size_t)kv->n_pages);
    for (int i = 0; i < kv->n_pages; i++) pt[i] = i;
    if (cudaMalloc(&kv->k_pool, elems * 2) != cudaSuccess || cudaMalloc(&kv->v_pool, elems * 2) != cudaSuccess ||
        cudaMalloc(&kv->page_table, pt.size() * 4) != cudaSuccess ||
        cudaMemset(kv->k_pool, 0, elems * 2) != cudaSuccess || cudaMemset(kv->v_pool, 0, elems * 2) != cudaSuccess ||
        cudaMemcpy(kv->page_table, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
        set_err(FIBER_ENOMEM, "kv_cache_init: allocating %.1f MB failed", 4.0 * elems / 1e6);
        kv_cache_free(kv);
        return nullptr;
    }
    return kv;
}

extern "C" kv_cache_t *kv_cache_init(int device, int n_layers, int n_kv_heads, int head_dim, int max_seq) {
    kv_cache_t *kv = kv_cache_init_paged(device, n_layers, n_kv_heads, head_dim, max_seq, 1, ATTN_P);
    if (kv)
        printf("KV Cache: %d layers, %d KV-heads, head_dim=%d, max_seq=%d (%.1f MB, paged fp16)\n", n_layers,
               n_kv_heads, head_dim, max_seq,
               4.0 * kv->n_pages * n_layers * n_kv_heads * kv->page_size * head_dim / (1024.0 * 1024.0));
    return kv;
}

static size_t kv_offset(const kv_cache_t *kv, int page, int layer, int head, int in_page) {
    return ((((size_t)page * kv->n_layers + layer) * kv->n_kv_heads + head) * kv->page_size + in_page) * kv->head_dim;
}

static int kv_copy(kv_cache_t *kv, int slot, int layer, int pos, int n_pos, float *k, float *v, bool write) {
    if (!kv || slot < 0 || slot >= kv->max_batch || layer < 0 || layer >= kv->n_layers || pos < 0 || n_pos < 0 ||
        pos + n_pos > kv->max_seq)
        return set_err(FIBER_EARG, "kv_cache copy: out of range (slot %d layer %d pos %d n %d)", slot, layer, pos, n_pos);
    CK(cudaSetDevice(kv->device));
    std::vector<int32_t> pt((size_t)kv->max_pages_per_seq);
    CK(cudaMemcpy(pt.data(), kv->page_table + (size_t)slot * kv->max_pages_per_seq, pt.size() * 4,
                  cudaMemcpyDeviceToHost));
    const int hd = kv->head_dim, kvd = kv->n_kv_heads * hd;
    std::vector<uint16_t> hk((size_t)hd), hv((size_t)hd);
    for (int t = 0; t < n_pos; t++) {
        const int p = pos + t, page = pt[p / kv->page_size], ip = p % kv->page_size;
        for (int h = 0; h < kv->n_kv_heads; h++) {
            const size_t off = kv_offset(kv, page, layer, h, ip);
            if (write) {
                for (int d = 0; d < hd; d++) {
                    hk[d] = __half_as_ushort(__float2half_rn(k[(size_t)t * kvd + h * hd + d]));
                    hv[d] = __half_as_ushort(__float2half_rn(v[(size_t)t * kvd + h * hd + d]));
                }
                CK(cudaMemcpy(kv->k_pool + off, hk.data(), (size_t)hd * 2, cudaMemcpyHostToDevice));
                CK(cudaMemcpy(kv->v_pool + off, hv.data(), (size_t)hd * 2, cudaMemcpyHostToDevice));
            } else {
                CK(cudaMemcpy(hk.data(), kv->k_pool + off, (size_t)hd * 2, cudaMemcpyDeviceToHost));
                CK(cudaMemcpy(hv.data(), kv->v_pool + off, (size_t)hd * 2, cudaMemcpyDeviceToHost));
                for (int d = 0; d < hd; d++) {
                    k[(size_t)t * kvd + h * hd + d] = __half2float(__ushort_as_half(hk[d]));
                    v[(size_t)t * kvd + h * hd + d] = __half2float(__ushort_as_half(hv[d]));
                }
            }
        }
    }
    return FIBER_OK;
}

extern "C" int kv_cache_write(kv_cache_t *kv, int slot, int layer, int pos, int n_pos, const float *k, const float *v) {
    return kv_copy(kv, slot, layer, pos, n_pos, const_cast<float *>(k), const_cast<float *>(v), true);
}

extern "C" int kv_cache_read(const kv_cache_t *kv, int slot, int layer, int pos, int n_pos, float *k, float *v) {
    return kv_copy(const_cast<kv_cache_t *>(kv), slot, layer, pos, n_pos, k, v, false);
}

// ---- context ---------------------------------------------------------------------------

struct LayerDev {
    const uint8_t *wq, *wk, *wv, *wo, *w1, *w2, *w3;
    const float *attn_norm, *ffn_norm;
    int tq, tk, tv, to, t1, t2, t3;
};

struct StepIO {  // device-side step state, one 32-byte block so it moves in one copy
    int32_t token, pos, argmax, err, step, pad[3];
};

struct Graph {
    cudaGraphExec_t exec = nullptr;
    const kv_cache_t *kv = nullptr;
};

struct gpu_context {
    int device = 0;
    cudaStream_t stream = nullptr;
    model_params_t p{};
    int max_seq = 0, max_chunks = 0, kvd = 0, G = 0;
    uint8_t *d_data = nullptr;
    size_t data_bytes = 0;
    std::vector<LayerDev> L;
    const uint8_t *embd = nullptr, *out = nullptr;
    const float *out_norm = nullptr;
    int t_embd = 0, t_out = 0;
    float *x = nullptr, *qkv = nullptr, *att = nullptr, *h = nullptr, *logits = nullptr;
    float2 *rope = nullptr;
    StepIO *io = nullptr;            // device
    int32_t *rec = nullptr;          // device [max_seq]: tokens of the greedy loop
    float *att_part = nullptr;       // attention split-K partials (scratch)
    unsigned int *att_cnt = nullptr; // attention merge tickets (scratch)
    float2 *am_part = nullptr;       // lm_head argmax partials (scratch)
    unsigned int *am_cnt = nullptr;  // lm_head merge ticket (scratch)
    StepIO *h_io = nullptr;          // pinned
    float *h_logits = nullptr;       // pinned
    std::vector<float> logits_copy;
    Graph g_step, g_loop;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    // persistent one-kernel step (persistent.cuh)
    int mode = 0;                  // 0: persistent kernel, 1: one kernel per phase, 2: dataflow kernel
                                   // (the default where the model fits it)
    bool pk_ok = false;            // the model fits the persistent kernel
    PPhase *d_phases = nullptr;
    std::vector<PPhase> phases;
    unsigned int *d_bar = nullptr;
    uint16_t *pk_gf[4] = {};       // phase-input fragments: QKV/lm_head, Wo, gate/up, down
    float *pk_ss[2] = {};          // per-CTA sums of squares: before gate/up, before QKV/lm_head
    int pk_ring = 0, pk_xfr = 0, pk_xs = 0, pk_nw = 0, pk_grid = 0;
    size_t pk_smem = 0;
    void *pk_kernel = nullptr;
    // dataflow one-kernel step (flow.cuh)
    bool fl_ok = false;               // the model fits the dataflow kernel
    uint64_t *fl_tp_local = nullptr;  // tensor parallel: this rank's exchange buffer of partial sums
    void *fl_tp_peer[FL_MAX_TP] = {}; // the other ranks' exchange buffers, mapped here (CUDA IPC)
    long long fl_tp_key_off = 0;      // word offset of the [world][2] argmax keys in the exchange buffers
    bool fl_lm_shard = false;         // this call wants no logits: ranks split the lm_head (greedy)
    FPhase *d_fphases = nullptr;
    std::vector<FPhase> fphases;
    uint64_t *fl_words = nullptr;     // tagged words of every phase output of one step
    unsigned int *fl_sync = nullptr;  // [0] launch tag, [1] exit count, [2] argmax ticket, [4..) attention tickets
    uint64_t *fl_att_words = nullptr; // tagged attention split states
    unsigned long long *fl_am = nullptr;  // per-CTA argmax keys
    int fl_ring = 0, fl_frag = 0, fl_xres = 0, fl_xin = 0, fl_nw = 0, fl_grid = 0, fl_max_split = 0;
    size_t fl_smem = 0;
    void *fl_kernel = nullptr;
    const void *fl_map_k = nullptr, *fl_map_v = nullptr;  // pools (and their row count) the maps describe
    long long fl_map_rows = 0;
    CUtensorMap fl_kmap, fl_vmap;
    // tensor parallelism: this rank's share of query heads, KV heads and FFN blocks
    // (the whole model when tp_world == 1)
    int tp_rank = 0, tp_world = 1;
    int nh_l = 0, nkv_l = 0, ffn_l = 0, h0 = 0, g0 = 0, f0b = 0;
    float *x2 = nullptr;            // second residual buffer: Wo's all-reduced output
    uint8_t *d_shard = nullptr;     // Wo / W_down shards along their input dimension
    ncclComm_t comm = nullptr;
    // one-shot peer all-reduce (allreduce.cuh): own slot/flag area, peers' areas (CUDA IPC)
    bool ar_ok = false;
    void *ar_local = nullptr;
    void *ar_peer[AR_MAX_WORLD] = {};
    unsigned int *ar_epoch = nullptr;
    ArParams ar{};
    // batched prefill (tensor-core GEMMs): buffers for a chunk of pf_cap tokens
    int prefill_mode = 0;           // 0: batched when the model allows it, 1: token by token
    int pf_cap = 0;
    float *pf_x = nullptr, *pf_qkv = nullptr, *pf_att = nullptr, *pf_hg = nullptr, *pf_hu = nullptr;
    float *pf_x2 = nullptr;            // tensor parallel: residual stream after Wo's all-reduce
    uint8_t *pf_bp = nullptr;          // GEMM input packed as the MMA's B operand (hi / lo fp16)
    std::vector<CUtensorMap> pf_maps;  // per layer: tensor maps of wq wk wv wo w1 w2 w3
    std::vector<const uint8_t *> pf_w; // per layer: the GEMMs' weights (wq .. w3; padded Q6_K copies)
    const uint8_t *pf_out = nullptr;   // the classifier as the GEMM reads it
    int32_t *pf_tok = nullptr;
    // batched decode: max_batch sequences per step, sequence t in KV slot t
    int max_batch = 1;
    CUtensorMap out_map;               // tensor map of the classifier (lm_head GEMM)
    int32_t *bt_pos = nullptr, *bt_arg = nullptr, *bt_rec = nullptr;  // [max_batch], [max_batch], [max_seq][max_batch]
    int *bt_step = nullptr;
    float *bt_logits = nullptr;        // [max_batch][vocab]
    Graph g_batch;                     // captured greedy batch step (g_batch_n sequences)
    int g_batch_n = 0;
    float *att_ws = nullptr;           // page-split attention states (batched layer pass)
    unsigned int *att_tickets = nullptr;
    std::vector<void *> pf_pad;        // Q6_K matrices re-laid with 16-byte-aligned rows
    unsigned long long *smp_rng = nullptr;  // device sampler state (sampling decode loop)
    int32_t *smp_out = nullptr;
};

static void free_graph(Graph &g) {
    if (g.exec) cudaGraphExecDestroy(g.exec);
    g.exec = nullptr;
    g.kv = nullptr;
}

extern "C" void fiber_cuda_free(fiber_ctx_t *c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    free_graph(c->g_step);
    free_graph(c->g_loop);
    free_graph(c->g_batch);
    for (void *q : c->ar_peer)
        if (q) cudaIpcCloseMemHandle(q);
    for (void *q : c->fl_tp_peer)
        if (q) cudaIpcCloseMemHandle(q);
    if (c->fl_tp_local) cudaFree(c->fl_tp_local);
    if (c->ar_local) cudaFree(c->ar_local);
    if (c->ar_epoch) cudaFree(c->ar_epoch);
    if (c->comm) ncclCommDestroy(c->comm);
    for (void *q : c->pf_pad) cudaFree(q);
    void *dev[] = {c->pf_x2, c->smp_rng, c->smp_out, c->att_ws, c->att_tickets, c->bt_pos, c->bt_arg, c->bt_rec, c->bt_step, c->bt_logits, c->pf_x, c->pf_qkv, c->pf_att, c->pf_hg, c->pf_hu, c->pf_bp, c->pf_tok, c->x2, c->d_shard, c->d_data, c->x, c->qkv, c->att, c->h, c->logits, c->rope, c->io, c->rec,
                   c->att_part, c->att_cnt, c->am_part, c->am_cnt, c->d_phases, c->d_bar,
                   c->d_fphases, c->fl_words, c->fl_sync, c->fl_att_words, c->fl_am,
                   c->pk_gf[0], c->pk_gf[1], c->pk_gf[2], c->pk_gf[3], c->pk_ss[0], c->pk_ss[1]};
    for (void *p : dev)
        if (p) cudaFree(p);
    if (c->h_io) cudaFreeHost(c->h_io);
    if (c->h_logits) cudaFreeHost(c->h_logits);
    if (c->ev0) cudaEventDestroy(c->ev0);
    if (c->ev1) cudaEventDestroy(c->ev1);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

static bool tc_type_ok(int t) { return t == T_Q4_K || t == T_Q6_K || t == T_F16; }
// the dataflow step also takes Q5_K (fp32 weights as hi + lo fp16 MMA fragments)
static bool fl_type_ok(int t) { return tc_type_ok(t) || t == T_Q5_K; }

static PSeg make_pseg(const uint8_t *w, const uint8_t *w2, int type, int rows, int out_off, int cols) {
    PSeg sg;
    memset(&sg, 0, sizeof(sg));
    sg.w = w;
    sg.w2 = w2;
    sg.type = type;
    sg.rows = rows;
    sg.out_off = out_off;
    sg.tiles = (rows + TC_M - 1) / TC_M;
    sg.row_bytes = cols / 256 * block_bytes(type);
    sg.per_row = sg.row_bytes % 16 == 0;
    sg.stride = sg.per_row ? sg.row_bytes + (16 - sg.row_bytes % 128 + 128) % 128 : sg.row_bytes;
    return sg;
}

template <int HD, int G>
static void *pk_kernel_ptr() {
    return reinterpret_cast<void *>(decode_persistent_kernel<HD, G>);
}

// Phase table and launch geometry of the persistent step kernel; leaves
// pk_ok false (per-phase kernels only) when the model does not fit it.
static int pk_build(gpu_context *c) {
    const model_params_t &p = c->p;
    const int dim = p.dim, ffn = p.ffn_dim, kvd = c->kvd, hd = p.head_dim;
    c->pk_ok = false;
    bool types_ok = tc_type_ok(c->t_out);
    for (const LayerDev &d : c->L) {
        const int ts[7] = {d.tq, d.tk, d.tv, d.to, d.t1, d.t2, d.t3};
        for (int t : ts) types_ok = types_ok && tc_type_ok(t);
        int distinct = 1 + (d.tk != d.tq) + (d.tv != d.tq && d.tv != d.tk);
        types_ok = types_ok && distinct <= 2;
    }
#define PK_CASE(H, GG) \
    if (hd == H && c->G == GG) c->pk_kernel = pk_kernel_ptr<H, GG>();
    PK_CASE(64, 1) PK_CASE(64, 2) PK_CASE(64, 4) PK_CASE(64, 8)
    PK_CASE(128, 1) PK_CASE(128, 2) PK_CASE(128, 4) PK_CASE(128, 8)
#undef PK_CASE
    if (!types_ok || !c->pk_kernel) return FIBER_OK;

    std::vector<PPhase> &ph = c->phases;
    ph.clear();
    auto base = [&](int kind, int cols, int layer) {
        PPhase f;
        memset(&f, 0, sizeof(f));
        f.kind = kind;
        f.cols = cols;
        f.layer = layer;
        f.nmat = 1;
        f.eps = p.rms_norm_eps;
        return f;
    };
    for (uint32_t l = 0; l < p.n_layers; l++) {
        const LayerDev &d = c->L[l];
        PPhase q = base(PH_QKV, dim, l);
        q.nseg = 3;
        q.seg[0] = make_pseg(d.wq, nullptr, d.tq, dim, 0, dim);
        q.seg[1] = make_pseg(d.wk, nullptr, d.tk, kvd, dim, dim);
        q.seg[2] = make_pseg(d.wv, nullptr, d.tv, kvd, dim + kvd, dim);
        q.x = c->x;
        q.norm_w = d.attn_norm;
        q.y = c->qkv;
        q.embed_in = l == 0;
        ph.push_back(q);
        ph.push_back(base(PH_ATTN, dim, l));
        PPhase o = base(PH_RESID, dim, l);
        o.nseg = 1;
        o.seg[0] = make_pseg(d.wo, nullptr, d.to, dim, 0, dim);
        o.x = c->att;
        o.resid = c->x;
        ph.push_back(o);
        PPhase u = base(PH_SWIGLU, dim, l);
        u.nseg = 1;
        u.nmat = 2;
        u.seg[0] = make_pseg(d.w1, d.w3, d.t1, ffn, 0, dim);
        u.x = c->x;
        u.norm_w = d.ffn_norm;
        u.y = c->h;
        ph.push_back(u);
        PPhase dn = base(PH_RESID, ffn, l);
        dn.nseg = 1;
        dn.seg[0] = make_pseg(d.w2, nullptr, d.t2, dim, 0, ffn);
        dn.x = c->h;
        dn.resid = c->x;
        ph.push_back(dn);
    }
    PPhase lm = base(PH_LM, dim, 0);
    lm.nseg = 1;
    lm.seg[0] = make_pseg(c->out, nullptr, c->t_out, p.vocab_size, 0, dim);
    lm.x = c->x;
    lm.norm_w = c->out_norm;
    lm.y = c->logits;
    ph.push_back(lm);
    int sms = 0;
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c->device));
    const int grid = std::min(sms, (int)((p.vocab_size + TC_M - 1) / TC_M));
    if (grid > 256) return FIBER_OK;  // per-CTA partial sums are staged in 256 slots

    // phase-input hand-off: each phase's epilogue writes the next phase's input
    // as fragments (one layout per weight type of the next phase) and, before a
    // normed phase, per-CTA sums of squares
    const size_t gf_bytes[4] = {2 * (size_t)dim * 4, 2 * (size_t)dim * 4, 2 * (size_t)dim * 4, 2 * (size_t)ffn * 4};
    for (int k = 0; k < 4; k++) CK(cudaMalloc(&c->pk_gf[k], gf_bytes[k]));
    for (int k = 0; k < 2; k++) {
        CK(cudaMalloc(&c->pk_ss[k], 256 * sizeof(float)));
        CK(cudaMemset(c->pk_ss[k], 0, 256 * sizeof(float)));
    }
    auto layouts = [](const PPhase &f, int &a, int &b) {
        a = f.seg[0].type;
        b = -1;
        for (int k = 1; k < f.nseg; k++)
            if (f.seg[k].type != a && b < 0) b = f.seg[k].type;
    };
    for (size_t i = 0; i + 1 < ph.size(); i++) {
        PPhase &f = ph[i], &nx = ph[i + 1];
        if (f.kind == PH_QKV) continue;  // q/k/v go to the attention phase
        layouts(nx, f.out_types[0], f.out_types[1]);
        f.n_out = nx.cols;
        if (f.kind == PH_ATTN) {
            f.gf_out = c->pk_gf[1];
        } else if (f.kind == PH_SWIGLU) {
            f.gf_out = c->pk_gf[3];
        } else {  // Wo (next: gate/up) or down (next: QKV or lm_head), both residual
            const bool wo = nx.kind == PH_SWIGLU;
            f.gf_out = c->pk_gf[wo ? 2 : 0];
            f.nw_out = nx.norm_w;
            f.ss_out = nx.norm_w ? c->pk_ss[wo ? 0 : 1] : nullptr;
        }
        if (!nx.embed_in) {
            nx.gf_in = reinterpret_cast<const uint2 *>(f.gf_out);
            nx.ss_in = f.ss_out;
        }
    }
    size_t max_tile = (size_t)4 * ATTN_P * hd;  // attention: one K page and one V page (fp16)
    // the Wo staging merges attention partials through the fragment region:
    // [n_heads][units per KV head] weights and [n_heads] sums
    int xfr = (int)(((size_t)p.n_heads * (3 * std::max(1, grid / (int)p.n_kv_heads) + 1) * 4 + 1023) & ~(size_t)1023);
    for (PPhase &f : ph) {
        f.n_tiles = 0;
        for (int k = 0; k < f.nseg; k++) {
            f.n_tiles += f.seg[k].tiles;
            max_tile = std::max(max_tile, (size_t)f.nmat * TC_M * f.seg[k].stride);
        }
        int types = 1;
        for (int k = 1; k < f.nseg; k++)
            if (f.seg[k].type != f.seg[0].type) types = 2;
        if (f.kind != PH_ATTN) xfr = std::max(xfr, types * (f.cols / 256) * 1024);
    }
    const int attn_need = [&] {
        switch (hd * 16 + c->G) {
        case 64 * 16 + 1: return attn_smem_bytes<64, 1>();
        case 64 * 16 + 2: return attn_smem_bytes<64, 2>();
        case 64 * 16 + 4: return attn_smem_bytes<64, 4>();
        case 64 * 16 + 8: return attn_smem_bytes<64, 8>();
        case 128 * 16 + 1: return attn_smem_bytes<128, 1>();
        case 128 * 16 + 2: return attn_smem_bytes<128, 2>();
        case 128 * 16 + 4: return attn_smem_bytes<128, 4>();
        default: return attn_smem_bytes<128, 8>();
        }
    }();
    int xs = std::max(dim, ffn);
    if (xfr + xs * 4 < attn_need) xs = (attn_need - xfr + 3) / 4;
    cudaFuncAttributes fa;
    CK(cudaFuncGetAttributes(&fa, c->pk_kernel));
    int optin = 0;
    CK(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, c->device));
    const int nw = dim;  // RMSNorm weights (every normed phase reads dim columns)
    const long long avail = (long long)optin - (long long)fa.sharedSizeBytes - xfr - (long long)(xs + nw) * 4 - 1024;
    if (avail < (long long)max_tile) return FIBER_OK;  // tiles do not fit: per-phase kernels
    c->pk_ring = (int)(avail & ~127ll);
    // tuning knob: cap the weight ring (KB); the default is all shared memory left
    if (const char *e = getenv("FIBER_PK_RING_KB")) {
        const long long cap = atoll(e) * 1024;
        if (cap >= (long long)max_tile && cap < c->pk_ring) c->pk_ring = (int)(cap & ~127ll);
    }
    c->pk_xfr = xfr;
    c->pk_xs = xs;
    c->pk_nw = nw;
    c->pk_smem = (size_t)c->pk_ring + xfr + (size_t)(xs + nw) * 4;
    CK(cudaFuncSetAttribute(c->pk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c->pk_smem));
    int per_sm = 0;
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, c->pk_kernel, PK_THREADS, c->pk_smem));
    if (per_sm < 1) return FIBER_OK;
    c->pk_grid = grid;
    CK(cudaMalloc(&c->d_phases, ph.size() * sizeof(PPhase)));
    CK(cudaMemcpy(c->d_phases, ph.data(), ph.size() * sizeof(PPhase), cudaMemcpyHostToDevice));
    CK(cudaMalloc(&c->d_bar, ph.size() * sizeof(unsigned int)));
    CK(cudaMemset(c->d_bar, 0, ph.size() * sizeof(unsigned int)));
    c->pk_ok = true;
    return FIBER_OK;
}

template <int HD, int G>
static void *fl_kernel_ptr(bool tp) {
    return tp ? reinterpret_cast<void *>(decode_flow_kernel<HD, G, true>)
              : reinterpret_cast<void *>(decode_flow_kernel<HD, G, false>);
}

// Tensor parallel: this rank's exchange buffer for the dataflow step (n_words tagged words,
// zeroed: tag 0 is never a launch's), and every other rank's, mapped here with CUDA IPC
// (handles all-gathered over the group's NCCL communicator).
static int fl_tp_setup(gpu_context *c, size_t n_words) {
    const int W = c->tp_world, R = c->tp_rank;
    CK(cudaMalloc(&c->fl_tp_local, n_words * 8));
    CK(cudaMemset(c->fl_tp_local, 0, n_words * 8));
    cudaIpcMemHandle_t mine;
    CK(cudaIpcGetMemHandle(&mine, c->fl_tp_local));
    uint8_t *d_h = nullptr;
    CK(cudaMalloc(&d_h, (size_t)(W + 1) * sizeof(mine)));
    std::vector<cudaIpcMemHandle_t> all(W);
    cudaError_t e = cudaMemcpy(d_h + (size_t)W * sizeof(mine), &mine, sizeof(mine), cudaMemcpyHostToDevice);
    if (e == cudaSuccess &&
        ncclAllGather(d_h + (size_t)W * sizeof(mine), d_h, sizeof(mine), ncclUint8, c->comm, c->stream) != ncclSuccess)
        e = cudaErrorUnknown;
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e == cudaSuccess) e = cudaMemcpy(all.data(), d_h, (size_t)W * sizeof(mine), cudaMemcpyDeviceToHost);
    cudaFree(d_h);
    if (e != cudaSuccess) return set_err(FIBER_ECUDA, "dataflow exchange setup (handle exchange): %s", cudaGetErrorString(e));
    for (int q = 0; q < W; q++) {
        if (q == R) continue;
        void *base = nullptr;
        CK(cudaIpcOpenMemHandle(&base, all[q], cudaIpcMemLazyEnablePeerAccess));
        c->fl_tp_peer[q] = base;
    }
    return FIBER_OK;
}

// Phase table, tagged-word buffers and launch geometry of the dataflow step kernel;
// leaves fl_ok false when the model does not fit it.
static int flow_build(gpu_context *c) {
    const model_params_t &p = c->p;
    // this rank's shard (the whole model on one GPU): query heads, KV heads, FFN rows
    const int dim = p.dim, hd = p.head_dim, L = (int)p.n_layers;
    const int qd = c->nh_l * hd, kvd = c->nkv_l * hd, ffn = c->ffn_l;
    const int W = c->tp_world > 1 ? c->tp_world : 1;
    c->fl_ok = false;
    if (W > FL_MAX_TP) return FIBER_OK;
    bool types_ok = fl_type_ok(c->t_out);
    for (const LayerDev &d : c->L) {
        const int ts[7] = {d.tq, d.tk, d.tv, d.to, d.t1, d.t2, d.t3};
        for (int t : ts) types_ok = types_ok && fl_type_ok(t);
        int distinct = 1 + (d.tk != d.tq) + (d.tv != d.tq && d.tv != d.tk);
        types_ok = types_ok && distinct <= 2;
    }
    int scratch = 0;
#define FL_CASE(H, GG)                                         \
    if (hd == H && c->G == GG) {                               \
        c->fl_kernel = fl_kernel_ptr<H, GG>(W > 1);            \
        scratch = FlowAttn<H, GG>::SCRATCH_FLOATS;             \
    }
    FL_CASE(64, 1) FL_CASE(64, 2) FL_CASE(64, 4) FL_CASE(64, 8)
    FL_CASE(128, 1) FL_CASE(128, 2) FL_CASE(128, 4) FL_CASE(128, 8)
#undef FL_CASE
    // per-chunk fragment scales are kept for at most FL_MAX_CHUNKS chunks of 256 inputs
    if (dim / 256 > FL_MAX_CHUNKS || ffn / 256 > FL_MAX_CHUNKS || qd % 256) types_ok = false;
    if (!types_ok || !c->fl_kernel) return FIBER_OK;
    int sms = 0;
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c->device));
    const int grid = sms;

    // tagged words: per layer x (input of QKV), q|k|v, attention, x after Wo, h; then the final x
    const size_t per_layer = (size_t)dim + (qd + 2 * kvd) + qd + dim + ffn;
    const size_t n_words = per_layer * L + dim;
    CK(cudaMalloc(&c->fl_words, n_words * 8));
    CK(cudaMemset(c->fl_words, 0, n_words * 8));  // tag 0: never a launch's tag
    auto xw = [&](int l) { return c->fl_words + per_layer * l; };
    auto qkvw = [&](int l) { return xw(l) + dim; };
    auto attw = [&](int l) { return qkvw(l) + qd + 2 * kvd; };
    auto x1w = [&](int l) { return attw(l) + qd; };
    auto hw = [&](int l) { return x1w(l) + dim; };
    auto xnext = [&](int l) { return l + 1 < L ? xw(l + 1) : c->fl_words + per_layer * L; };
    // tensor parallel: the exchange buffer, [layer][Wo, W_down][world][dim] words in every
    // rank, mapped into the others; a residual phase stores its partial sums to every rank,
    // the next norm phase adds them (rank order) to the residual it keeps
    auto tp_block = [&](int l, int k) { return (long long)((size_t)(2 * l + k) * W * dim); };
    if (W > 1) {
        // + [world][2] words: each rank's best (logit, row) key of a sharded lm_head
        c->fl_tp_key_off = (long long)2 * L * W * dim;
        const int rc = fl_tp_setup(c, (size_t)2 * L * W * dim + 2 * W);
        if (rc != FIBER_OK) return rc;
    }

    std::vector<FPhase> &ph = c->fphases;
    ph.clear();
    auto base = [&](int kind, int cols, int layer) {
        FPhase f;
        memset(&f, 0, sizeof(f));
        f.kind = kind;
        f.cols = cols;
        f.layer = layer;
        f.nmat = 1;
        f.eps = p.rms_norm_eps;
        f.tp_off = -1;
        return f;
    };
    auto tiles_of = [](FPhase &f) {
        f.n_tiles = 0;
        for (int k = 0; k < f.nseg; k++) f.n_tiles += f.seg[k].tiles;
    };
    for (int l = 0; l < L; l++) {
        const LayerDev &d = c->L[l];
        FPhase q = base(FL_QKV, dim, l);
        q.nseg = 3;
        q.seg[0] = make_pseg(d.wq, nullptr, d.tq, qd, 0, dim);
        q.seg[1] = make_pseg(d.wk, nullptr, d.tk, kvd, qd, dim);
        q.seg[2] = make_pseg(d.wv, nullptr, d.tv, kvd, qd + kvd, dim);
        q.embed_in = l == 0;
        q.in = l == 0 ? nullptr : (W > 1 ? c->fl_tp_local + tp_block(l - 1, 1) : xw(l));
        q.tp_sum = l > 0 && W > 1;
        q.norm_w = d.attn_norm;
        q.out = qkvw(l);
        tiles_of(q);
        FPhase a = base(FL_ATTN, qd, l);
        a.in = qkvw(l);
        a.out = attw(l);
        FPhase o = base(FL_RESID, qd, l);
        o.nseg = 1;
        o.seg[0] = make_pseg(d.wo, nullptr, d.to, dim, 0, qd);
        o.in = attw(l);
        o.out = x1w(l);
        if (W > 1) o.tp_off = tp_block(l, 0);
        tiles_of(o);
        FPhase u = base(FL_SWIGLU, dim, l);
        u.nseg = 1;
        u.nmat = 2;
        u.seg[0] = make_pseg(d.w1, d.w3, d.t1, ffn, 0, dim);
        u.seg[0].tiles = (ffn + TC_M / 2 - 1) / (TC_M / 2);  // 8 rows of gate + the same 8 of up
        u.in = W > 1 ? c->fl_tp_local + tp_block(l, 0) : x1w(l);
        u.tp_sum = W > 1;
        u.norm_w = d.ffn_norm;
        u.out = hw(l);
        tiles_of(u);
        FPhase dn = base(FL_RESID, ffn, l);
        dn.nseg = 1;
        dn.seg[0] = make_pseg(d.w2, nullptr, d.t2, dim, 0, ffn);
        dn.in = hw(l);
        dn.out = xnext(l);
        if (W > 1) dn.tp_off = tp_block(l, 1);
        tiles_of(dn);
        // a norm phase keeps its fp32 input as the residual of the next residual phase (and,
        // tensor parallel, of the next norm phase: then every CTA stages every norm phase)
        q.stage_ctas = W > 1 ? grid : std::min(grid, std::max(q.n_tiles, o.n_tiles));
        o.stage_ctas = std::min(grid, o.n_tiles);
        u.stage_ctas = W > 1 ? grid : std::min(grid, std::max(u.n_tiles, dn.n_tiles));
        dn.stage_ctas = std::min(grid, dn.n_tiles);
        ph.push_back(q);
        ph.push_back(a);
        ph.push_back(o);
        ph.push_back(u);
        ph.push_back(dn);
    }
    FPhase lm = base(FL_LM, dim, 0);
    lm.nseg = 1;
    lm.seg[0] = make_pseg(c->out, nullptr, c->t_out, p.vocab_size, 0, dim);
    lm.in = W > 1 ? c->fl_tp_local + tp_block(L - 1, 1) : xnext(L - 1);
    lm.tp_sum = W > 1;
    lm.norm_w = c->out_norm;
    lm.logits = c->logits;
    tiles_of(lm);
    lm.stage_ctas = W > 1 ? grid : std::min(grid, lm.n_tiles);
    ph.push_back(lm);

    // shared memory: fragments (one layout per weight type of a phase), the residual
    // copy, the non-normed input (and attention scratch), the RMSNorm weights, the ring
    size_t max_tile = (size_t)4 * ATTN_P * hd;  // attention: one K page and one V page (fp16)
    int frag = 0;
    for (FPhase &f : ph) {
        if (f.kind == FL_ATTN) continue;
        int types = 1;
        for (int k = 0; k < f.nseg; k++) {
            max_tile = std::max(max_tile, (size_t)TC_M * f.seg[k].stride);
            if (f.seg[k].type != f.seg[0].type) types = 2;
        }
        frag = std::max(frag, types * f.cols * 4);
    }
    frag = (frag + 127) & ~127;
    // attention splits per KV head: about eight pages each at max_seq, at most 8 and at most
    // a grid's worth of units (split 0 merges the others; fewer splits, less scratch)
    const int max_pages = (c->max_seq + ATTN_P - 1) / ATTN_P;
    const int max_split = std::max(1, std::min(std::min(8, grid / c->nkv_l),
                                               (max_pages + FL_PAGES_PER_UNIT - 1) / FL_PAGES_PER_UNIT));
    scratch += (max_split - 1) * c->G * (hd + 2);
    const int xres = (dim + 31) & ~31;
    const int xin = (std::max(std::max(dim, ffn), scratch) + 31) & ~31;
    const int nw = (dim + 31) & ~31;
    cudaFuncAttributes fa;
    CK(cudaFuncGetAttributes(&fa, c->fl_kernel));
    // the producer / consumer register split (setmaxnreg) must fit the registers the
    // block is launched with, or the consumers' increase would wait forever
    if ((long long)fa.numRegs * FL_THREADS < 4LL * 32 * FL_REG_PRODUCER + 8LL * 32 * FL_REG_CONSUMER) {
        fprintf(stderr, "fiber: dataflow kernel launched with %d registers per thread; register split does not fit\n",
                fa.numRegs);
        return FIBER_OK;
    }
    int optin = 0;
    CK(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, c->device));
    const long long avail =
        (long long)optin - (long long)fa.sharedSizeBytes - FL_RING_PAD - frag - (long long)(xres + xin + nw) * 4 - 1024;
    if (avail < (long long)max_tile + 1024) return FIBER_OK;  // tiles do not fit
    c->fl_ring = (int)(avail & ~1023ll);
    if (const char *e = getenv("FIBER_FL_RING_KB")) {  // tuning knob: cap the ring (KB)
        const long long cap = atoll(e) * 1024;
        if (cap >= (long long)max_tile && cap < c->fl_ring) c->fl_ring = (int)(cap & ~127ll);
    }
    c->fl_frag = frag;
    c->fl_xres = xres;
    c->fl_xin = xin;
    c->fl_nw = nw;
    c->fl_smem = (size_t)FL_RING_PAD + c->fl_ring + frag + (size_t)(xres + xin + nw) * 4;
    CK(cudaFuncSetAttribute(c->fl_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c->fl_smem));
    int per_sm = 0;
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, c->fl_kernel, FL_THREADS, c->fl_smem));
    if (per_sm < 1) return FIBER_OK;
    c->fl_grid = grid;
    c->fl_max_split = max_split;
    const size_t att_words = (size_t)L * p.n_kv_heads * max_split * c->G * (hd + 2);
    CK(cudaMalloc(&c->fl_att_words, att_words * 8));
    CK(cudaMemset(c->fl_att_words, 0, att_words * 8));
    CK(cudaMalloc(&c->fl_am, (size_t)grid * 8));
    const size_t n_sync = 4 + p.n_kv_heads;
    CK(cudaMalloc(&c->fl_sync, n_sync * 4));
    CK(cudaMemset(c->fl_sync, 0, n_sync * 4));
    const unsigned int one = 1u;  // first launch tag
    CK(cudaMemcpy(c->fl_sync, &one, 4, cudaMemcpyHostToDevice));
    CK(cudaMalloc(&c->d_fphases, ph.size() * sizeof(FPhase)));
    CK(cudaMemcpy(c->d_fphases, ph.data(), ph.size() * sizeof(FPhase), cudaMemcpyHostToDevice));
    c->fl_ok = true;
    return FIBER_OK;
}

static int tp_setup(gpu_context *c, const model_t *m, int rank, int world, const uint8_t *nccl_id);

static int ctx_init(gpu_context *c, const model_t *m, int device, int max_seq, int rank, int world,
                    const uint8_t *nccl_id) {
    const model_params_t &p = m->params;
    c->device = device;
    c->p = p;
    c->max_seq = max_seq;
    c->kvd = (int)(p.n_kv_heads * p.head_dim);
    c->G = (int)(p.n_heads / p.n_kv_heads);
    c->max_chunks = (max_seq + ATTN_P - 1) / ATTN_P;
    if (c->max_chunks > ATTN_MAX_CHUNKS)
        return set_err(FIBER_EUNSUPPORTED, "max_seq %d exceeds %d positions", max_seq, ATTN_MAX_CHUNKS * ATTN_P);
    if (p.dim % 256 || p.ffn_dim % 256)
        return set_err(FIBER_EUNSUPPORTED, "dim (%u) and ffn_dim (%u) must be multiples of 256", p.dim, p.ffn_dim);
    if (!(p.head_dim == 64 || p.head_dim == 128))
        return set_err(FIBER_EUNSUPPORTED, "head_dim %u not supported (64 or 128)", p.head_dim);
    if (!(c->G == 1 || c->G == 2 || c->G == 4 || c->G == 8))
        return set_err(FIBER_EUNSUPPORTED, "GQA group %d not supported (1, 2, 4, 8)", c->G);
    if (!m->output_norm || m->output_norm_type != GGML_TYPE_F32)
        return set_err(FIBER_EUNSUPPORTED, "output_norm.weight must be F32");
    if (!matrix_type_ok(m->output_type))
        return set_err(FIBER_EUNSUPPORTED, "classifier type %s not supported", tname(m->output_type));
    c->t_embd = m->token_embd_type;
    if (!(matrix_type_ok(c->t_embd) || c->t_embd == T_F32))
        return set_err(FIBER_EUNSUPPORTED, "token_embd type %s not supported", tname(m->token_embd_type));
    for (uint32_t l = 0; l < p.n_layers; l++) {
        const layer_weights_t &w = m->layers[l];
        const int ts[7] = {w.wq_type, w.wk_type, w.wv_type, w.wo_type, w.w1_type, w.w2_type, w.w3_type};
        for (int t : ts)
            if (!matrix_type_ok(t)) return set_err(FIBER_EUNSUPPORTED, "layer %u: weight type %s not supported", l, tname(t));
        if (w.attn_norm_type != GGML_TYPE_F32 || w.ffn_norm_type != GGML_TYPE_F32)
            return set_err(FIBER_EUNSUPPORTED, "layer %u: norms must be F32", l);
        if (w.w1_type != w.w3_type)
            return set_err(FIBER_EUNSUPPORTED, "layer %u: ffn_gate and ffn_up must share a type", l);
    }

    CK(cudaSetDevice(device));
    CK(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    CK(cudaEventCreate(&c->ev0));
    CK(cudaEventCreate(&c->ev1));

    // GGUF data section, unchanged
    const gguf_file_t *gf = m->gf;
    c->data_bytes = gf->file_size - gf->data_offset;
    // + 256 bytes: the prefill GEMM reads Q6_K blocks through 16-byte-aligned spans
    if (cudaMalloc(&c->d_data, c->data_bytes + 256) != cudaSuccess)
        return set_err(FIBER_ENOMEM, "cannot allocate %.1f MB for weights", c->data_bytes / 1e6);
    CK(cudaMemcpy(c->d_data, (const uint8_t *)gf->data + gf->data_offset, c->data_bytes, cudaMemcpyHostToDevice));
    auto dp = [&](uint64_t off) { return c->d_data + off; };
    c->L.resize(p.n_layers);
    for (uint32_t l = 0; l < p.n_layers; l++) {
        const layer_weights_t &w = m->layers[l];
        const layer_offsets_t &o = m->layer_off[l];
        LayerDev &d = c->L[l];
        d.wq = dp(o.wq); d.wk = dp(o.wk); d.wv = dp(o.wv); d.wo = dp(o.wo);
        d.w1 = dp(o.w1); d.w2 = dp(o.w2); d.w3 = dp(o.w3);
        d.attn_norm = (const float *)dp(o.attn_norm);
        d.ffn_norm = (const float *)dp(o.ffn_norm);
        d.tq = w.wq_type; d.tk = w.wk_type; d.tv = w.wv_type; d.to = w.wo_type;
        d.t1 = w.w1_type; d.t2 = w.w2_type; d.t3 = w.w3_type;
    }
    c->embd = dp(m->token_embd_off);
    c->out = dp(m->output_off);
    c->out_norm = (const float *)dp(m->output_norm_off);
    c->t_out = m->output_type;

    const int dim = p.dim, ffn = p.ffn_dim, V = p.vocab_size;
    const int lm_tiles = (V + GEMV_TILE - 1) / GEMV_TILE;
    CK(cudaMalloc(&c->x, (size_t)dim * 4));
    CK(cudaMalloc(&c->qkv, (size_t)(dim + 2 * c->kvd) * 4));
    CK(cudaMalloc(&c->att, (size_t)dim * 4));
    CK(cudaMalloc(&c->h, (size_t)ffn * 4));
    CK(cudaMalloc(&c->logits, (size_t)V * 4));
    CK(cudaMalloc(&c->rope, (size_t)max_seq * (p.head_dim / 2) * sizeof(float2)));
    CK(cudaMalloc(&c->io, sizeof(StepIO)));
    CK(cudaMalloc(&c->rec, (size_t)max_seq * 4));
    // records of hd + 2 floats (per-phase kernels) or PK_REC(hd) floats (persistent kernel)
    CK(cudaMalloc(&c->att_part, (size_t)p.n_kv_heads * c->max_chunks * c->G * (p.head_dim + 4) * 4));
    CK(cudaMalloc(&c->att_cnt, (size_t)p.n_kv_heads * 4));
    CK(cudaMalloc(&c->am_part, (size_t)lm_tiles * sizeof(float2)));
    CK(cudaMalloc(&c->am_cnt, 4));
    CK(cudaMemset(c->att_cnt, 0, (size_t)p.n_kv_heads * 4));
    CK(cudaMemset(c->am_cnt, 0, 4));
    CK(cudaMemset(c->io, 0, sizeof(StepIO)));
    CK(cudaMemset(c->x, 0, (size_t)dim * 4));
    CK(cudaMallocHost(&c->h_io, sizeof(StepIO)));
    CK(cudaMallocHost(&c->h_logits, (size_t)V * 4));
    memset(c->h_io, 0, sizeof(StepIO));
    c->logits_copy.resize(V);

    // RoPE table with the CPU path's expressions (src/fiber_proof.m:33-35)
    const int hd = p.head_dim;
    std::vector<float2> tab((size_t)max_seq * (hd / 2));
    for (int pos = 0; pos < max_seq; pos++)
        for (int i = 0; i < hd / 2; i++) {
            const float freq = 1.0f / powf(p.rope_freq_base, 2.0f * i / (float)hd);
            const float angle = pos * freq;
            tab[(size_t)pos * (hd / 2) + i] = make_float2(cosf(angle), sinf(angle));
        }
    CK(cudaMemcpy(c->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice));
    int rc = tp_setup(c, m, rank, world, nccl_id);
    if (rc) return rc;
    if (world > 1) {
        // sharded steps: the dataflow kernel with the exchange fused into it where the model
        // fits it, else the per-phase kernels with an all-reduce after Wo and W_down
        c->mode = 1;
        if ((rc = flow_build(c)) != FIBER_OK) return rc;
        if (c->fl_ok) c->mode = 2;
        return FIBER_OK;
    }
    if ((rc = pk_build(c)) != FIBER_OK) return rc;
    if ((rc = flow_build(c)) != FIBER_OK) return rc;
    if (c->fl_ok) c->mode = 2;  // the fastest step where the model fits it (dataflow kernel)
    return FIBER_OK;
}

// ---- tensor parallelism ------------------------------------------------------------

extern "C" int fiber_tp_plan(const model_params_t *p, int rank, int world, fiber_tp_plan_t *out) {
    if (!p || !out) return set_err(FIBER_EARG, "fiber_tp_plan: null argument");
    if (world < 1 || rank < 0 || rank >= world) return set_err(FIBER_EARG, "rank %d of world %d", rank, world);
    const int nh = (int)p->n_heads, nkv = (int)p->n_kv_heads, hd = (int)p->head_dim, nblk = (int)p->ffn_dim / 256;
    if (nh % world || nkv % world)
        return set_err(FIBER_EUNSUPPORTED, "%d query / %d KV heads do not split over %d ranks", nh, nkv, world);
    if ((nh / world) * hd % 256)
        return set_err(FIBER_EUNSUPPORTED, "Wo shards of %d columns are not whole super-blocks", (nh / world) * hd);
    if (p->ffn_dim % 256 || nblk < world)
        return set_err(FIBER_EUNSUPPORTED, "ffn_dim %u does not split into %d shards of super-blocks", p->ffn_dim, world);
    out->rank = rank;
    out->world = world;
    out->heads = nh / world;
    out->head0 = rank * out->heads;
    out->kv_heads = nkv / world;
    out->kv_head0 = rank * out->kv_heads;
    out->ffn_block0 = rank * nblk / world;
    out->ffn_blocks = (rank + 1) * nblk / world - out->ffn_block0;
    return FIBER_OK;
}

extern "C" int fiber_tp_unique_id(uint8_t out[FIBER_TP_ID_BYTES]) {
    static_assert(sizeof(ncclUniqueId) == FIBER_TP_ID_BYTES, "ncclUniqueId size");
    if (!out) return set_err(FIBER_EARG, "fiber_tp_unique_id: null argument");
    ncclUniqueId id;
    const ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return set_err(FIBER_ECUDA, "ncclGetUniqueId: %s", ncclGetErrorString(r));
    memcpy(out, &id, sizeof(id));
    return FIBER_OK;
}

// Shard the model for rank `rank`: row ranges of Wq/Wk/Wv and W_gate/W_up are
// addressed in place in the uploaded GGUF data; Wo and W_down are cut along their
// input dimension (whole super-blocks of every row) into d_shard; an NCCL
// communicator joins the ranks.
// The one-shot all-reduce's buffers: every rank allocates its slot area (zeroed: epoch
// 0, before any call), the areas' IPC handles are all-gathered over NCCL (which also
// orders every rank's zeroing before any peer's first push), and each rank maps its
// peers' areas.
static int ar_setup(gpu_context *c, int n_max) {
    const int W = c->tp_world, R = c->tp_rank;
    const size_t total = (size_t)2 * W * n_max * sizeof(unsigned long long);
    CK(cudaMalloc(&c->ar_local, total));
    CK(cudaMemset(c->ar_local, 0, total));
    CK(cudaMalloc(&c->ar_epoch, sizeof(unsigned int)));
    CK(cudaMemset(c->ar_epoch, 0, sizeof(unsigned int)));
    cudaIpcMemHandle_t mine;
    CK(cudaIpcGetMemHandle(&mine, c->ar_local));
    uint8_t *d_h = nullptr;
    CK(cudaMalloc(&d_h, (size_t)(W + 1) * sizeof(mine)));
    std::vector<cudaIpcMemHandle_t> all(W);
    cudaError_t e = cudaMemcpy(d_h + (size_t)W * sizeof(mine), &mine, sizeof(mine), cudaMemcpyHostToDevice);
    if (e == cudaSuccess &&
        ncclAllGather(d_h + (size_t)W * sizeof(mine), d_h, sizeof(mine), ncclUint8, c->comm, c->stream) != ncclSuccess)
        e = cudaErrorUnknown;
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e == cudaSuccess) e = cudaMemcpy(all.data(), d_h, (size_t)W * sizeof(mine), cudaMemcpyDeviceToHost);
    cudaFree(d_h);
    if (e != cudaSuccess) return set_err(FIBER_ECUDA, "all-reduce setup (handle exchange): %s", cudaGetErrorString(e));
    ArParams &a = c->ar;
    memset(&a, 0, sizeof(a));
    a.n_max = n_max;
    a.rank = R;
    a.world = W;
    a.epoch = c->ar_epoch;
    a.err = &c->io->err;
    for (int p = 0; p < W; p++) {
        void *base = c->ar_local;
        if (p != R) {
            CK(cudaIpcOpenMemHandle(&base, all[p], cudaIpcMemLazyEnablePeerAccess));
            c->ar_peer[p] = base;
        }
        a.slots[p] = (unsigned long long *)base;
    }
    c->ar_ok = true;
    return FIBER_OK;
}

static int tp_setup(gpu_context *c, const model_t *m, int rank, int world, const uint8_t *nccl_id) {
    const model_params_t &p = c->p;
    fiber_tp_plan_t plan;
    int rc = fiber_tp_plan(&p, rank, world, &plan);
    if (rc) return rc;
    const int dim = p.dim, hd = p.head_dim;
    c->tp_rank = rank;
    c->tp_world = world;
    c->nh_l = plan.heads;
    c->nkv_l = plan.kv_heads;
    c->h0 = plan.head0;
    c->g0 = plan.kv_head0;
    c->f0b = plan.ffn_block0;
    c->ffn_l = plan.ffn_blocks * 256;
    if (world == 1) return FIBER_OK;
    auto rb = [](int cols, int type) { return (size_t)(cols / 256) * block_bytes(type); };
    const uint8_t *host = (const uint8_t *)m->gf->data + m->gf->data_offset;
    size_t shard_bytes = 0;
    for (uint32_t l = 0; l < p.n_layers; l++)
        shard_bytes += (size_t)dim * (rb(c->nh_l * hd, c->L[l].to) + rb(c->ffn_l, c->L[l].t2));
    CK(cudaMalloc(&c->d_shard, shard_bytes));
    uint8_t *dst = c->d_shard;
    for (uint32_t l = 0; l < p.n_layers; l++) {
        LayerDev &d = c->L[l];
        const layer_offsets_t &o = m->layer_off[l];
        d.wq += (size_t)c->h0 * hd * rb(dim, d.tq);
        d.wk += (size_t)c->g0 * hd * rb(dim, d.tk);
        d.wv += (size_t)c->g0 * hd * rb(dim, d.tv);
        d.w1 += (size_t)c->f0b * 256 * rb(dim, d.t1);
        d.w3 += (size_t)c->f0b * 256 * rb(dim, d.t3);
        const size_t wo_row = rb(dim, d.to), wo_cut = rb(c->nh_l * hd, d.to), wo_off = rb(c->h0 * hd, d.to);
        CK(cudaMemcpy2D(dst, wo_cut, host + o.wo + wo_off, wo_row, wo_cut, dim, cudaMemcpyHostToDevice));
        d.wo = dst;
        dst += (size_t)dim * wo_cut;
        const size_t w2_row = rb(p.ffn_dim, d.t2), w2_cut = rb(c->ffn_l, d.t2), w2_off = rb(c->f0b * 256, d.t2);
        CK(cudaMemcpy2D(dst, w2_cut, host + o.w2 + w2_off, w2_row, w2_cut, dim, cudaMemcpyHostToDevice));
        d.w2 = dst;
        dst += (size_t)dim * w2_cut;
    }
    CK(cudaMalloc(&c->x2, (size_t)dim * 4));
    CK(cudaMemset(c->x2, 0, (size_t)dim * 4));
    ncclUniqueId id;
    memcpy(&id, nccl_id, sizeof(id));
    const ncclResult_t r = ncclCommInitRank(&c->comm, world, id, rank);
    if (r != ncclSuccess) return set_err(FIBER_ECUDA, "ncclCommInitRank: %s", ncclGetErrorString(r));
    const char *coll = getenv("FIBER_TP_ALLREDUCE");
    if (world <= AR_MAX_WORLD && !(coll && strcmp(coll, "nccl") == 0)) return ar_setup(c, dim);
    return FIBER_OK;
}

extern "C" fiber_ctx_t *fiber_cuda_init_tp(const model_t *m, int device, int rank, int world,
                                           const uint8_t nccl_id[FIBER_TP_ID_BYTES], int max_seq) {
    if (!m || !m->layers || (world > 1 && !nccl_id)) {
        set_err(FIBER_EARG, "fiber_cuda_init_tp: no model or no communicator id");
        return nullptr;
    }
    if (max_seq <= 0) max_seq = (int)m->params.context_length;
    gpu_context *c = new gpu_context();
    if (ctx_init(c, m, device, max_seq, rank, world, nccl_id) != FIBER_OK) {
        fprintf(stderr, "fiber_cuda_init_tp: %s\n", g_err);
        fiber_cuda_free(c);
        return nullptr;
    }
    return c;
}

extern "C" int fiber_tp_info(fiber_ctx_t *c, fiber_tp_plan_t *out) {
    if (!c || !out) return set_err(FIBER_EARG, "fiber_tp_info: null argument");
    out->rank = c->tp_rank;
    out->world = c->tp_world;
    out->heads = c->nh_l;
    out->head0 = c->h0;
    out->kv_heads = c->nkv_l;
    out->kv_head0 = c->g0;
    out->ffn_block0 = c->f0b;
    out->ffn_blocks = c->ffn_l / 256;
    return FIBER_OK;
}

static bool batched_ok(const gpu_context *c);

extern "C" fiber_ctx_t *fiber_cuda_init(const model_t *m, int device, int max_batch, int max_seq) {
    if (!m || !m->layers) {
        set_err(FIBER_EARG, "fiber_cuda_init: no model");
        return nullptr;
    }
    if (max_batch < 1 || max_batch > FIBER_MAX_BATCH) {
        set_err(FIBER_EARG, "fiber_cuda_init: max_batch %d outside [1, %d]", max_batch, FIBER_MAX_BATCH);
        return nullptr;
    }
    if (max_seq <= 0) max_seq = (int)m->params.context_length;
    gpu_context *c = new gpu_context();
    if (ctx_init(c, m, device, max_seq, 0, 1, nullptr) != FIBER_OK) {
        fprintf(stderr, "fiber_cuda_init: %s\n", g_err);
        fiber_cuda_free(c);
        return nullptr;
    }
    if (max_batch > 1 && !batched_ok(c)) {
        set_err(FIBER_EUNSUPPORTED,
                "fiber_cuda_init: batched decode needs Q4_K/Q5_K/Q6_K/F16 matrices, 16-byte aligned, GQA group <= 8");
        fiber_cuda_free(c);
        return nullptr;
    }
    c->max_batch = max_batch;
    return c;
}

// ---- the decode step ------------------------------------------------------------------

static cudaError_t enqueue_qkv(gpu_context *c, const LayerDev &d, cudaStream_t st) {
    const int dim = c->p.dim, qd = c->nh_l * (int)c->p.head_dim, kvd = c->nkv_l * (int)c->p.head_dim;
    GemvParams p;
    memset(&p, 0, sizeof(p));
    p.cols = dim;
    p.x = c->x;
    p.norm_w = d.attn_norm;
    p.eps = c->p.rms_norm_eps;
    p.y = c->qkv;
    const uint8_t *ws[3] = {d.wq, d.wk, d.wv};
    const int ts[3] = {d.tq, d.tk, d.tv}, rows[3] = {qd, kvd, kvd}, offs[3] = {0, qd, qd + kvd};
    // group consecutive segments sharing a type into one launch
    int s = 0;
    while (s < 3) {
        GemvParams q = p;
        q.nseg = 0;
        const int t = ts[s];
        while (s < 3 && ts[s] == t) {
            q.seg[q.nseg] = {ws[s], t, rows[s], offs[s]};
            q.tiles[q.nseg] = (rows[s] + GEMV_TILE - 1) / GEMV_TILE;
            q.nseg++;
            s++;
        }
        cudaError_t e = launch_gemv<EPI_STORE>(t, q, grid_of(q), st);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

template <int HD, int G>
static cudaError_t launch_attn_t(const AttnParams &a, cudaStream_t st) {
    return launch_pdl(attn_decode_kernel<HD, G>, dim3(a.max_chunks, a.n_kv), dim3(ATTN_THREADS), 0, st, a);
}

static cudaError_t launch_attn(gpu_context *c, const AttnParams &a, cudaStream_t st) {
    const int hd = c->p.head_dim, G = c->G;
#define ATT_CASE(H, GG) \
    if (hd == H && G == GG) return launch_attn_t<H, GG>(a, st);
    ATT_CASE(64, 1) ATT_CASE(64, 2) ATT_CASE(64, 4) ATT_CASE(64, 8)
    ATT_CASE(128, 1) ATT_CASE(128, 2) ATT_CASE(128, 4) ATT_CASE(128, 8)
#undef ATT_CASE
    return cudaErrorInvalidValue;
}

static cudaError_t launch_embed(gpu_context *c, cudaStream_t st) {
    const int dim = c->p.dim, V = c->p.vocab_size, grid = (dim + 255) / 256;
    int *err = &c->io->err;
    const int32_t *tok = &c->io->token;
    const dim3 g(grid), b(256);
    switch (c->t_embd) {
    case T_Q4_K: return launch_pdl(embed_kernel<T_Q4_K>, g, b, 0, st, c->embd, tok, c->x, dim, V, err);
    case T_Q5_K: return launch_pdl(embed_kernel<T_Q5_K>, g, b, 0, st, c->embd, tok, c->x, dim, V, err);
    case T_Q6_K: return launch_pdl(embed_kernel<T_Q6_K>, g, b, 0, st, c->embd, tok, c->x, dim, V, err);
    case T_F16: return launch_pdl(embed_kernel<T_F16>, g, b, 0, st, c->embd, tok, c->x, dim, V, err);
    case T_F32: return launch_pdl(embed_kernel<T_F32>, g, b, 0, st, c->embd, tok, c->x, dim, V, err);
    default: return cudaErrorInvalidValue;
    }
}

static cudaError_t enqueue_lm_head(gpu_context *c, bool loop, cudaStream_t st) {
    GemvParams p = one_seg(c->out, c->t_out, (int)c->p.vocab_size, 0, (int)c->p.dim);
    p.x = c->x;
    p.norm_w = c->out_norm;
    p.eps = c->p.rms_norm_eps;
    p.y = c->logits;
    p.am_part = c->am_part;
    p.am_count = c->am_cnt;
    p.am_out = &c->io->argmax;
    if (loop) {
        p.adv_token = &c->io->token;
        p.adv_pos = &c->io->pos;
        p.rec_tokens = c->rec;
        p.rec_step = &c->io->step;
    }
    return launch_gemv<EPI_ARGMAX>(c->t_out, p, grid_of(p), st);
}

static AttnParams attn_params(gpu_context *c, const kv_cache_t *kv) {
    const model_params_t &p = c->p;
    AttnParams a;
    memset(&a, 0, sizeof(a));
    a.qkv = c->qkv;
    a.rope = c->rope;
    a.k_pool = kv->k_pool;
    a.v_pool = kv->v_pool;
    a.page_table = kv->page_table;
    a.pos_ptr = &c->io->pos;
    a.part = c->att_part;
    a.count = c->att_cnt;
    a.out = c->att;
    a.n_layers = p.n_layers;
    a.n_kv = c->nkv_l;
    a.n_heads = c->nh_l;
    a.max_chunks = c->max_chunks;
    a.max_seq = c->max_seq < kv->max_seq ? c->max_seq : kv->max_seq;
    a.scale = 1.0f / sqrtf((float)p.head_dim);
    a.err = &c->io->err;
    return a;
}

// One kernel kind of layer l as the decode step issues it (kind: 0 QKV,
// 1 attention, 2 Wo, 3 gate/up+SwiGLU, 4 down, 5 lm_head, 6 embedding).
static cudaError_t enqueue_kind(gpu_context *c, const kv_cache_t *kv, int kind, int l, bool loop, cudaStream_t st) {
    const model_params_t &p = c->p;
    const int dim = p.dim, ffn = p.ffn_dim;
    const LayerDev &d = c->L[l];
    switch (kind) {
    case 0: return enqueue_qkv(c, d, st);
    case 1: {
        AttnParams a = attn_params(c, kv);
        a.layer = l;
        return launch_attn(c, a, st);
    }
    case 2: {
        // TP: each rank's partial product over its heads goes to x2 (rank 0 adds the
        // residual) and is all-reduced by the caller; otherwise in place on x
        GemvParams wo = one_seg(d.wo, d.to, dim, 0, c->nh_l * (int)p.head_dim);
        wo.x = c->att;
        wo.resid = c->tp_world > 1 && c->tp_rank > 0 ? nullptr : c->x;
        wo.y = c->tp_world > 1 ? c->x2 : nullptr;
        return launch_gemv<EPI_RESID>(d.to, wo, grid_of(wo), st);
    }
    case 3: {
        GemvParams up = one_seg(d.w1, d.t1, c->ffn_l, 0, dim);
        up.w_up = d.w3;
        up.x = c->tp_world > 1 ? c->x2 : c->x;
        up.norm_w = d.ffn_norm;
        up.eps = p.rms_norm_eps;
        up.y = c->h;
        return launch_gemv<EPI_SWIGLU>(d.t1, up, grid_of(up), st);
    }
    case 4: {
        GemvParams dn = one_seg(d.w2, d.t2, dim, 0, c->ffn_l);
        dn.x = c->h;
        dn.resid = c->tp_world > 1 ? (c->tp_rank > 0 ? nullptr : c->x2) : c->x;
        dn.y = c->tp_world > 1 ? c->x : nullptr;
        return launch_gemv<EPI_RESID>(d.t2, dn, grid_of(dn), st);
    }
    case 5: return enqueue_lm_head(c, loop, st);
    case 6: return launch_embed(c, st);
    default: return cudaErrorInvalidValue;
    }
}

// Enqueue one full decode step. `loop` makes the lm_head feed its argmax back as
// the next token and advance the position (device-resident greedy decoding).
static cudaError_t enqueue_persistent(gpu_context *c, const kv_cache_t *kv, bool loop, cudaStream_t st,
                                      unsigned long long *trace = nullptr) {
    PParams P;
    memset(&P, 0, sizeof(P));
    P.phases = c->d_phases;
    P.n_phases = (int)c->phases.size();
    P.bar = c->d_bar;
    P.embd = c->embd;
    P.embd_type = c->t_embd;
    P.dim = c->p.dim;
    P.vocab = c->p.vocab_size;
    P.x = c->x;
    P.attn = attn_params(c, kv);
    P.am_part = c->am_part;
    P.am_count = c->am_cnt;
    P.io_token = &c->io->token;
    P.io_pos = &c->io->pos;
    P.io_argmax = &c->io->argmax;
    P.io_err = &c->io->err;
    P.io_step = &c->io->step;
    P.rec_tokens = c->rec;
    P.loop = loop ? 1 : 0;
    P.ring_bytes = c->pk_ring;
    P.xf_bytes = c->pk_xfr;
    P.xs_floats = c->pk_xs;
    P.nw_floats = c->pk_nw;
    P.trace = trace;
    cudaError_t e = cudaMemsetAsync(c->d_bar, 0, c->phases.size() * sizeof(unsigned int), st);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c->pk_grid);
    cfg.blockDim = dim3(PK_THREADS);
    cfg.dynamicSmemBytes = c->pk_smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: the grid barriers rely on it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *args[] = {&P};
    return cudaLaunchKernelExC(&cfg, c->pk_kernel, args);
}

// Decode modes: 0 the grid-barrier persistent kernel, 1 one kernel per phase (CUDA
// graph), 2 the dataflow kernel (tagged-word hand-off between phases).
static bool use_flow(const gpu_context *c) { return c->mode == 2 && c->fl_ok; }
static bool use_pk(const gpu_context *c) { return c->mode == 0 && c->pk_ok; }

// 2D tensor map of a K or V pool for the dataflow attention: rows = page * layer * kv_head
// * 64 positions, head_dim fp16 columns; box 64 columns x 64 rows, 128-byte swizzle.
static bool fl_make_kv_map(CUtensorMap *map, const uint16_t *pool, const kv_cache_t *kv) {
    memset(map, 0, sizeof(*map));
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn)
            return false;
        encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    }
    const cuuint64_t rows = (cuuint64_t)kv->n_pages * kv->n_layers * kv->n_kv_heads * kv->page_size;
    const cuuint64_t dims[2] = {(cuuint64_t)kv->head_dim, rows};
    const cuuint64_t strides[1] = {(cuuint64_t)kv->head_dim * 2};
    const cuuint32_t box[2] = {64u, (cuuint32_t)kv->page_size};
    const cuuint32_t estr[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (void *)pool, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Enqueue one decode step as one launch of the dataflow kernel (cooperative: all
// CTAs co-resident, one per SM). No per-launch memset: every hand-off word carries
// the launch tag, which the kernel advances when its last CTA exits.
static cudaError_t enqueue_flow(gpu_context *c, const kv_cache_t *kv, bool loop, cudaStream_t st,
                                unsigned long long *trace = nullptr) {
    const model_params_t &p = c->p;
    const long long rows = (long long)kv->n_pages * kv->n_layers * kv->n_kv_heads * kv->page_size;
    if (c->fl_map_k != kv->k_pool || c->fl_map_v != kv->v_pool || c->fl_map_rows != rows) {
        c->fl_map_k = c->fl_map_v = nullptr;
        if (!fl_make_kv_map(&c->fl_kmap, kv->k_pool, kv) || !fl_make_kv_map(&c->fl_vmap, kv->v_pool, kv))
            return cudaErrorInvalidValue;
        c->fl_map_k = kv->k_pool;
        c->fl_map_v = kv->v_pool;
        c->fl_map_rows = rows;
    }
    FParams P;
    memset(&P, 0, sizeof(P));
    P.kmap = c->fl_kmap;
    P.vmap = c->fl_vmap;
    P.phases = c->d_fphases;
    P.n_phases = (int)c->fphases.size();
    P.embd = c->embd;
    P.embd_type = c->t_embd;
    P.dim = p.dim;
    P.vocab = p.vocab_size;
    P.rope = c->rope;
    P.k_pool = kv->k_pool;
    P.v_pool = kv->v_pool;
    P.page_table = kv->page_table;
    P.n_layers = p.n_layers;
    P.n_kv = c->nkv_l;
    P.n_heads = c->nh_l;
    P.max_seq = c->max_seq < kv->max_seq ? c->max_seq : kv->max_seq;
    P.att_scale = 1.0f / sqrtf((float)p.head_dim);
    P.att_max_split = c->fl_max_split;
    P.tp_world = c->tp_world > 1 ? c->tp_world : 1;
    P.tp_rank = c->tp_world > 1 ? c->tp_rank : 0;
    for (int q = 0; q < FL_MAX_TP; q++)
        P.tp_bufs[q] = q < P.tp_world ? (q == P.tp_rank ? c->fl_tp_local : (uint64_t *)c->fl_tp_peer[q]) : nullptr;
    P.lm_shard = P.tp_world > 1 && c->fl_lm_shard ? 1 : 0;
    P.tp_key_off = c->fl_tp_key_off;
    P.att_words = c->fl_att_words;
    P.hd = (int)p.head_dim;
    P.G = c->G;
    P.am_key = c->fl_am;
    P.am_count = c->fl_sync + 2;
    P.io_token = &c->io->token;
    P.io_pos = &c->io->pos;
    P.io_argmax = &c->io->argmax;
    P.io_err = &c->io->err;
    P.io_step = &c->io->step;
    P.rec_tokens = c->rec;
    P.loop = loop ? 1 : 0;
    P.epoch = c->fl_sync;
    P.exit_count = c->fl_sync + 1;
    P.ring_bytes = c->fl_ring;
    P.frag_bytes = c->fl_frag;
    P.xres_floats = c->fl_xres;
    P.xin_floats = c->fl_xin;
    P.nw_floats = c->fl_nw;
    P.trace = trace;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c->fl_grid);
    cfg.blockDim = dim3(FL_THREADS);
    cfg.dynamicSmemBytes = c->fl_smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: consumers wait on other CTAs' words
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *args[] = {&P};
    return cudaLaunchKernelExC(&cfg, c->fl_kernel, args);
}

static cudaError_t enqueue_step(gpu_context *c, const kv_cache_t *kv, bool loop, cudaStream_t st) {
    if (use_flow(c)) return enqueue_flow(c, kv, loop, st);
    if (use_pk(c)) return enqueue_persistent(c, kv, loop, st);
    cudaError_t e = enqueue_kind(c, kv, 6, 0, loop, st);
    for (uint32_t l = 0; l < c->p.n_layers && e == cudaSuccess; l++)
        for (int kind = 0; kind <= 4 && e == cudaSuccess; kind++) {
            e = enqueue_kind(c, kv, kind, (int)l, loop, st);
            if (e == cudaSuccess && c->tp_world > 1 && (kind == 2 || kind == 4)) {
                // sum of the ranks' partial products (+ residual from rank 0)
                float *buf = kind == 2 ? c->x2 : c->x;
                if (c->ar_ok) {
                    ArParams a = c->ar;
                    a.buf = buf;
                    a.n = c->p.dim;
                    ar_oneshot_kernel<<<1, AR_THREADS, 0, st>>>(a);
                    e = cudaGetLastError();
                } else if (ncclAllReduce(buf, buf, c->p.dim, ncclFloat, ncclSum, c->comm, st) != ncclSuccess) {
                    e = cudaErrorUnknown;
                }
            }
        }
    if (e == cudaSuccess) e = enqueue_lm_head(c, loop, st);
    return e;
}

static int get_graph(gpu_context *c, const kv_cache_t *kv, bool loop, cudaGraphExec_t *out) {
    Graph &g = loop ? c->g_loop : c->g_step;
    if (g.exec && g.kv == kv) {
        *out = g.exec;
        return FIBER_OK;
    }
    free_graph(g);
    cudaGraph_t graph;
    CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = enqueue_step(c, kv, loop, c->stream);
    cudaError_t e2 = cudaStreamEndCapture(c->stream, &graph);
    if (e != cudaSuccess) return set_err(FIBER_ECUDA, "capturing the decode step: %s", cudaGetErrorString(e));
    if (e2 != cudaSuccess) return set_err(FIBER_ECUDA, "end capture: %s", cudaGetErrorString(e2));
    e = cudaGraphInstantiate(&g.exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return set_err(FIBER_ECUDA, "graph instantiate: %s", cudaGetErrorString(e));
    g.kv = kv;
    *out = g.exec;
    return FIBER_OK;
}

// One decode step on the context stream: the persistent kernel is launched
// directly (one memset + one kernel), the per-phase path replays its graph.
static int run_step(gpu_context *c, const kv_cache_t *kv, bool loop) {
    if (use_flow(c)) {
        cudaError_t e = enqueue_flow(c, kv, loop, c->stream);
        if (e != cudaSuccess) return set_err(FIBER_ECUDA, "dataflow step launch: %s", cudaGetErrorString(e));
        return FIBER_OK;
    }
    if (use_pk(c)) {
        cudaError_t e = enqueue_persistent(c, kv, loop, c->stream);
        if (e != cudaSuccess) return set_err(FIBER_ECUDA, "persistent step launch: %s", cudaGetErrorString(e));
        return FIBER_OK;
    }
    cudaGraphExec_t g;
    int rc = get_graph(c, kv, loop, &g);
    if (rc != FIBER_OK) return rc;
    CK(cudaGraphLaunch(g, c->stream));
    return FIBER_OK;
}

static int check_kv(gpu_context *c, const kv_cache_t *kv) {
    if (!kv) return set_err(FIBER_EARG, "no KV cache");
    if (kv->device != c->device || kv->n_layers != (int)c->p.n_layers || kv->n_kv_heads != c->nkv_l ||
        kv->head_dim != (int)c->p.head_dim || kv->page_size != ATTN_P)
        return set_err(FIBER_EARG, "KV cache does not match the model/device");
    return FIBER_OK;
}

static int device_status(gpu_context *c) {
    if (c->h_io->err == 1) return set_err(FIBER_EARG, "position out of range on the device");
    if (c->h_io->err == 2) return set_err(FIBER_EARG, "token id out of range on the device");
    if (c->h_io->err == 7)
        return set_err(FIBER_ETIMEOUT, "tensor-parallel all-reduce: a peer's data did not arrive in time");
    if (c->h_io->err == 5)
        return set_err(FIBER_EUNSUPPORTED, use_flow(c) ? "a non-finite activation in the decode step"
                                                       : "an activation exceeded the fp16 fragment range of the "
                                                         "persistent kernel; use decode mode 1 or 2");
    if (c->h_io->err == 4) {
        // a bounded wait gave up mid-step: merge tickets may be left non-zero
        cudaMemset(c->att_cnt, 0, (size_t)c->p.n_kv_heads * sizeof(unsigned int));
        cudaMemset(c->am_cnt, 0, sizeof(unsigned int));
        if (c->fl_sync) cudaMemset(c->fl_sync + 1, 0, (3 + c->p.n_kv_heads) * sizeof(unsigned int));
        cudaDeviceSynchronize();
        return set_err(FIBER_ETIMEOUT, "a device-side wait timed out during the decode step");
    }
    return FIBER_OK;
}

static int forward_batch(gpu_context *c, kv_cache_t *kv, const int32_t *tokens, const int32_t *pos, int batch,
                         float *logits_or_null, int32_t *argmax_or_null);

extern "C" int fiber_forward_token(fiber_ctx_t *c, kv_cache_t *kv, const int32_t *tokens, const int32_t *pos,
                                   int batch, float *logits_or_null, int32_t *argmax_or_null) {
    if (!c || !tokens || !pos) return set_err(FIBER_EARG, "fiber_forward_token: null argument");
    if (batch != 1) return forward_batch(c, kv, tokens, pos, batch, logits_or_null, argmax_or_null);
    int rc = check_kv(c, kv);
    if (rc) return rc;
    const int lim = c->max_seq < kv->max_seq ? c->max_seq : kv->max_seq;
    if (pos[0] < 0 || pos[0] >= lim) return set_err(FIBER_EARG, "position %d outside [0, %d)", pos[0], lim);
    if (tokens[0] < 0 || tokens[0] >= (int)c->p.vocab_size) return set_err(FIBER_EARG, "token %d out of range", tokens[0]);
    CK(cudaSetDevice(c->device));
    c->h_io->token = tokens[0];
    c->h_io->pos = pos[0];
    c->h_io->err = 0;
    CK(cudaMemcpyAsync(c->io, c->h_io, sizeof(StepIO), cudaMemcpyHostToDevice, c->stream));
    c->fl_lm_shard = !logits_or_null;  // token only: tensor-parallel ranks split the lm_head
    rc = run_step(c, kv, false);
    c->fl_lm_shard = false;
    if (rc != FIBER_OK) return rc;
    if (logits_or_null)
        CK(cudaMemcpyAsync(c->h_logits, c->logits, (size_t)c->p.vocab_size * 4, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaMemcpyAsync(c->h_io, c->io, sizeof(StepIO), cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    if ((rc = device_status(c)) != FIBER_OK) return rc;
    if (logits_or_null) memcpy(logits_or_null, c->h_logits, (size_t)c->p.vocab_size * 4);
    if (argmax_or_null) argmax_or_null[0] = c->h_io->argmax;
    return FIBER_OK;
}

// ---- batched prefill ------------------------------------------------------------------

constexpr int PF_CHUNK = FIBER_PREFILL_CHUNK;  // tokens per pass of the layer stack

static cudaError_t launch_g5(const G5Params &p, cudaStream_t st);

static bool g5_type_ok(int t) { return t == T_Q4_K || t == T_Q5_K || t == T_Q6_K || t == T_F16; }

// The batched layer pass (tensor-core GEMMs) covers this model: prefill chunks and
// batched decode steps.
static bool batched_ok(const gpu_context *c) {
    if ((c->nh_l * (int)c->p.head_dim) % 256) return false;  // Wo's input columns: whole super-blocks
    if (!g5_type_ok(c->t_out) || c->G > 8 || ((uintptr_t)c->out & 15)) return false;
    for (const LayerDev &d : c->L) {
        const int ts[7] = {d.tq, d.tk, d.tv, d.to, d.t1, d.t2, d.t3};
        for (int t : ts)
            if (!g5_type_ok(t)) return false;
        // the GEMM streams weight rows with 16-byte-aligned bulk / tensor copies
        const uint8_t *ws[7] = {d.wq, d.wk, d.wv, d.wo, d.w1, d.w2, d.w3};
        for (const uint8_t *w : ws)
            if ((uintptr_t)w & 15) return false;
    }
    return true;
}

static bool prefill_batched_ok(const gpu_context *c) { return c->prefill_mode == 0 && batched_ok(c); }

constexpr int ATT_PART_ENTRIES = 2048;  // (token, KV head, split) states of one page-split launch

template <int HD, int G>
static cudaError_t launch_attn_prefill_t(const AttnPrefillParams &a, int n, int ps, cudaStream_t st) {
    attn_prefill_kernel<HD, G><<<dim3(n, a.n_kv, ps), ATTN_THREADS, 0, st>>>(a);
    return cudaGetLastError();
}

// Page split: enough (token, KV head, split) CTAs for about eight waves, each split
// keeping at least 4 of the longest context's pages (short contexts stay unsplit).
static int attn_psplit(int n, int n_kv, int max_pos) {
    const int base = n * n_kv, pages = (max_pos + ATTN_P - 1) / ATTN_P;
    int ps = (8 * sm_count() + base - 1) / base;
    ps = std::min(ps, std::min(16, pages / 4));
    ps = std::min(ps, ATT_PART_ENTRIES / base);
    return ps < 1 ? 1 : ps;
}

template <int HD, int G>
static cudaError_t launch_attn_prefill_tb_t(const AttnPrefillParams &a, int n, cudaStream_t st) {
    constexpr int TB = apf_tb(HD, G);
    attn_prefill_tb_kernel<HD, G, TB><<<dim3((n + TB - 1) / TB, a.n_kv), ATTN_THREADS, 0, st>>>(a, n);
    return cudaGetLastError();
}

static cudaError_t launch_attn_prefill(const gpu_context *c, const AttnPrefillParams &a, int n, cudaStream_t st) {
    const int hd = c->p.head_dim, G = c->G;
    const int ps = (a.part && a.tickets) ? attn_psplit(n, a.n_kv, a.at.max_pos) : 1;
    if (ps == 1 && !a.at.pos && a.at.slot_step == 0 && G < 8) {  // prompt chunk: blocks of tokens
#define APT_CASE(H, GG) \
    if (hd == H && G == GG) return launch_attn_prefill_tb_t<H, GG>(a, n, st);
        APT_CASE(64, 1) APT_CASE(64, 2) APT_CASE(64, 4)
        APT_CASE(128, 1) APT_CASE(128, 2) APT_CASE(128, 4)
#undef APT_CASE
    }
#define APF_CASE(H, GG) \
    if (hd == H && G == GG) return launch_attn_prefill_t<H, GG>(a, n, ps, st);
    APF_CASE(64, 1) APF_CASE(64, 2) APF_CASE(64, 4) APF_CASE(64, 8)
    APF_CASE(128, 1) APF_CASE(128, 2) APF_CASE(128, 4) APF_CASE(128, 8)
#undef APF_CASE
    return cudaErrorInvalidValue;
}

static cudaError_t launch_embed_rows(const gpu_context *c, const int32_t *tok, float *X, int n, cudaStream_t st) {
    const int dim = c->p.dim, V = c->p.vocab_size;
    const dim3 g((dim + 255) / 256, n), b(256);
    int *err = &c->io->err;
    switch (c->t_embd) {
    case T_Q4_K: embed_rows_kernel<T_Q4_K><<<g, b, 0, st>>>(c->embd, tok, X, dim, V, err); break;
    case T_Q5_K: embed_rows_kernel<T_Q5_K><<<g, b, 0, st>>>(c->embd, tok, X, dim, V, err); break;
    case T_Q6_K: embed_rows_kernel<T_Q6_K><<<g, b, 0, st>>>(c->embd, tok, X, dim, V, err); break;
    case T_F16: embed_rows_kernel<T_F16><<<g, b, 0, st>>>(c->embd, tok, X, dim, V, err); break;
    case T_F32: embed_rows_kernel<T_F32><<<g, b, 0, st>>>(c->embd, tok, X, dim, V, err); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

// Row length in bytes of a weight matrix as the GEMM reads it: Q6_K rows are padded to
// a multiple of 16 bytes (tensor copies need 16-byte-aligned row strides).
static size_t g5_row_bytes(int type, int cols) {
    const size_t rb = (size_t)cols / 256 * block_bytes(type);
    return type == T_Q6_K ? (rb + 15) / 16 * 16 : rb;
}

// 2D tensor map over a weight matrix (rows of g5_row_bytes, 16-byte aligned) with a box
// of 128 rows x one K unit: a super-block (Q4_K 144, Q5_K 176 bytes; Q6_K the 224-byte
// span around its 210-byte block) or 128 fp16 values.
static bool g5_make_map(CUtensorMap *map, const uint8_t *w, int type, int rows, int cols) {
    memset(map, 0, sizeof(*map));
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn)
            return false;
        encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    }
    const bool q4 = type != T_F16;  // byte elements, one super-block per box row
    const cuuint32_t bb = type == T_Q4_K ? 144u : (type == T_Q5_K ? 176u : 224u);
    const cuuint64_t row_bytes = g5_row_bytes(type, cols);
    const cuuint64_t dims[2] = {q4 ? row_bytes : (cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {q4 ? bb : 128u, (cuuint32_t)G5_M};
    const cuuint32_t estr[2] = {1, 1};
    return encode(map, q4 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (void *)w, dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The weights as the GEMM reads them: w itself, or for Q6_K rows that are not a multiple
// of 16 bytes long a copy with padded rows (kept in c->pf_pad, or handed to the caller
// to free when c is null).
static cudaError_t g5_weights(gpu_context *c, const uint8_t *w, int type, int rows, int cols, const uint8_t **out,
                              void **owned = nullptr) {
    const size_t rb = (size_t)cols / 256 * block_bytes(type), prb = g5_row_bytes(type, cols);
    *out = w;
    if (prb == rb) return cudaSuccess;
    void *d = nullptr;
    cudaError_t e = cudaMalloc(&d, prb * rows);
    if (e != cudaSuccess) return e;
    e = cudaMemcpy2D(d, prb, w, rb, rb, rows, cudaMemcpyDeviceToDevice);
    if (e != cudaSuccess) {
        cudaFree(d);
        return e;
    }
    if (c) c->pf_pad.push_back(d);
    if (owned) *owned = d;
    *out = (const uint8_t *)d;
    return cudaSuccess;
}

static cudaError_t launch_g5_pack(const G5PackParams &a, cudaStream_t st) {
    const dim3 grid(((a.ntok + G5_T - 1) / G5_T) * (G5_T / 4), a.cols / G5_PACK_COLS);
    return launch_pdl(g5_pack_kernel, grid, dim3(128), 0, st, a);
}

// Pack n rows of x (RMS-normalised with weights nw when given) into c->pf_bp.
static cudaError_t pf_pack(gpu_context *c, const float *x, int cols, const float *nw, int n, cudaStream_t st) {
    G5PackParams a;
    memset(&a, 0, sizeof(a));
    a.x = x;
    a.ldx = cols;
    a.ntok = n;
    a.cols = cols;
    a.nw = nw;
    a.own_rms = nw != nullptr;
    a.eps = c->p.rms_norm_eps;
    a.bp = c->pf_bp;
    a.err = &c->io->err;
    return launch_g5_pack(a, st);
}

// One tensor-core GEMM of the prefill on the packed input: y[t][off + r] (+)= W[r,:] . xn[t,:]
static cudaError_t pf_gemm(gpu_context *c, const CUtensorMap &map, const uint8_t *w, int type, int rows, int cols,
                           float *y, int ldy, int off, bool acc, int n, cudaStream_t st,
                           const float *resid = nullptr) {
    G5Params g;
    memset(&g, 0, sizeof(g));
    g.resid = resid;
    g.wmap = map;
    g.w = w;
    g.type = type;
    g.rows = rows;
    g.cols = cols;
    g.ntok = n;
    g.bp = c->pf_bp;
    g.y = y;
    g.ldy = ldy;
    g.out_off = off;
    g.epi = acc ? G5_RESID : G5_STORE;
    g.err = &c->io->err;
    return launch_g5(g, st);
}

// The layers over `n` tokens whose hidden states are in c->pf_x, each at its place
// (position, KV slot): per layer RMSNorm + packing of the input, QKV GEMMs, RoPE + KV
// append, causal attention, Wo GEMM (+residual), RMSNorm + packing, gate/up GEMMs,
// SwiGLU, down GEMM (+residual).
static cudaError_t enqueue_layers(gpu_context *c, const kv_cache_t *kv, int n, const TokenPlace &at, cudaStream_t st) {
    const model_params_t &p = c->p;
    // this rank's share (the whole model when tp_world == 1): query / KV heads, FFN rows
    const int dim = p.dim, hd = p.head_dim, qd = c->nh_l * hd, kvd = c->nkv_l * hd, ffn = c->ffn_l;
    const int ldq = qd + 2 * kvd;
    const bool tp = c->tp_world > 1, lead = c->tp_rank == 0;
    // tensor parallel: partial products summed over the ranks (rank 0 adds the residual)
    auto reduce = [&](float *buf) -> cudaError_t {
        if (!tp) return cudaSuccess;
        return ncclAllReduce(buf, buf, (size_t)n * dim, ncclFloat, ncclSum, c->comm, st) == ncclSuccess
                   ? cudaSuccess
                   : cudaErrorUnknown;
    };
    cudaError_t e = cudaSuccess;
    for (uint32_t l = 0; l < p.n_layers && e == cudaSuccess; l++) {
        const LayerDev &d = c->L[l];
        const CUtensorMap *mp = &c->pf_maps[7 * l];
        const uint8_t *const *pw = &c->pf_w[7 * l];
        if ((e = pf_pack(c, c->pf_x, dim, d.attn_norm, n, st))) break;
        if ((e = pf_gemm(c, mp[0], pw[0], d.tq, qd, dim, c->pf_qkv, ldq, 0, false, n, st))) break;
        if ((e = pf_gemm(c, mp[1], pw[1], d.tk, kvd, dim, c->pf_qkv, ldq, qd, false, n, st))) break;
        if ((e = pf_gemm(c, mp[2], pw[2], d.tv, kvd, dim, c->pf_qkv, ldq, qd + kvd, false, n, st))) break;
        RopeKvParams rk;
        rk.qkv = c->pf_qkv;
        rk.ldq = ldq;
        rk.at = at;
        rk.rope = c->rope;
        rk.n_heads = c->nh_l;
        rk.n_kv = c->nkv_l;
        rk.hd = hd;
        rk.k_pool = kv->k_pool;
        rk.v_pool = kv->v_pool;
        rk.page_table = kv->page_table;
        rk.layer = l;
        rk.n_layers = p.n_layers;
        rope_kv_kernel<<<n, 256, 0, st>>>(rk);
        if ((e = cudaGetLastError()) != cudaSuccess) break;
        AttnPrefillParams ap;
        ap.qkv = c->pf_qkv;
        ap.ldq = ldq;
        ap.out = c->pf_att;
        ap.ldo = qd;
        ap.at = at;
        ap.k_pool = kv->k_pool;
        ap.v_pool = kv->v_pool;
        ap.page_table = kv->page_table;
        ap.layer = l;
        ap.n_layers = p.n_layers;
        ap.n_kv = c->nkv_l;
        ap.n_heads = c->nh_l;
        ap.scale = 1.0f / sqrtf((float)hd);
        ap.part = c->att_ws;
        ap.tickets = c->att_tickets;
        if ((e = launch_attn_prefill(c, ap, n, st))) break;
        if ((e = pf_pack(c, c->pf_att, qd, nullptr, n, st))) break;
        // residual stream after Wo: pf_x (single GPU) or pf_x2 (sum over the ranks)
        float *xa = tp ? c->pf_x2 : c->pf_x;
        if (tp) {
            if ((e = pf_gemm(c, mp[3], pw[3], d.to, dim, qd, xa, dim, 0, false, n, st, lead ? c->pf_x : nullptr))) break;
            if ((e = reduce(xa))) break;
        } else if ((e = pf_gemm(c, mp[3], pw[3], d.to, dim, qd, xa, dim, 0, true, n, st))) {
            break;
        }
        if ((e = pf_pack(c, xa, dim, d.ffn_norm, n, st))) break;
        if ((e = pf_gemm(c, mp[4], pw[4], d.t1, ffn, dim, c->pf_hg, ffn, 0, false, n, st))) break;
        if ((e = pf_gemm(c, mp[6], pw[6], d.t3, ffn, dim, c->pf_hu, ffn, 0, false, n, st))) break;
        swiglu_rows_kernel<<<(n * ffn + 255) / 256, 256, 0, st>>>(c->pf_hg, c->pf_hu, (size_t)n * ffn);
        if ((e = cudaGetLastError()) != cudaSuccess) break;
        if ((e = pf_pack(c, c->pf_hg, ffn, nullptr, n, st))) break;
        if (tp) {
            if ((e = pf_gemm(c, mp[5], pw[5], d.t2, dim, ffn, c->pf_x, dim, 0, false, n, st, lead ? xa : nullptr))) break;
            e = reduce(c->pf_x);
        } else {
            e = pf_gemm(c, mp[5], pw[5], d.t2, dim, ffn, c->pf_x, dim, 0, true, n, st);
        }
    }
    return e;
}

static TokenPlace place_of(gpu_context *c, const kv_cache_t *kv) {
    TokenPlace at;
    memset(&at, 0, sizeof(at));
    at.max_pages = kv->max_pages_per_seq;
    at.max_pos = c->max_seq < kv->max_seq ? c->max_seq : kv->max_seq;
    at.err = &c->io->err;
    return at;
}

// A prompt chunk of `n` tokens (c->pf_tok) of KV slot `slot` at positions start ..:
// embedding rows and the layers; leaves the last token's hidden state in c->x.
static cudaError_t enqueue_prefill_chunk(gpu_context *c, const kv_cache_t *kv, int n, int start, int slot,
                                         cudaStream_t st) {
    TokenPlace at = place_of(c, kv);
    at.start = start;
    at.slot = slot;
    cudaError_t e = launch_embed_rows(c, c->pf_tok, c->pf_x, n, st);
    if (e == cudaSuccess) e = enqueue_layers(c, kv, n, at, st);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(c->x, c->pf_x + (size_t)(n - 1) * c->p.dim, (size_t)c->p.dim * 4,
                            cudaMemcpyDeviceToDevice, st);
    return e;
}

// One greedy decode step of `n` sequences: token c->pf_tok[t] at position c->bt_pos[t]
// of KV slot t. Embedding rows, the layers, final RMSNorm + the classifier as one GEMM
// over the n rows (c->bt_logits), argmax per row (c->bt_arg). `loop` feeds the argmax
// back as the next tokens, advances the positions and records the tokens.
static cudaError_t enqueue_batch_step(gpu_context *c, const kv_cache_t *kv, int n, bool loop, cudaStream_t st) {
    const int dim = c->p.dim, V = c->p.vocab_size;
    TokenPlace at = place_of(c, kv);
    at.pos = c->bt_pos;
    at.slot_step = 1;
    cudaError_t e = launch_embed_rows(c, c->pf_tok, c->pf_x, n, st);
    if (e == cudaSuccess) e = enqueue_layers(c, kv, n, at, st);
    if (e == cudaSuccess) e = pf_pack(c, c->pf_x, dim, c->out_norm, n, st);
    if (e == cudaSuccess) e = pf_gemm(c, c->out_map, c->pf_out, c->t_out, V, dim, c->bt_logits, V, 0, false, n, st);
    if (e == cudaSuccess) {
        argmax_rows_kernel<<<n, 256, 0, st>>>(c->bt_logits, V, V, c->bt_arg);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess && loop) {
        batch_advance_kernel<<<1, 64, 0, st>>>(c->bt_arg, c->pf_tok, c->bt_pos, c->bt_rec, c->bt_step, n);
        e = cudaGetLastError();
    }
    return e;
}

// Buffers and tensor maps of the batched layer pass, made on first use.
static int pf_alloc(gpu_context *c) {
    if (c->pf_cap) return FIBER_OK;
    const model_params_t &p = c->p;
    const size_t T = PF_CHUNK;
    CK(cudaMalloc(&c->pf_x, T * p.dim * 4));
    CK(cudaMalloc(&c->pf_qkv, T * (p.dim + 2 * c->kvd) * 4));
    CK(cudaMalloc(&c->pf_att, T * p.dim * 4));
    CK(cudaMalloc(&c->pf_hg, T * p.ffn_dim * 4));
    CK(cudaMalloc(&c->pf_hu, T * p.ffn_dim * 4));
    const size_t kmax = p.dim > p.ffn_dim ? p.dim : p.ffn_dim;
    CK(cudaMalloc(&c->pf_bp, (T + G5_T - 1) / G5_T * G5_T * kmax * 4));
    CK(cudaMalloc(&c->pf_tok, T * 4));
    if (c->tp_world > 1) CK(cudaMalloc(&c->pf_x2, T * p.dim * 4));
    const size_t B = c->max_batch;
    CK(cudaMalloc(&c->bt_pos, B * 4));
    CK(cudaMalloc(&c->bt_arg, B * 4));
    CK(cudaMalloc(&c->bt_rec, B * c->max_seq * 4));
    CK(cudaMalloc(&c->bt_step, sizeof(int)));
    CK(cudaMalloc(&c->bt_logits, B * p.vocab_size * 4));
    CK(cudaMalloc(&c->att_ws, (size_t)ATT_PART_ENTRIES * c->G * (p.head_dim + 2) * 4));
    CK(cudaMalloc(&c->att_tickets, ATT_PART_ENTRIES * sizeof(unsigned int)));
    CK(cudaMemset(c->att_tickets, 0, ATT_PART_ENTRIES * sizeof(unsigned int)));
    c->pf_maps.assign(7 * p.n_layers, CUtensorMap{});
    c->pf_w.assign(7 * p.n_layers, nullptr);
    // this rank's share: rows of Wq / Wk / Wv / W1 / W3, input columns of Wo / W2
    const int dim = p.dim, hd = p.head_dim, qd = c->nh_l * hd, kvd = c->nkv_l * hd, ffn = c->ffn_l;
    for (uint32_t l = 0; l < p.n_layers; l++) {
        const LayerDev &d = c->L[l];
        const uint8_t *ws[7] = {d.wq, d.wk, d.wv, d.wo, d.w1, d.w2, d.w3};
        const int ts[7] = {d.tq, d.tk, d.tv, d.to, d.t1, d.t2, d.t3};
        const int rows[7] = {qd, kvd, kvd, dim, ffn, dim, ffn}, cols[7] = {dim, dim, dim, qd, dim, ffn, dim};
        for (int k = 0; k < 7; k++) {
            const uint8_t **pw = &c->pf_w[7 * l + k];
            CK(g5_weights(c, ws[k], ts[k], rows[k], cols[k], pw));
            if (!g5_make_map(&c->pf_maps[7 * l + k], *pw, ts[k], rows[k], cols[k]))
                return set_err(FIBER_ECUDA, "batched layer pass: cannot build the weight tensor maps");
        }
    }
    CK(g5_weights(c, c->out, c->t_out, (int)p.vocab_size, dim, &c->pf_out));
    if (!g5_make_map(&c->out_map, c->pf_out, c->t_out, (int)p.vocab_size, dim))
        return set_err(FIBER_ECUDA, "batched layer pass: cannot build the classifier tensor map");
    c->pf_cap = PF_CHUNK;
    return FIBER_OK;
}



static void reset_g5_tickets(gpu_context *c);

static int prefill_batched(gpu_context *c, kv_cache_t *kv, int slot, const int32_t *tokens, int n, int start_pos,
                           int32_t *argmax_out) {
    int rc = pf_alloc(c);
    if (rc) return rc;
    c->h_io->err = 0;
    CK(cudaMemcpyAsync(c->io, c->h_io, sizeof(StepIO), cudaMemcpyHostToDevice, c->stream));
    for (int i = 0; i < n; i += c->pf_cap) {
        const int m = std::min(c->pf_cap, n - i);
        CK(cudaMemcpyAsync(c->pf_tok, tokens + i, (size_t)m * 4, cudaMemcpyHostToDevice, c->stream));
        cudaError_t e = enqueue_prefill_chunk(c, kv, m, start_pos + i, slot, c->stream);
        if (e != cudaSuccess) return set_err(FIBER_ECUDA, "batched prefill: %s", cudaGetErrorString(e));
        CK(cudaStreamSynchronize(c->stream));  // pf_tok is reused by the next chunk
    }
    cudaError_t e = enqueue_lm_head(c, false, c->stream);
    if (e != cudaSuccess) return set_err(FIBER_ECUDA, "prefill lm_head: %s", cudaGetErrorString(e));
    CK(cudaMemcpyAsync(c->h_io, c->io, sizeof(StepIO), cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    if (c->h_io->err == 6) {
        reset_g5_tickets(c);
        return set_err(FIBER_ETIMEOUT, "batched prefill: a tensor-core wait timed out");
    }
    if ((rc = device_status(c))) return rc;
    if (argmax_out) *argmax_out = c->h_io->argmax;
    return FIBER_OK;
}

extern "C" int fiber_set_prefill_mode(fiber_ctx_t *c, int mode) {
    if (!c || mode < 0 || mode > 1) return set_err(FIBER_EARG, "fiber_set_prefill_mode: mode must be 0 or 1");
    c->prefill_mode = mode;
    return FIBER_OK;
}

static int prefill_checks(gpu_context *c, kv_cache_t *kv, const int32_t *tokens, int n, int start_pos) {
    int rc = check_kv(c, kv);
    if (rc) return rc;
    const int lim = c->max_seq < kv->max_seq ? c->max_seq : kv->max_seq;
    if (start_pos < 0 || start_pos + n > lim)
        return set_err(FIBER_EARG, "prefill positions %d..%d outside [0, %d)", start_pos, start_pos + n - 1, lim);
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= (int)c->p.vocab_size)
            return set_err(FIBER_EARG, "token %d out of range", tokens[i]);
    return FIBER_OK;
}

extern "C" int fiber_prefill(fiber_ctx_t *c, kv_cache_t *kv, const int32_t *tokens, int n, int start_pos,
                             int32_t *argmax_out) {
    if (!c || !tokens || n <= 0) return set_err(FIBER_EARG, "fiber_prefill: empty prompt");
    if (n > 1 && prefill_batched_ok(c)) {
        int rc = prefill_checks(c, kv, tokens, n, start_pos);
        if (rc) return rc;
        CK(cudaSetDevice(c->device));
        return prefill_batched(c, kv, 0, tokens, n, start_pos, argmax_out);
    }
    for (int i = 0; i < n; i++) {
        const int32_t pos = start_pos + i;
        int rc = fiber_forward_token(c, kv, tokens + i, &pos, 1, nullptr, i == n - 1 ? argmax_out : nullptr);
        if (rc) return rc;
    }
    return FIBER_OK;
}

extern "C" int fiber_prefill_slot(fiber_ctx_t *c, kv_cache_t *kv, int slot, const int32_t *tokens, int n,
                                  int start_pos, int32_t *argmax_out) {
    if (!c || !tokens || n <= 0) return set_err(FIBER_EARG, "fiber_prefill_slot: empty prompt");
    if (!kv || slot < 0 || slot >= kv->max_batch) return set_err(FIBER_EARG, "fiber_prefill_slot: no slot %d", slot);
    if (!batched_ok(c)) return set_err(FIBER_EUNSUPPORTED, "fiber_prefill_slot: the batched layer pass does not cover this model");
    int rc = prefill_checks(c, kv, tokens, n, start_pos);
    if (rc) return rc;
    CK(cudaSetDevice(c->device));
    return prefill_batched(c, kv, slot, tokens, n, start_pos, argmax_out);
}

// ---- batched decode -------------------------------------------------------------------

static int batch_checks(gpu_context *c, kv_cache_t *kv, const int32_t *tokens, const int32_t *pos, int batch,
                        int n_steps) {
    if (!tokens || !pos) return set_err(FIBER_EARG, "batched decode: null argument");
    if (batch < 1 || batch > c->max_batch)
        return set_err(FIBER_EARG, "batch %d outside [1, max_batch %d]", batch, c->max_batch);
    int rc = check_kv(c, kv);
    if (rc) return rc;
    if (batch > kv->max_batch) return set_err(FIBER_EARG, "batch %d exceeds the KV cache's %d slots", batch, kv->max_batch);
    const int lim = c->max_seq < kv->max_seq ? c->max_seq : kv->max_seq;
    for (int t = 0; t < batch; t++) {
        if (pos[t] < 0 || pos[t] + n_steps > lim)
            return set_err(FIBER_EARG, "sequence %d: positions %d..%d outside [0, %d)", t, pos[t], pos[t] + n_steps - 1,
                           lim);
        if (tokens[t] < 0 || tokens[t] >= (int)c->p.vocab_size)
            return set_err(FIBER_EARG, "sequence %d: token %d out of range", t, tokens[t]);
    }
    return FIBER_OK;
}

// After a timed-out GEMM, split-K tickets may be left non-zero.
static void reset_g5_tickets(gpu_context *c) {
    if (c->att_tickets) cudaMemset(c->att_tickets, 0, ATT_PART_ENTRIES * sizeof(unsigned int));
    cudaDeviceSynchronize();
}

static int batch_status(gpu_context *c) {
    if (c->h_io->err == 6) {
        reset_g5_tickets(c);
        return set_err(FIBER_ETIMEOUT, "batched decode: a tensor-core wait timed out");
    }
    if (c->h_io->err == 3) return set_err(FIBER_EARG, "batched decode: a position left the cache on the device");
    return device_status(c);
}

static int forward_batch(gpu_context *c, kv_cache_t *kv, const int32_t *tokens, const int32_t *pos, int batch,
                         float *logits_or_null, int32_t *argmax_or_null) {
    int rc = batch_checks(c, kv, tokens, pos, batch, 1);
    if (rc) return rc;
    CK(cudaSetDevice(c->device));
    if ((rc = pf_alloc(c))) return rc;
    c->h_io->err = 0;
    CK(cudaMemcpyAsync(c->io, c->h_io, sizeof(StepIO), cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(c->pf_tok, tokens, (size_t)batch * 4, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(c->bt_pos, pos, (size_t)batch * 4, cudaMemcpyHostToDevice, c->stream));
    cudaError_t e = enqueue_batch_step(c, kv, batch, false, c->stream);
    if (e != cudaSuccess) return set_err(FIBER_ECUDA, "batched decode step: %s", cudaGetErrorString(e));
    if (logits_or_null)
        CK(cudaMemcpyAsync(logits_or_null, c->bt_logits, (size_t)batch * c->p.vocab_size * 4, cudaMemcpyDeviceToHost,
                           c->stream));
    if (argmax_or_null)
        CK(cudaMemcpyAsync(argmax_or_null, c->bt_arg, (size_t)batch * 4, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaMemcpyAsync(c->h_io, c->io, sizeof(StepIO), cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    return batch_status(c);
}

extern "C" int fiber_decode_greedy_batch(fiber_ctx_t *c, kv_cache_t *kv, const int32_t *first_tokens,
                                         const int32_t *start_pos, int batch, int n_steps, int32_t *h_tokens_out,
                                         float *ms_out) {
    if (!c || n_steps <= 0) return set_err(FIBER_EARG, "fiber_decode_greedy_batch: bad arguments");
    if (!batched_ok(c)) return set_err(FIBER_EUNSUPPORTED, "batched decode does not cover this model");
    int rc = batch_checks(c, kv, first_tokens, start_pos, batch, n_steps);
    if (rc) return rc;
    CK(cudaSetDevice(c->device));
    if ((rc = pf_alloc(c))) return rc;
    c->h_io->err = 0;
    CK(cudaMemcpyAsync(c->io, c->h_io, sizeof(StepIO), cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(c->pf_tok, first_tokens, (size_t)batch * 4, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(c->bt_pos, start_pos, (size_t)batch * 4, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemsetAsync(c->bt_step, 0, sizeof(int), c->stream));
    Graph &g = c->g_batch;
    if (!(g.exec && g.kv == kv && c->g_batch_n == batch)) {  // capture before the timed region
        free_graph(g);
        cudaGraph_t graph;
        CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
        cudaError_t e = enqueue_batch_step(c, kv, batch, true, c->stream);
        cudaError_t e2 = cudaStreamEndCapture(c->stream, &graph);
        if (e != cudaSuccess) return set_err(FIBER_ECUDA, "capturing the batch step: %s", cudaGetErrorString(e));
        if (e2 != cudaSuccess) return set_err(FIBER_ECUDA, "end capture: %s", cudaGetErrorString(e2));
        e = cudaGraphInstantiate(&g.exec, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) return set_err(FIBER_ECUDA, "graph instantiate: %s", cudaGetErrorString(e));
        g.kv = kv;
        c->g_batch_n = batch;
    }
    CK(cudaEventRecord(c->ev0, c->stream));
    for (int i = 0; i < n_steps; i++) CK(cudaGraphLaunch(g.exec, c->stream));
    CK(cudaEventRecord(c->ev1, c->stream));
    CK(cudaEventSynchronize(c->ev1));
    if (ms_out) CK(cudaEventElapsedTime(ms_out, c->ev0, c->ev1));
    if (h_tokens_out)
        CK(cudaMemcpyAsync(h_tokens_out, c->bt_rec, (size_t)n_steps * batch * 4, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaMemcpyAsync(c->h_io, c->io, sizeof(StepIO), cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    return batch_status(c);
}

extern "C" int fiber_set_decode_mode(fiber_ctx_t *c, int mode) {
    if (!c || mode < 0 || mode > 2) return set_err(FIBER_EARG, "fiber_set_decode_mode: mode must be 0, 1 or 2");
    if (mode == 0 && !c->pk_ok) return set_err(FIBER_EUNSUPPORTED, "the persistent step kernel does not fit this model");
    if (mode == 2 && !c->fl_ok) return set_err(FIBER_EUNSUPPORTED, "the dataflow step kernel does not fit this model");
    if (c->mode != mode) {
        free_graph(c->g_step);
        free_graph(c->g_loop);
        c->mode = mode;
    }
    return FIBER_OK;
}

extern "C" int fiber_get_decode_mode(fiber_ctx_t *c) {
    if (!c) return set_err(FIBER_EARG, "no context");
    return use_flow(c) ? 2 : use_pk(c) ? 0 : 1;
}

extern "C" int fiber_step_launches(fiber_ctx_t *c) {
    if (!c) return set_err(FIBER_EARG, "no context");
    if (use_flow(c) || use_pk(c)) return 1;
    int n = 2;  // embed + lm_head
    for (const LayerDev &d : c->L) n += 4 + 1 + (d.tk != d.tq) + (d.tv != d.tk);
    return n;
}

extern "C" int fiber_step_ring_bytes(fiber_ctx_t *c) {
    if (!c) return set_err(FIBER_EARG, "no context");
    return use_flow(c) ? c->fl_ring : use_pk(c) ? c->pk_ring : 0;
}

extern "C" int fiber_trace_step(fiber_ctx_t *c, kv_cache_t *kv, int token, int pos, uint64_t *out, size_t cap,
                                int *n_phases, int *n_ctas) {
    if (!c || !out || !n_phases || !n_ctas) return set_err(FIBER_EARG, "fiber_trace_step: null argument");
    const bool fl = use_flow(c);
    if (!fl && !c->pk_ok) return set_err(FIBER_EUNSUPPORTED, "the persistent step kernels do not cover this model");
    int rc = check_kv(c, kv);
    if (rc) return rc;
    const int lim = c->max_seq < kv->max_seq ? c->max_seq : kv->max_seq;
    if (pos < 0 || pos >= lim) return set_err(FIBER_EARG, "position %d outside [0, %d)", pos, lim);
    if (token < 0 || token >= (int)c->p.vocab_size) return set_err(FIBER_EARG, "token %d out of range", token);
    const size_t n = fl ? c->fphases.size() * (size_t)c->fl_grid * FL_TRACE_FIELDS
                        : c->phases.size() * (size_t)c->pk_grid * PK_TRACE_FIELDS;
    *n_phases = (int)(fl ? c->fphases.size() : c->phases.size());
    *n_ctas = fl ? c->fl_grid : c->pk_grid;
    if (cap < n) return set_err(FIBER_EARG, "trace buffer holds %zu values, %zu needed", cap, n);
    CK(cudaSetDevice(c->device));
    unsigned long long *d_tr = nullptr;
    CK(cudaMalloc(&d_tr, n * 8));
    cudaError_t e = cudaMemsetAsync(d_tr, 0, n * 8, c->stream);
    c->h_io->token = token;
    c->h_io->pos = pos;
    c->h_io->err = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(c->io, c->h_io, sizeof(StepIO), cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = fl ? enqueue_flow(c, kv, false, c->stream, d_tr) : enqueue_persistent(c, kv, false, c->stream, d_tr);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, d_tr, n * 8, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(c->h_io, c->io, sizeof(StepIO), cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(d_tr);
    if (e != cudaSuccess) return set_err(FIBER_ECUDA, "trace step: %s", cudaGetErrorString(e));
    return device_status(c);
}

static double kind_bytes(gpu_context *c, int kind, int l, int pos) {
    const model_params_t &p = c->p;
    const LayerDev &d = c->L[l];
    auto mb = [&](int t, double rows, double cols) { return rows * cols / 256.0 * block_bytes(t); };
    switch (kind) {
    case 0: return mb(d.tq, p.dim, p.dim) + mb(d.tk, c->kvd, p.dim) + mb(d.tv, c->kvd, p.dim) + 4.0 * p.dim * 2 +
                   4.0 * (p.dim + 2 * c->kvd);
    case 1: return 2.0 * c->kvd * 2.0 * (pos + 1) + 4.0 * (p.dim + 2 * c->kvd) + 4.0 * p.dim;
    case 2: return mb(d.to, p.dim, p.dim) + 4.0 * p.dim * 3;
    case 3: return mb(d.t1, p.ffn_dim, p.dim) + mb(d.t3, p.ffn_dim, p.dim) + 4.0 * p.dim * 2 + 4.0 * p.ffn_dim;
    case 4: return mb(d.t2, p.dim, p.ffn_dim) + 4.0 * p.ffn_dim + 4.0 * p.dim * 2;
    case 5: return mb(c->t_out, p.vocab_size, p.dim) + 4.0 * p.dim * 2 + 4.0 * p.vocab_size;
    case 6: return (double)p.dim / 256.0 * block_bytes(c->t_embd) + 4.0 * p.dim;
    default: return 0.0;
    }
}

extern "C" int fiber_time_kernel(fiber_ctx_t *c, kv_cache_t *kv, int kind, int pos, int reps, double *us_per_launch,
                                 double *bytes_per_launch) {
    if (!c || kind < 0 || kind > 6 || reps <= 0) return set_err(FIBER_EARG, "fiber_time_kernel: bad arguments");
    int rc = check_kv(c, kv);
    if (rc) return rc;
    const int lim = c->max_seq < kv->max_seq ? c->max_seq : kv->max_seq;
    if (pos < 0 || pos >= lim) return set_err(FIBER_EARG, "fiber_time_kernel: position %d outside [0, %d)", pos, lim);
    CK(cudaSetDevice(c->device));
    c->h_io->pos = pos;
    c->h_io->err = 0;
    CK(cudaMemcpyAsync(c->io, c->h_io, sizeof(StepIO), cudaMemcpyHostToDevice, c->stream));
    const int L = (int)c->p.n_layers;
    cudaGraph_t graph;
    CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = cudaSuccess;
    double bytes = 0.0;
    for (int l = 0; l < L && e == cudaSuccess; l++) {
        e = enqueue_kind(c, kv, kind, l, false, c->stream);
        bytes += kind_bytes(c, kind, l, pos);
    }
    cudaError_t e2 = cudaStreamEndCapture(c->stream, &graph);
    if (e != cudaSuccess || e2 != cudaSuccess)
        return set_err(FIBER_ECUDA, "fiber_time_kernel capture: %s", cudaGetErrorString(e != cudaSuccess ? e : e2));
    cudaGraphExec_t exec;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return set_err(FIBER_ECUDA, "fiber_time_kernel instantiate: %s", cudaGetErrorString(e));
    e = cudaGraphLaunch(exec, c->stream);  // warm-up replay
    if (e == cudaSuccess) e = cudaEventRecord(c->ev0, c->stream);
    for (int r = 0; r < reps && e == cudaSuccess; r++) e = cudaGraphLaunch(exec, c->stream);
    if (e == cudaSuccess) e = cudaEventRecord(c->ev1, c->stream);
    if (e == cudaSuccess) e = cudaEventSynchronize(c->ev1);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, c->ev0, c->ev1);
    cudaGraphExecDestroy(exec);
    if (e != cudaSuccess) return set_err(FIBER_ECUDA, "fiber_time_kernel: %s", cudaGetErrorString(e));
    if (us_per_launch) *us_per_launch = 1e3 * ms / ((double)reps * L);
    if (bytes_per_launch) *bytes_per_launch = bytes / L;
    return FIBER_OK;
}


extern "C" int fiber_decode_greedy(fiber_ctx_t *c, kv_cache_t *kv, int32_t first_token, int start_pos, int n_steps,
                                   int32_t *h_tokens_out, float *ms_out) {
    if (!c || n_steps <= 0) return set_err(FIBER_EARG, "fiber_decode_greedy: bad arguments");
    int rc = check_kv(c, kv);
    if (rc) return rc;
    const int lim = c->max_seq < kv->max_seq ? c->max_seq : kv->max_seq;
    if (start_pos < 0 || start_pos + n_steps > lim)
        return set_err(FIBER_EARG, "decode of %d steps from %d exceeds max_seq %d", n_steps, start_pos, lim);
    if (first_token < 0 || first_token >= (int)c->p.vocab_size) return set_err(FIBER_EARG, "token %d out of range", first_token);
    CK(cudaSetDevice(c->device));
    c->h_io->token = first_token;
    c->h_io->pos = start_pos;
    c->h_io->step = 0;
    c->h_io->err = 0;
    CK(cudaMemcpyAsync(c->io, c->h_io, sizeof(StepIO), cudaMemcpyHostToDevice, c->stream));
    {
        if (!use_flow(c) && !use_pk(c)) {  // build the graph before the timed region
            cudaGraphExec_t g;
            if ((rc = get_graph(c, kv, true, &g)) != FIBER_OK) return rc;
        }
        CK(cudaEventRecord(c->ev0, c->stream));
        c->fl_lm_shard = true;  // tokens only: tensor-parallel ranks split the lm_head
        for (int i = 0; i < n_steps && rc == FIBER_OK; i++) rc = run_step(c, kv, true);
        c->fl_lm_shard = false;
        if (rc != FIBER_OK) return rc;
        CK(cudaEventRecord(c->ev1, c->stream));
        CK(cudaEventSynchronize(c->ev1));
        if (ms_out) CK(cudaEventElapsedTime(ms_out, c->ev0, c->ev1));
    }
    CK(cudaMemcpyAsync(c->h_io, c->io, sizeof(StepIO), cudaMemcpyDeviceToHost, c->stream));
    if (h_tokens_out) CK(cudaMemcpyAsync(h_tokens_out, c->rec, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    return device_status(c);
}

// ---- reference-named API (include/gpu_ffn.h) --------------------------------------------

extern "C" gpu_context_t *gpu_init(const model_t *m) {
    gpu_context_t *c = fiber_cuda_init(m, 0, 1, m ? (int)m->params.context_length : 0);
    if (c) {
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, 0) == cudaSuccess) printf("GPU: %s\n", prop.name);
        printf("GPU: %.1f MB of GGUF tensor data resident in HBM\n", c->data_bytes / (1024.0 * 1024.0));
    }
    return c;
}

extern "C" void gpu_free(gpu_context_t *c) { fiber_cuda_free(c); }

extern "C" void gpu_embed(gpu_context_t *c, const model_t *m, int token_id) {
    (void)m;
    if (c) c->h_io->token = token_id;
}

extern "C" double gpu_forward_token(gpu_context_t *c, const model_t *m, kv_cache_t *kv, int pos) {
    (void)m;
    if (!c) return -1.0;
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    const int32_t tok = c->h_io->token, p = pos;
    const int rc = fiber_forward_token(c, kv, &tok, &p, 1, c->logits_copy.data(), nullptr);
    clock_gettime(CLOCK_MONOTONIC, &t1);
    if (rc != FIBER_OK) {
        fprintf(stderr, "gpu_forward_token: %s\n", g_err);
        return -1.0;
    }
    return (t1.tv_sec - t0.tv_sec) * 1e3 + (t1.tv_nsec - t0.tv_nsec) / 1e6;
}

extern "C" const float *gpu_get_logits(gpu_context_t *c) { return c ? c->logits_copy.data() : nullptr; }

extern "C" void gpu_forward_classifier(gpu_context_t *c, const model_t *m) {
    (void)m;
    if (!c) return;
    if (cudaSetDevice(c->device) != cudaSuccess || enqueue_lm_head(c, false, c->stream) != cudaSuccess ||
        cudaMemcpyAsync(c->logits_copy.data(), c->logits, (size_t)c->p.vocab_size * 4, cudaMemcpyDeviceToHost,
                        c->stream) != cudaSuccess ||
        cudaStreamSynchronize(c->stream) != cudaSuccess)
        fprintf(stderr, "gpu_forward_classifier: CUDA error\n");
}

extern "C" int gpu_get_device(gpu_context_t *c) { return c ? c->device : -1; }

// ---- kernel-level entry points -----------------------------------------------------------

extern "C" int fiber_gemv(int type, const void *d_w, const float *d_x, float *d_y, int rows, int cols, void *stream) {
    if (!matrix_type_ok(type)) return set_err(FIBER_EARG, "fiber_gemv: type %d not supported", type);
    if (!d_w || !d_x || !d_y || rows <= 0 || cols <= 0 || cols % 256)
        return set_err(FIBER_EARG, "fiber_gemv: bad shape %dx%d (cols must be a positive multiple of 256)", rows, cols);
    if (((uintptr_t)d_w & 15) || ((uintptr_t)d_x & 15))
        return set_err(FIBER_EARG, "fiber_gemv: weights and x must be 16-byte aligned");
    GemvParams p = one_seg((const uint8_t *)d_w, type, rows, 0, cols);
    p.x = d_x;
    p.y = d_y;
    CK(launch_gemv<EPI_STORE>(type, p, grid_of(p), (cudaStream_t)stream));
    return FIBER_OK;
}

extern "C" int fiber_gemv_host(int type, const void *d_w, const float *h_x, float *h_y, int rows, int cols,
                               float *d_x, float *d_y, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    CK(cudaMemcpyAsync(d_x, h_x, (size_t)cols * 4, cudaMemcpyHostToDevice, st));
    int rc = fiber_gemv(type, d_w, d_x, d_y, rows, cols, stream);
    if (rc) return rc;
    CK(cudaMemcpyAsync(h_y, d_y, (size_t)rows * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    return FIBER_OK;
}

extern "C" int fiber_dequant(int type, const void *d_w, void *d_out, int rows, int cols, void *stream) {
    if (!matrix_type_ok(type) || !d_w || !d_out || rows <= 0 || cols <= 0 || cols % 256)
        return set_err(FIBER_EARG, "fiber_dequant: bad arguments");
    cudaStream_t st = (cudaStream_t)stream;
    const int grid = 148 * 8;
    const uint8_t *w = (const uint8_t *)d_w;
    switch (type) {
    case T_Q4_K: dequant_kernel<T_Q4_K><<<grid, 256, 0, st>>>(w, d_out, rows, cols); break;
    case T_Q5_K: dequant_kernel<T_Q5_K><<<grid, 256, 0, st>>>(w, d_out, rows, cols); break;
    case T_Q6_K: dequant_kernel<T_Q6_K><<<grid, 256, 0, st>>>(w, d_out, rows, cols); break;
    case T_F16: dequant_kernel<T_F16><<<grid, 256, 0, st>>>(w, d_out, rows, cols); break;
    }
    CK(cudaGetLastError());
    return FIBER_OK;
}

// ---- tensor-core dequant-GEMM (prefill) -------------------------------------------------

// Clusters of `ks` GEMM CTAs that fit on the device at once (per device, type and ks).
template <int T>
static int g5_cluster_capacity(int ks) {
    static int cache[64][G5_MAX_KSPLIT + 1];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    int &v = cache[dev][ks];
    if (v == 0) {
        cudaLaunchConfig_t cfg;
        memset(&cfg, 0, sizeof(cfg));
        cfg.gridDim = dim3(1, 1, ks);
        cfg.blockDim = dim3(G5_THREADS);
        cfg.dynamicSmemBytes = g5_smem_bytes(T);
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = ks;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_tc5_kernel<T>, &cfg) != cudaSuccess || n <= 0) n = -1;
        v = n;
    }
    return v;
}

template <int T>
static cudaError_t launch_g5_t(const G5Params &p, cudaStream_t st) {
    const int smem = g5_smem_bytes(T);
    cudaError_t e = cudaFuncSetAttribute(gemm_tc5_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    // K splits: as many as help (g5_choose_ksplit) while every cluster is resident at once
    const int base = ((p.rows + G5_M - 1) / G5_M) * ((p.ntok + G5_T - 1) / G5_T);
    int ks = g5_choose_ksplit(T, p.rows, p.cols, p.ntok, sm_count());
    while (ks > 1 && g5_cluster_capacity<T>(ks) < base) ks--;
    cudaGetLastError();  // clear a failed occupancy query
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3((p.rows + G5_M - 1) / G5_M, (p.ntok + G5_T - 1) / G5_T, ks);
    cfg.blockDim = dim3(G5_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;  // the K splits of a tile: one cluster
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = ks;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, gemm_tc5_kernel<T>, p);
}

static cudaError_t launch_g5(const G5Params &p, cudaStream_t st) {
    switch (p.type) {
    case T_Q4_K: return launch_g5_t<T_Q4_K>(p, st);
    case T_Q5_K: return launch_g5_t<T_Q5_K>(p, st);
    case T_Q6_K: return launch_g5_t<T_Q6_K>(p, st);
    case T_F16: return launch_g5_t<T_F16>(p, st);
    default: return cudaErrorInvalidValue;
    }
}

static __device__ int g_g5_err;

extern "C" int fiber_gemm(int ggml_type, const void *d_w, int rows, int cols, const float *d_x, int ntok, int ldx,
                          const float *d_rrms, const float *d_nw, float *d_y, int ldy, int out_off, int accumulate,
                          void *stream) {
    if (!d_w || !d_x || !d_y || rows <= 0 || ntok <= 0 || cols <= 0 || cols % 256 || ldx < cols ||
        ldy < out_off + rows || ldx % 4 || ((uintptr_t)d_w & 15) || ((uintptr_t)d_x & 15) || ((uintptr_t)d_nw & 15))
        return set_err(FIBER_EARG, "fiber_gemm: bad arguments");
    if (!g5_type_ok(ggml_type))
        return set_err(FIBER_EUNSUPPORTED, "fiber_gemm: type %s not supported (Q4_K, Q5_K, Q6_K, F16)",
                       tname(ggml_type));
    cudaStream_t st = (cudaStream_t)stream;
    G5Params p;
    memset(&p, 0, sizeof(p));
    const uint8_t *w = (const uint8_t *)d_w;
    void *pad = nullptr;  // Q6_K rows re-laid at a 16-byte stride for this call
    CK(g5_weights(nullptr, w, ggml_type, rows, cols, &w, &pad));
    if (!g5_make_map(&p.wmap, w, ggml_type, rows, cols)) {
        if (pad) cudaFree(pad);
        return set_err(FIBER_ECUDA, "fiber_gemm: cannot build the weight tensor map");
    }
    int *err = nullptr;
    CK(cudaGetSymbolAddress((void **)&err, g_g5_err));
    CK(cudaMemsetAsync(err, 0, sizeof(int), st));
    uint8_t *bp = nullptr;
    CK(cudaMalloc(&bp, (size_t)(ntok + G5_T - 1) / G5_T * G5_T * cols * 4));
    G5PackParams a;
    memset(&a, 0, sizeof(a));
    a.x = d_x;
    a.ldx = ldx;
    a.ntok = ntok;
    a.cols = cols;
    a.rrms = d_rrms;
    a.nw = d_nw;
    a.bp = bp;
    a.err = err;
    p.w = w;
    p.type = ggml_type;
    p.rows = rows;
    p.cols = cols;
    p.ntok = ntok;
    p.bp = bp;
    p.y = d_y;
    p.ldy = ldy;
    p.out_off = out_off;
    p.epi = accumulate ? G5_RESID : G5_STORE;
    p.err = err;
    cudaError_t e = launch_g5_pack(a, st);
    if (e == cudaSuccess) e = launch_g5(p, st);
    int h_err = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&h_err, err, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaFree(bp);
    if (pad) cudaFree(pad);
    if (e != cudaSuccess) return set_err(FIBER_ECUDA, "fiber_gemm: %s", cudaGetErrorString(e));
    if (h_err == 5) return set_err(FIBER_EARG, "fiber_gemm: an input value does not fit fp16");
    if (h_err) return set_err(FIBER_ETIMEOUT, "fiber_gemm: a tensor-core wait timed out");
    return FIBER_OK;
}

// ---- sampling on the device (src/sampler.c:48-112) ---------------------------------------

// Fills p.k / p.inv_temp and the shared-memory size; 0 or a FIBER_E* status.
static int sample_setup(SampleParams &p, int vocab, float temperature, int top_k, float top_p, size_t *smem) {
    int k = top_k > 0 ? top_k : vocab;
    if (k > vocab) k = vocab;
    if (k < vocab && k > SMP_MAX_K)
        return set_err(FIBER_EUNSUPPORTED, "device sampler: top_k %d above %d (use the host sampler)", k, SMP_MAX_K);
    if (k == vocab && vocab > SMP_MAX_UNSORTED)
        return set_err(FIBER_EUNSUPPORTED, "device sampler: unsorted top_k over a vocabulary above %d", SMP_MAX_UNSORTED);
    p.k = k;
    p.inv_temp = 1.0f / temperature;
    p.top_p = top_p;
    p.vocab = vocab;
    *smem = k < vocab ? (size_t)SMP_MAX_K * 12 : (size_t)vocab * 4;
    return FIBER_OK;
}

static cudaError_t launch_sample(const SampleParams &p, size_t smem, cudaStream_t st) {
    cudaError_t e = cudaFuncSetAttribute(sample_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    sample_rows_kernel<<<p.rows, SMP_THREADS, smem, st>>>(p);
    return cudaGetLastError();
}

static bool greedy_temperature(float t) { return t <= 0.0f || t < 1e-6f; }

extern "C" int fiber_sample(const float *d_logits, int rows, int vocab, int ld, float temperature, int top_k,
                            float top_p, unsigned long long *d_rng, int32_t *d_out, void *stream) {
    if (!d_logits || !d_out || rows <= 0 || vocab <= 0 || ld < vocab)
        return set_err(FIBER_EARG, "fiber_sample: bad arguments");
    cudaStream_t st = (cudaStream_t)stream;
    if (greedy_temperature(temperature)) {  // the reference's argmax (first maximum)
        argmax_rows_kernel<<<rows, 256, 0, st>>>(d_logits, vocab, ld, d_out);
        CK(cudaGetLastError());
        return FIBER_OK;
    }
    if (!d_rng) return set_err(FIBER_EARG, "fiber_sample: no random state");
    SampleParams p;
    memset(&p, 0, sizeof(p));
    size_t smem = 0;
    int rc = sample_setup(p, vocab, temperature, top_k, top_p, &smem);
    if (rc) return rc;
    p.logits = d_logits;
    p.ld = ld;
    p.rows = rows;
    p.rng = d_rng;
    p.out = d_out;
    CK(launch_sample(p, smem, st));
    return FIBER_OK;
}

extern "C" int fiber_decode_sample(fiber_ctx_t *c, kv_cache_t *kv, int32_t first_token, int start_pos, int n_steps,
                                   float temperature, int top_k, float top_p, unsigned long long *rng_state,
                                   int32_t *h_tokens_out, float *ms_out) {
    if (!c || !rng_state) return set_err(FIBER_EARG, "fiber_decode_sample: bad arguments");
    if (greedy_temperature(temperature))
        return fiber_decode_greedy(c, kv, first_token, start_pos, n_steps, h_tokens_out, ms_out);
    if (n_steps <= 0) return set_err(FIBER_EARG, "fiber_decode_sample: bad arguments");
    int rc = check_kv(c, kv);
    if (rc) return rc;
    const int lim = c->max_seq < kv->max_seq ? c->max_seq : kv->max_seq;
    if (start_pos < 0 || start_pos + n_steps > lim)
        return set_err(FIBER_EARG, "decode of %d steps from %d exceeds max_seq %d", n_steps, start_pos, lim);
    if (first_token < 0 || first_token >= (int)c->p.vocab_size)
        return set_err(FIBER_EARG, "token %d out of range", first_token);
    SampleParams sp;
    memset(&sp, 0, sizeof(sp));
    size_t smem = 0;
    if ((rc = sample_setup(sp, (int)c->p.vocab_size, temperature, top_k, top_p, &smem))) return rc;
    CK(cudaSetDevice(c->device));
    if (!c->smp_rng) {
        CK(cudaMalloc(&c->smp_rng, sizeof(unsigned long long)));
        CK(cudaMalloc(&c->smp_out, sizeof(int32_t)));
    }
    sp.logits = c->logits;
    sp.ld = (int)c->p.vocab_size;
    sp.rows = 1;
    sp.rng = c->smp_rng;
    sp.out = c->smp_out;
    sp.adv_token = &c->io->token;
    sp.adv_pos = &c->io->pos;
    sp.rec = c->rec;
    sp.rec_step = &c->io->step;
    c->h_io->token = first_token;
    c->h_io->pos = start_pos;
    c->h_io->step = 0;
    c->h_io->err = 0;
    CK(cudaMemcpyAsync(c->io, c->h_io, sizeof(StepIO), cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(c->smp_rng, rng_state, sizeof(unsigned long long), cudaMemcpyHostToDevice, c->stream));
    if (!use_flow(c) && !use_pk(c)) {  // build the step graph before the timed region
        cudaGraphExec_t g;
        if ((rc = get_graph(c, kv, false, &g)) != FIBER_OK) return rc;
    }
    CK(cudaEventRecord(c->ev0, c->stream));
    for (int i = 0; i < n_steps; i++) {
        if ((rc = run_step(c, kv, false)) != FIBER_OK) return rc;  // logits of io->token at io->pos
        CK(launch_sample(sp, smem, c->stream));                    // next token, position + 1
    }
    CK(cudaEventRecord(c->ev1, c->stream));
    CK(cudaEventSynchronize(c->ev1));
    if (ms_out) CK(cudaEventElapsedTime(ms_out, c->ev0, c->ev1));
    CK(cudaMemcpyAsync(c->h_io, c->io, sizeof(StepIO), cudaMemcpyDeviceToHost, c->stream));
    if (h_tokens_out) CK(cudaMemcpyAsync(h_tokens_out, c->rec, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaMemcpyAsync(rng_state, c->smp_rng, sizeof(unsigned long long), cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    return device_status(c);
}

extern "C" int fiber_tp_collective(fiber_ctx_t *c) {
    if (!c) return set_err(FIBER_EARG, "no context");
    if (c->tp_world <= 1) return 0;
    if (c->mode == 2 && c->fl_ok) return 3;  // fused: peer stores in the dataflow step's residual phases
    return c->ar_ok ? 2 : 1;
}

extern "C" int fiber_set_max_batch(fiber_ctx_t *c, int max_batch) {
    if (!c || max_batch < 1 || max_batch > FIBER_MAX_BATCH)
        return set_err(FIBER_EARG, "fiber_set_max_batch: max_batch outside [1, %d]", FIBER_MAX_BATCH);
    if (c->pf_cap) return set_err(FIBER_EARG, "fiber_set_max_batch: the batched buffers already exist");
    if (max_batch > 1 && !batched_ok(c))
        return set_err(FIBER_EUNSUPPORTED, "batched decode does not cover this model");
    c->max_batch = max_batch;
    return FIBER_OK;
}

