// noalloc.cu — greedy lm_head step (GEMV + argmax) that allocates no device memory.
//
// The regular decode path keeps the argmax kernel's cross-CTA scratch (one
// (value, index) pair per CTA plus a merge ticket) in buffers that
// fiber_cuda_init obtains with cudaMalloc. Some callers cannot allocate at the
// point where they want to run this step: a host application that hands all
// device memory to its own pool up front and forbids further cudaMalloc, or a
// latency-critical loop where cudaMalloc's implicit device synchronization and
// unbounded latency are not acceptable. For them this file keeps that scratch
// in a fixed file-scope device array instead; the caller still passes the
// weights, the input vector and the two outputs.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "fiber_cuda.h"
#include "gemv.cuh"

using namespace fiber;

void fiber_set_error_message(const char *msg);  // fiber_cuda.cu

namespace {

constexpr int NA_ROWS = 2;                       // rows per warp, as in the decode path
constexpr int NA_TILE = NA_ROWS * GEMV_WARPS;    // rows per CTA
constexpr int NA_MAX_CTAS = FIBER_NOALLOC_MAX_ROWS / NA_TILE;
constexpr size_t NA_PART_BYTES = (size_t)NA_MAX_CTAS * sizeof(float2);  // multiple of 256
constexpr size_t NA_BYTES = NA_PART_BYTES + 256;                        // + merge ticket
static_assert(FIBER_NOALLOC_MAX_ROWS % NA_TILE == 0, "row limit must be whole CTAs");
static_assert(NA_PART_BYTES % 256 == 0, "ticket must stay 256-byte aligned");

// Shared by every call on a device; holds the last call's contents until exit.
static __device__ __align__(256) unsigned char g_scratch[NA_BYTES];

constexpr int NA_MAX_DEVICES = 64;
std::mutex g_mu;
unsigned char *g_addr[NA_MAX_DEVICES];  // device address of g_scratch, per device

thread_local char g_msg[256];

int fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    fiber_set_error_message(g_msg);
    return code;
}

// The host-side name g_scratch is only a stand-in; the kernel needs the device
// address, looked up once per device with that device current.
int scratch_for_current_device(unsigned char **out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(FIBER_ECUDA, "fiber_gemv_argmax_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= NA_MAX_DEVICES) return fail(FIBER_EARG, "fiber_gemv_argmax_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_scratch);
        if (e != cudaSuccess || !p)
            return fail(FIBER_ECUDA, "fiber_gemv_argmax_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        g_addr[dev] = static_cast<unsigned char *>(p);
    }
    *out = g_addr[dev];
    return FIBER_OK;
}

template <int T>
cudaError_t launch(const GemvParams &p, int grid, cudaStream_t st) {
    const size_t smem = (size_t)p.cols * sizeof(float);
    auto k = gemv_kernel<T, EPI_ARGMAX, NA_ROWS>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    k<<<grid, GEMV_THREADS, smem, st>>>(p);
    return cudaGetLastError();
}

}  // namespace

extern "C" int fiber_gemv_argmax_noalloc(int type, const void *d_w, const float *d_x, float *d_y,
                                         int32_t *d_argmax, int rows, int cols, void *stream) {
    if (!(type == T_Q4_K || type == T_Q5_K || type == T_Q6_K || type == T_F16))
        return fail(FIBER_EARG, "fiber_gemv_argmax_noalloc: type %d not supported", type);
    if (!d_w || !d_x || !d_y || !d_argmax || rows <= 0 || cols <= 0 || cols % 256)
        return fail(FIBER_EARG, "fiber_gemv_argmax_noalloc: bad shape %dx%d (cols must be a positive multiple of 256)",
                    rows, cols);
    if (rows > FIBER_NOALLOC_MAX_ROWS)
        return fail(FIBER_EARG, "fiber_gemv_argmax_noalloc: %d rows exceed the static scratch limit of %d rows",
                    rows, FIBER_NOALLOC_MAX_ROWS);
    if (((uintptr_t)d_w & 15) || ((uintptr_t)d_x & 15))
        return fail(FIBER_EARG, "fiber_gemv_argmax_noalloc: weights and x must be 16-byte aligned");
    unsigned char *scratch = nullptr;
    int rc = scratch_for_current_device(&scratch);
    if (rc != FIBER_OK) return rc;

    cudaStream_t st = (cudaStream_t)stream;
    unsigned int *ticket = reinterpret_cast<unsigned int *>(scratch + NA_PART_BYTES);
    // the merge ticket must start at zero; an interrupted earlier call could have left it set
    cudaError_t e = cudaMemsetAsync(ticket, 0, sizeof(unsigned int), st);
    if (e != cudaSuccess) return fail(FIBER_ECUDA, "fiber_gemv_argmax_noalloc: clearing ticket: %s", cudaGetErrorString(e));

    GemvParams p;
    memset(&p, 0, sizeof(p));
    p.seg[0] = {static_cast<const uint8_t *>(d_w), type, rows, 0};
    p.nseg = 1;
    p.tiles[0] = (rows + NA_TILE - 1) / NA_TILE;
    p.cols = cols;
    p.x = d_x;
    p.y = d_y;
    p.am_part = reinterpret_cast<float2 *>(scratch);
    p.am_count = ticket;
    p.am_out = d_argmax;
    const int grid = p.tiles[0];
    switch (type) {
    case T_Q4_K: e = launch<T_Q4_K>(p, grid, st); break;
    case T_Q5_K: e = launch<T_Q5_K>(p, grid, st); break;
    case T_Q6_K: e = launch<T_Q6_K>(p, grid, st); break;
    default: e = launch<T_F16>(p, grid, st); break;
    }
    if (e != cudaSuccess) return fail(FIBER_ECUDA, "fiber_gemv_argmax_noalloc: launch: %s", cudaGetErrorString(e));
    return FIBER_OK;
}
