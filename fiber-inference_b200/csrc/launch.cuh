// launch.cuh — kernel launches with programmatic dependent launch (PDL).
//
// Every decode kernel is launched with programmatic stream serialization, so the
// next kernel's CTAs may be scheduled while the current one runs and can do
// their input-independent prologue (barrier set-up, weight TMA) early; each
// kernel's pdl_wait() restores the stream order for everything that touches
// activations. Captured into CUDA graphs as programmatic edges. Setting the
// environment variable FIBER_NO_PDL=1 launches without the attribute.
#pragma once
#include <cuda_runtime.h>
#include <stdlib.h>

#include <utility>

namespace fiber {

inline bool pdl_enabled() {
    static const int on = [] {
        const char *e = getenv("FIBER_NO_PDL");
        return (e && e[0] == '1') ? 0 : 1;
    }();
    return on != 0;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace fiber
