// Kernel launch with programmatic dependent launch enabled, so a kernel's CTAs may
// be scheduled while the previous kernel in the stream drains (its griddepcontrol
// wait still orders every read of that kernel's output).
#pragma once

#include "common.cuh"

namespace w4a8 {

// Set to 0 by w4a8_set_pdl(0) (for A/B timing); read at every launch.
extern int g_use_pdl;

template <typename Kernel, typename... Args>
w4a8_status launch_pdl(const char* what, Kernel kernel, dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = g_use_pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
    if (e != cudaSuccess) return set_error(W4A8_ECUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
    return W4A8_OK;
}

}  // namespace w4a8
