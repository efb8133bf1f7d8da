// Instantiation and launch of the GEMV family for one (group, has_min) pair; each
// gemv_g*_m*.cu includes this once so the instantiations compile in parallel.
#pragma once

#include "gemv.cuh"
#include "launch.cuh"

namespace w4a8 {

template <int G, bool HAS_MIN, int ACT, int MODE, int OUT>
w4a8_status launch_gemv_mt(const GemvParams& p, int nwarps, int grid, cudaStream_t st) {
    const dim3 g(grid), b(nwarps * 32);
    const char* what = "w4a8 gemv";
    if (p.m <= 1) return launch_pdl(what, gemv_kernel<G, HAS_MIN, ACT, MODE, 1, OUT>, g, b, 0, st, p);
    if (p.m <= 2) return launch_pdl(what, gemv_kernel<G, HAS_MIN, ACT, MODE, 2, OUT>, g, b, 0, st, p);
    if (p.m <= 4) return launch_pdl(what, gemv_kernel<G, HAS_MIN, ACT, MODE, 4, OUT>, g, b, 0, st, p);
    if (p.m <= 8) return launch_pdl(what, gemv_kernel<G, HAS_MIN, ACT, MODE, 8, OUT>, g, b, 0, st, p);
    return launch_pdl(what, gemv_kernel<G, HAS_MIN, ACT, MODE, 16, OUT>, g, b, 0, st, p);
}

template <int G, bool HAS_MIN>
w4a8_status launch_gemv_gh(const GemvParams& p, int act, int mode, int out, int nwarps, int grid,
                           cudaStream_t st) {
    if (out == OUT_DOTS) return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_TOKEN, W4A8_STORE, OUT_DOTS>(p, nwarps, grid, st);
    if (act == W4A8_ACT_TOKEN) {
        if (out == OUT_ARGMAX) return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_TOKEN, W4A8_STORE, OUT_ARGMAX>(p, nwarps, grid, st);
        if (mode == W4A8_STORE) return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_TOKEN, W4A8_STORE, OUT_Y>(p, nwarps, grid, st);
        if (mode == W4A8_ADD) return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_TOKEN, W4A8_ADD, OUT_Y>(p, nwarps, grid, st);
        return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_TOKEN, W4A8_SWIGLU, OUT_Y>(p, nwarps, grid, st);
    }
    if (out == OUT_ARGMAX) return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_GROUP32, W4A8_STORE, OUT_ARGMAX>(p, nwarps, grid, st);
    if (mode == W4A8_STORE) return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_GROUP32, W4A8_STORE, OUT_Y>(p, nwarps, grid, st);
    if (mode == W4A8_ADD) return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_GROUP32, W4A8_ADD, OUT_Y>(p, nwarps, grid, st);
    return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_GROUP32, W4A8_SWIGLU, OUT_Y>(p, nwarps, grid, st);
}

}  // namespace w4a8
