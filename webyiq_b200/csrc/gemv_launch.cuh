// Instantiation and launch of the GEMV family for one (group, has_min) pair; each
// gemv_g*_m*.cu includes this once so the instantiations compile in parallel.
#pragma once

#include "gemv.cuh"
#include "launch.cuh"

namespace w4a8 {

int sm_count();  // capi.cu

// Launch plan: 2 CTAs per SM on balanced contiguous row ranges of at least 4
// rows (fewer CTAs when rows are scarce); T = a multiple of k/32 threads.
template <typename Kernel>
w4a8_status launch_gemv_kernel(Kernel kernel, FuncAttr& attr, GemvParams p, int group, int nr, cudaStream_t st) {
    const int kc = p.k / 32;
    if (kc > kGemvMaxKC) return set_error(W4A8_EINVAL, "w4a8 gemv: k=%d too large (max %d)", p.k, kGemvMaxKC * 32);
    const int threads = gemv_threads(kc);
    const size_t smem = gemv_smem_bytes(p.m, p.k, group, nr);
    if (smem > 48 * 1024) {  // `attr` belongs to this one kernel instantiation
        const w4a8_status a = ensure_smem(kernel, attr, smem, -1, "w4a8 gemv");
        if (a != W4A8_OK) return a;
    }
    const int sms = sm_count();
    int ctas = 2 * sms;
    if (ctas > (p.n_out + 3) / 4) ctas = (p.n_out + 3) / 4;
    if (ctas < 1) ctas = 1;
    return launch_pdl("w4a8 gemv", kernel, dim3(ctas), dim3(threads), smem, st, p);
}

template <int G, bool HAS_MIN, int ACT, int MODE, int MT, int OUT>
w4a8_status launch_gemv_inst(const GemvParams& p, cudaStream_t st) {
    static FuncAttr attr;  // dynamic smem this instantiation may use, per device
    return launch_gemv_kernel(gemv_kernel<G, HAS_MIN, ACT, MODE, MT, OUT>, attr, p, G,
                              MODE == W4A8_SWIGLU ? 2 : 1, st);
}

// Tokens go in blocks of up to kGemvMaxMT per launch (the weights stay in L2 for
// the later blocks).
template <int G, bool HAS_MIN, int ACT, int MODE, int OUT>
w4a8_status launch_gemv_mt(GemvParams p, cudaStream_t st) {
    const int m = p.m;
    const int kc = p.k / 32, kg = p.k / G;
    for (int t0 = 0; t0 < m; t0 += kGemvMaxMT) {
        GemvParams b = p;
        b.m = m - t0 < kGemvMaxMT ? m - t0 : kGemvMaxMT;
        b.xq = p.xq + static_cast<size_t>(t0) * p.k;
        b.xs = p.xs + (ACT == W4A8_ACT_TOKEN ? static_cast<size_t>(t0) : static_cast<size_t>(t0) * kc * 2);
        if (p.y) b.y = p.y + static_cast<size_t>(t0) * p.y_stride;
        if (p.dots) b.dots = p.dots + static_cast<size_t>(t0) * p.n_out * kg;
        if (p.ws_best) b.ws_best = p.ws_best + t0;
        if (p.best_key) b.best_key = p.best_key + t0;
        if (p.tok_out) b.tok_out = p.tok_out + t0;
        w4a8_status s;
        if (b.m == 1)
            s = launch_gemv_inst<G, HAS_MIN, ACT, MODE, 1, OUT>(b, st);
        else if (b.m == 2)
            s = launch_gemv_inst<G, HAS_MIN, ACT, MODE, 2, OUT>(b, st);
        else
            s = launch_gemv_inst<G, HAS_MIN, ACT, MODE, 4, OUT>(b, st);
        if (s != W4A8_OK) return s;
    }
    return W4A8_OK;
}

template <int G, bool HAS_MIN>
w4a8_status launch_gemv_gh(const GemvParams& p, int act, int mode, int out, cudaStream_t st) {
    if (out == OUT_DOTS) return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_TOKEN, W4A8_STORE, OUT_DOTS>(p, st);
    if (act == W4A8_ACT_TOKEN) {
        if (out == OUT_ARGMAX) return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_TOKEN, W4A8_STORE, OUT_ARGMAX>(p, st);
        if (mode == W4A8_STORE) return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_TOKEN, W4A8_STORE, OUT_Y>(p, st);
        if (mode == W4A8_ADD) return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_TOKEN, W4A8_ADD, OUT_Y>(p, st);
        return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_TOKEN, W4A8_SWIGLU, OUT_Y>(p, st);
    }
    if (out == OUT_ARGMAX) return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_GROUP32, W4A8_STORE, OUT_ARGMAX>(p, st);
    if (mode == W4A8_STORE) return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_GROUP32, W4A8_STORE, OUT_Y>(p, st);
    if (mode == W4A8_ADD) return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_GROUP32, W4A8_ADD, OUT_Y>(p, st);
    return launch_gemv_mt<G, HAS_MIN, W4A8_ACT_GROUP32, W4A8_SWIGLU, OUT_Y>(p, st);
}

}  // namespace w4a8
