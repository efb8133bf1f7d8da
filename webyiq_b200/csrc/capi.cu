// The extern "C" boundary (include/w4a8.h): argument validation, launch-shape
// choice and dispatch.  Validation mirrors the reference's host checks
// (graph.rs:362-380 shape guards, manifest.rs:82 quant check) and adds the
// alignment rules of the 16-byte vector loads.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "gemv.cuh"
#include "launch.cuh"
#include "xchg.cuh"

namespace w4a8 {

int g_use_pdl = 1;
int g_use_mma = 1;
int g_use_tc_gemm = 1;

namespace {
thread_local char t_err[512] = "";
}  // namespace

int current_device(const char* what) {
    int dev = -1;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        set_error(W4A8_ECUDA, "%s: cudaGetDevice: %s", what, cudaGetErrorString(e));
        return -1;
    }
    if (dev < 0 || dev >= kMaxDevices) {
        set_error(W4A8_ECUDA, "%s: device %d beyond the library's %d", what, dev, kMaxDevices);
        return -1;
    }
    return dev;
}

// SMs of the current device, read once per device (benign race: every thread that
// reads it first stores the same value).
int sm_count() {
    static std::atomic<int> counts[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
    int n = counts[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        counts[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

w4a8_status set_error(w4a8_status st, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof(t_err), fmt, ap);
    va_end(ap);
    return st;
}

w4a8_status check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(W4A8_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    return W4A8_OK;
}

w4a8_status launch_gemv_g32_m0(const GemvParams&, int, int, int, cudaStream_t);
w4a8_status launch_gemv_g32_m1(const GemvParams&, int, int, int, cudaStream_t);
w4a8_status launch_gemv_g128_m0(const GemvParams&, int, int, int, cudaStream_t);
w4a8_status launch_gemv_g128_m1(const GemvParams&, int, int, int, cudaStream_t);
w4a8_status launch_quant(const float*, const float*, float, int, int, int, int8_t*, float*, cudaStream_t);
w4a8_status launch_argmax(const float*, int, int, const uint32_t*, uint32_t*, cudaStream_t);

w4a8_status launch_gemv_mma(const GemvParams& g, bool has_min, int mode, int out, cudaStream_t st);
bool gemv_dec_covers(const GemvParams& g, int group, int act, int mode, int out);
w4a8_status launch_gemv_dec(const GemvParams& g, bool has_min, int mode, cudaStream_t st);
bool lmhead_stream_covers(const GemvParams& g, int group, int act);
w4a8_status lmhead_argmax_impl(const w4a8_weight* w, int32_t row_offset, const int8_t* xq, const float* xs,
                               int32_t act, int32_t m, float* logits, uint64_t* best_key, uint32_t* tok_out,
                               const uint32_t* ids, void* workspace, size_t workspace_bytes, void* stream,
                               const XchgArgs* x, bool* fused);
w4a8_status launch_lmhead_stream(const GemvParams& g, bool has_min, cudaStream_t st);
w4a8_status device_error(unsigned int* code, cudaStream_t st);
w4a8_status selftest_wait_timeout(cudaStream_t st);
w4a8_status launch_gemm_tc(const w4a8_weight* w, const int8_t* xq, const float* dx, int m, int mode, float* y,
                           int* dots, cudaStream_t st);

// The formats the tcgen05 GEMM covers: group-128 symmetric weights, per-token dx.
bool tc_gemm_format(const w4a8_weight* w, int act) {
    return w->group == 128 && !w->has_min && act == W4A8_ACT_TOKEN && w->k % 128 == 0;
}

// Group-128 weights with per-token activations go to the tensor-core GEMV;
// everything else (the engine's group-32 format, per-32 activations) to the dp4a one.
w4a8_status launch_gemv(const GemvParams& p, int group, bool has_min, int act, int mode, int out, cudaStream_t st) {
    // The group-128 per-token lm_head argmax streams the vocabulary through its own
    // kernel (lmhead_stream.cu); the tensor-core GEMV takes the other group-128
    // per-token calls, the dp4a GEMV everything else.
    if (out == OUT_ARGMAX && g_use_mma && lmhead_stream_covers(p, group, act))
        return launch_lmhead_stream(p, has_min, st);
    // One or two tokens into y whose rows fit the decode GEMV (gemv_dec.cu) go there.
    if (g_use_mma && gemv_dec_covers(p, group, act, mode, out)) return launch_gemv_dec(p, has_min, mode, st);
    if (group == 128 && (act == W4A8_ACT_TOKEN || out == OUT_DOTS) && out != OUT_ARGMAX && g_use_mma)
        return launch_gemv_mma(p, has_min, mode, out, st);
    if (group == 32) return has_min ? launch_gemv_g32_m1(p, act, mode, out, st) : launch_gemv_g32_m0(p, act, mode, out, st);
    return has_min ? launch_gemv_g128_m1(p, act, mode, out, st) : launch_gemv_g128_m0(p, act, mode, out, st);
}

// Argument checks shared by every entry point that takes a weight or activations.
w4a8_status check_weight(const w4a8_weight* w, const char* what) {
    if (!w) return set_error(W4A8_EINVAL, "%s: weight is NULL", what);
    if (!w->q || !w->s) return set_error(W4A8_EINVAL, "%s: weight pointers are NULL", what);
    if (w->group != 32 && w->group != 128)
        return set_error(W4A8_EINVAL, "%s: group %d unsupported (32 or 128)", what, w->group);
    if (w->k <= 0 || w->k % w->group != 0)
        return set_error(W4A8_EINVAL, "%s: k=%d is not a positive multiple of group %d", what, w->k, w->group);
    if (w->n <= 0) return set_error(W4A8_EINVAL, "%s: n=%d", what, w->n);
    if (!aligned(w->q, 16)) return set_error(W4A8_EINVAL, "%s: q not 16-byte aligned", what);
    if (!aligned(w->s, 4)) return set_error(W4A8_EINVAL, "%s: s not 4-byte aligned", what);
    return W4A8_OK;
}

w4a8_status check_act(const int8_t* xq, const float* xs, int act, const char* what) {
    if (!xq || !xs) return set_error(W4A8_EINVAL, "%s: activation pointers are NULL", what);
    if (act != W4A8_ACT_GROUP32 && act != W4A8_ACT_TOKEN)
        return set_error(W4A8_EINVAL, "%s: act=%d unknown", what, act);
    if (!aligned(xq, 16)) return set_error(W4A8_EINVAL, "%s: xq not 16-byte aligned", what);
    if (!aligned(xs, act == W4A8_ACT_GROUP32 ? 8 : 4)) return set_error(W4A8_EINVAL, "%s: xs misaligned", what);
    return W4A8_OK;
}

}  // namespace w4a8

using namespace w4a8;

extern "C" {

const char* w4a8_last_error(void) { return t_err; }

const char* w4a8_version(void) { return "webyiq-b200 w4a8 0.1 (sm_100a)"; }

void w4a8_set_pdl(int enable) { g_use_pdl = enable ? 1 : 0; }

void w4a8_set_gemv_kernel(int tensor_core) { g_use_mma = tensor_core ? 1 : 0; }

void w4a8_set_gemm_kernel(int tensor_core) { g_use_tc_gemm = tensor_core ? 1 : 0; }

w4a8_status w4a8_device_error(uint32_t* code, void* stream) {
    return device_error(code, static_cast<cudaStream_t>(stream));
}

w4a8_status w4a8_selftest_wait_timeout(void* stream) {
    return selftest_wait_timeout(static_cast<cudaStream_t>(stream));
}

w4a8_status w4a8_weight_view(const void* q, const void* s, int32_t n, int32_t k, int32_t group, int32_t has_min,
                             w4a8_weight* out) {
    if (!out) return set_error(W4A8_EINVAL, "w4a8_weight_view: out is NULL");
    w4a8_weight w{q, s, n, k, group, has_min ? 1 : 0};
    const w4a8_status st = check_weight(&w, "w4a8_weight_view");
    if (st != W4A8_OK) return st;
    *out = w;
    return W4A8_OK;
}

w4a8_status w4a8_quant(const float* x, const float* norm_w, float eps, int32_t m, int32_t k, int32_t act, int8_t* xq,
                       float* xs, void* stream) {
    if (!x || !xq || !xs) return set_error(W4A8_EINVAL, "w4a8_quant: NULL pointer");
    if (m <= 0 || m > 65535 || k <= 0 || k % 32 != 0)
        return set_error(W4A8_EINVAL, "w4a8_quant: m=%d k=%d (need 1 <= m <= 65535, k %% 32 == 0)", m, k);
    if (act != W4A8_ACT_GROUP32 && act != W4A8_ACT_TOKEN) return set_error(W4A8_EINVAL, "w4a8_quant: act=%d", act);
    if (!aligned(x, 16) || (norm_w && !aligned(norm_w, 16)) || !aligned(xq, 16) || !aligned(xs, 8))
        return set_error(W4A8_EINVAL, "w4a8_quant: misaligned pointer");
    return launch_quant(x, norm_w, eps, m, k, act, xq, xs, static_cast<cudaStream_t>(stream));
}

w4a8_status w4a8_gemv(const w4a8_weight* w, const int8_t* xq, const float* xs, int32_t act, int32_t m, int32_t mode,
                      float* y, void* stream) {
    w4a8_status st = check_weight(w, "w4a8_gemv");
    if (st != W4A8_OK) return st;
    if ((st = check_act(xq, xs, act, "w4a8_gemv")) != W4A8_OK) return st;
    if (!y) return set_error(W4A8_EINVAL, "w4a8_gemv: y is NULL");
    if (m < 1 || m > W4A8_GEMV_MAX_M) return set_error(W4A8_EINVAL, "w4a8_gemv: m=%d not in [1, %d]", m, W4A8_GEMV_MAX_M);
    if (mode < W4A8_STORE || mode > W4A8_SWIGLU) return set_error(W4A8_EINVAL, "w4a8_gemv: mode=%d", mode);
    if (mode == W4A8_SWIGLU && w->n % 2) return set_error(W4A8_EINVAL, "w4a8_gemv: SWIGLU needs even n (%d)", w->n);
    GemvParams p{};
    p.q = static_cast<const uint4*>(w->q);
    p.s = w->s;
    p.xq = xq;
    p.xs = xs;
    p.y = y;
    p.n_out = mode == W4A8_SWIGLU ? w->n / 2 : w->n;
    p.y_stride = p.n_out;
    p.k = w->k;
    p.m = m;
    return launch_gemv(p, w->group, w->has_min != 0, act, mode, OUT_Y, static_cast<cudaStream_t>(stream));
}

w4a8_status w4a8_gemv_x(const w4a8_weight* w, const float* x, int32_t m, int32_t mode, float* y, void* stream) {
    w4a8_status st = check_weight(w, "w4a8_gemv_x");
    if (st != W4A8_OK) return st;
    if (w->group != 128) return set_error(W4A8_ENOTSUP, "w4a8_gemv_x: group-128 weights only (group %d)", w->group);
    if (!x || !aligned(x, 16)) return set_error(W4A8_EINVAL, "w4a8_gemv_x: x NULL or not 16-byte aligned");
    if (!y) return set_error(W4A8_EINVAL, "w4a8_gemv_x: y is NULL");
    if (m < 1 || m > W4A8_GEMV_MAX_M) return set_error(W4A8_EINVAL, "w4a8_gemv_x: m=%d not in [1, %d]", m, W4A8_GEMV_MAX_M);
    if (mode < W4A8_STORE || mode > W4A8_SWIGLU) return set_error(W4A8_EINVAL, "w4a8_gemv_x: mode=%d", mode);
    if (mode == W4A8_SWIGLU && w->n % 2) return set_error(W4A8_EINVAL, "w4a8_gemv_x: SWIGLU needs even n (%d)", w->n);
    GemvParams p{};
    p.q = static_cast<const uint4*>(w->q);
    p.s = w->s;
    p.xf32 = x;
    p.y = y;
    p.n_out = mode == W4A8_SWIGLU ? w->n / 2 : w->n;
    p.y_stride = p.n_out;
    p.k = w->k;
    p.m = m;
    if (g_use_mma && gemv_dec_covers(p, 128, W4A8_ACT_TOKEN, mode, OUT_Y))
        return launch_gemv_dec(p, w->has_min != 0, mode, static_cast<cudaStream_t>(stream));
    return launch_gemv_mma(p, w->has_min != 0, mode, OUT_Y, static_cast<cudaStream_t>(stream));
}

w4a8_status w4a8_gemv_xn(const w4a8_weight* w, const float* x, const float* norm_w, float eps, int32_t m, int32_t mode,
                         float* y, void* stream) {
    w4a8_status st = check_weight(w, "w4a8_gemv_xn");
    if (st != W4A8_OK) return st;
    if (w->group != 128) return set_error(W4A8_ENOTSUP, "w4a8_gemv_xn: group-128 weights only (group %d)", w->group);
    if (!x || !aligned(x, 16)) return set_error(W4A8_EINVAL, "w4a8_gemv_xn: x NULL or not 16-byte aligned");
    if (!norm_w || !aligned(norm_w, 16)) return set_error(W4A8_EINVAL, "w4a8_gemv_xn: norm_w NULL or not 16-byte aligned");
    if (!y) return set_error(W4A8_EINVAL, "w4a8_gemv_xn: y is NULL");
    if (m < 1 || m > 2) return set_error(W4A8_ENOTSUP, "w4a8_gemv_xn: m=%d (1 or 2 tokens)", m);
    if (mode < W4A8_STORE || mode > W4A8_SWIGLU) return set_error(W4A8_EINVAL, "w4a8_gemv_xn: mode=%d", mode);
    if (mode == W4A8_SWIGLU && w->n % 2) return set_error(W4A8_EINVAL, "w4a8_gemv_xn: SWIGLU needs even n (%d)", w->n);
    GemvParams p{};
    p.q = static_cast<const uint4*>(w->q);
    p.s = w->s;
    p.xf32 = x;
    p.norm_w = norm_w;
    p.eps = eps;
    p.y = y;
    p.n_out = mode == W4A8_SWIGLU ? w->n / 2 : w->n;
    p.y_stride = p.n_out;
    p.k = w->k;
    p.m = m;
    if (!gemv_dec_covers(p, 128, W4A8_ACT_TOKEN, mode, OUT_Y))
        return set_error(W4A8_ENOTSUP, "w4a8_gemv_xn: n=%d k=%d outside the decode kernel's plan", w->n, w->k);
    return launch_gemv_dec(p, w->has_min != 0, mode, static_cast<cudaStream_t>(stream));
}

w4a8_status w4a8_group_dots(const w4a8_weight* w, const int8_t* xq, int32_t m, int32_t* dots, void* stream) {
    w4a8_status st = check_weight(w, "w4a8_group_dots");
    if (st != W4A8_OK) return st;
    if (!xq || !dots || !aligned(xq, 16)) return set_error(W4A8_EINVAL, "w4a8_group_dots: bad xq/dots");
    if (m < 1 || m > W4A8_GEMV_MAX_M) return set_error(W4A8_EINVAL, "w4a8_group_dots: m=%d", m);
    GemvParams p{};
    p.q = static_cast<const uint4*>(w->q);
    p.s = w->s;
    p.xq = xq;
    p.dots = dots;
    p.n_out = w->n;
    p.y_stride = w->n;
    p.k = w->k;
    p.m = m;
    return launch_gemv(p, w->group, w->has_min != 0, W4A8_ACT_TOKEN, W4A8_STORE, OUT_DOTS,
                       static_cast<cudaStream_t>(stream));
}

w4a8_status w4a8_gemm(const w4a8_weight* w, const int8_t* xq, const float* xs, int32_t act, int32_t m, int32_t mode,
                      float* y, void* stream) {
    w4a8_status st = check_weight(w, "w4a8_gemm");
    if (st != W4A8_OK) return st;
    if ((st = check_act(xq, xs, act, "w4a8_gemm")) != W4A8_OK) return st;
    if (!y) return set_error(W4A8_EINVAL, "w4a8_gemm: y is NULL");
    if (m < 1) return set_error(W4A8_EINVAL, "w4a8_gemm: m=%d", m);
    if (mode < W4A8_STORE || mode > W4A8_SWIGLU) return set_error(W4A8_EINVAL, "w4a8_gemm: mode=%d", mode);
    if (mode == W4A8_SWIGLU && w->n % 2) return set_error(W4A8_EINVAL, "w4a8_gemm: SWIGLU needs even n (%d)", w->n);
    if (g_use_tc_gemm && tc_gemm_format(w, act)) {
        if (!aligned(y, 4)) return set_error(W4A8_EINVAL, "w4a8_gemm: y misaligned");
        return launch_gemm_tc(w, xq, xs, m, mode, y, nullptr, static_cast<cudaStream_t>(stream));
    }
    // Token blocks of up to 16 through the GEMV kernels.
    const int n_out = mode == W4A8_SWIGLU ? w->n / 2 : w->n;
    for (int t0 = 0; t0 < m; t0 += W4A8_GEMV_MAX_M) {
        const int mb = m - t0 < W4A8_GEMV_MAX_M ? m - t0 : W4A8_GEMV_MAX_M;
        const float* xsb = act == W4A8_ACT_TOKEN ? xs + t0 : xs + static_cast<size_t>(t0) * (w->k / 32) * 2;
        st = w4a8_gemv(w, xq + static_cast<size_t>(t0) * w->k, xsb, act, mb, mode, y + static_cast<size_t>(t0) * n_out,
                       stream);
        if (st != W4A8_OK) return st;
    }
    return W4A8_OK;
}

w4a8_status w4a8_gemm_group_dots(const w4a8_weight* w, const int8_t* xq, int32_t m, int32_t* dots, void* stream) {
    w4a8_status st = check_weight(w, "w4a8_gemm_group_dots");
    if (st != W4A8_OK) return st;
    if (!xq || !dots || !aligned(xq, 16) || !aligned(dots, 4))
        return set_error(W4A8_EINVAL, "w4a8_gemm_group_dots: bad xq/dots");
    if (m < 1) return set_error(W4A8_EINVAL, "w4a8_gemm_group_dots: m=%d", m);
    if (!tc_gemm_format(w, W4A8_ACT_TOKEN))
        return set_error(W4A8_ENOTSUP, "w4a8_gemm_group_dots: group-128 symmetric weights only");
    return launch_gemm_tc(w, xq, nullptr, m, W4A8_STORE, nullptr, dots, static_cast<cudaStream_t>(stream));
}

w4a8_status w4a8_matmul(const w4a8_weight* w, const int8_t* xq, const float* xs, int32_t act, int32_t m, int32_t mode,
                        float* y, void* stream) {
    if (m >= 1 && m <= W4A8_GEMV_MAX_M) return w4a8_gemv(w, xq, xs, act, m, mode, y, stream);
    return w4a8_gemm(w, xq, xs, act, m, mode, y, stream);
}

w4a8_status w4a8_argmax(const float* logits, int32_t m, int32_t v, const uint32_t* ids, uint32_t* tok_out,
                        void* stream) {
    if (!logits || !tok_out) return set_error(W4A8_EINVAL, "w4a8_argmax: NULL pointer");
    if (m < 1 || m > 65535 || v < 1) return set_error(W4A8_EINVAL, "w4a8_argmax: m=%d v=%d", m, v);
    return launch_argmax(logits, m, v, ids, tok_out, static_cast<cudaStream_t>(stream));
}

size_t w4a8_lmhead_workspace_bytes(int32_t n, int32_t m) {
    (void)n;
    (void)m;
    return 256;  // u32 counter at 0, u64 running keys at 128 (16 tokens)
}

w4a8_status w4a8_lmhead_argmax(const w4a8_weight* w, int32_t row_offset, const int8_t* xq, const float* xs,
                               int32_t act, int32_t m, float* logits, uint64_t* best_key, uint32_t* tok_out,
                               const uint32_t* ids, void* workspace, size_t workspace_bytes, void* stream) {
    return lmhead_argmax_impl(w, row_offset, xq, xs, act, m, logits, best_key, tok_out, ids, workspace,
                              workspace_bytes, stream, nullptr, nullptr);
}

}  // extern "C"

namespace w4a8 {

w4a8_status lmhead_argmax_impl(const w4a8_weight* w, int32_t row_offset, const int8_t* xq, const float* xs,
                               int32_t act, int32_t m, float* logits, uint64_t* best_key, uint32_t* tok_out,
                               const uint32_t* ids, void* workspace, size_t workspace_bytes, void* stream,
                               const XchgArgs* x, bool* fused) {
    w4a8_status st = check_weight(w, "w4a8_lmhead_argmax");
    if (st != W4A8_OK) return st;
    if ((st = check_act(xq, xs, act, "w4a8_lmhead_argmax")) != W4A8_OK) return st;
    if (!best_key) return set_error(W4A8_EINVAL, "w4a8_lmhead_argmax: best_key is NULL");
    if (m < 1 || m > W4A8_GEMV_MAX_M) return set_error(W4A8_EINVAL, "w4a8_lmhead_argmax: m=%d", m);
    if (row_offset < 0) return set_error(W4A8_EINVAL, "w4a8_lmhead_argmax: row_offset=%d", row_offset);
    if (!workspace || workspace_bytes < w4a8_lmhead_workspace_bytes(w->n, m) || !aligned(workspace, 16))
        return set_error(W4A8_EINVAL, "w4a8_lmhead_argmax: workspace NULL, small or misaligned");
    GemvParams p{};
    p.q = static_cast<const uint4*>(w->q);
    p.s = w->s;
    p.xq = xq;
    p.xs = xs;
    p.y = logits;
    p.counter = static_cast<unsigned int*>(workspace);
    p.ws_best = reinterpret_cast<unsigned long long*>(static_cast<char*>(workspace) + 128);
    p.best_key = reinterpret_cast<unsigned long long*>(best_key);
    p.ids = ids;
    p.n_out = w->n;
    p.y_stride = w->n;
    p.k = w->k;
    p.m = m;
    p.row_offset = row_offset;
    // with an exchange, the streaming kernel merges in its last CTA; any other
    // kernel leaves the shard's key and no token for the merge kernel
    const bool fuse = x && x->world > 0 && g_use_mma && lmhead_stream_covers(p, w->group, act);
    if (fused) *fused = fuse;
    p.xchg = fuse ? x : nullptr;
    p.tok_out = (x && !fuse) ? nullptr : tok_out;
    return launch_gemv(p, w->group, w->has_min != 0, act, W4A8_STORE, OUT_ARGMAX, static_cast<cudaStream_t>(stream));
}

}  // namespace w4a8
