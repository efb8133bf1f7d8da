// Gated DeltaNet token mixer of the hybrid (Qwen3.5-style) decoder, fused: the causal
// depthwise conv (+ SiLU) of the q/k/v channels, L2-normalized q and k, the gated
// delta-rule recurrence on the head's state S [KD, VD] and the gated RMSNorm.
//
// Reference: crates/engine/src/shaders/deltanet.wgsl:80-160 (one workgroup per head,
// thread j owns column j of S in registers and output dim j; tokens of a step in
// order).  Per token: decay = exp(neg_a * softplus(a + dt_bias)), beta = sigmoid(b),
//   delta = (v - decay S^T k) beta,  o = decay S^T q + delta (k . q),
//   S <- decay S + k delta^T,        o <- o / rms(o) * gate_norm * silu(z).
// State (conv window and S) in three slots, the current one in params[3]; without
// spec it is updated in place, with spec (draft verification) the state after token m
// goes to slot (slot + 1 + m) % 3.
//
// B200 view: the state is 64 KB of f32 per head, read and written once per step with
// coalesced loads (thread j reads column j, consecutive threads consecutive floats),
// held in 128 registers a thread across the step's tokens; the two reductions per
// token (|q|^2 and |k|^2 together, then |o|^2) are warp shuffles plus one exchange of
// four warp partials in shared memory.  The projection row comes from the previous
// kernel, so it is read with coherent loads after the dependency wait.
#include "common.cuh"
#include "launch.cuh"

namespace w4a8 {

namespace {

constexpr int kKD = 128, kVD = 128;

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

// Sum over the CTA's 128 threads of (a, b); every thread gets the totals.
__device__ __forceinline__ float2 cta_sum2(float a, float b, float2* red) {
    for (int off = 16; off > 0; off >>= 1) {
        a += __shfl_xor_sync(kFull, a, off);
        b += __shfl_xor_sync(kFull, b, off);
    }
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[warp] = make_float2(a, b);
    __syncthreads();
    const float2 r = make_float2((red[0].x + red[1].x) + (red[2].x + red[3].x), (red[0].y + red[1].y) + (red[2].y + red[3].y));
    __syncthreads();  // red is reused by the next call
    return r;
}

__global__ void __launch_bounds__(kVD) deltanet_kernel(const float* proj, const float4* conv_w, float* conv_state,
                                                       float* state, float* out, const float* neg_a,
                                                       const float* dt_bias, const float* gate_norm,
                                                       const uint32_t* params, int NH, int m, float eps, int spec) {
    __shared__ float qs[kKD], ks[kKD];
    __shared__ float2 red[4];
    pdl_launch_dependents();
    pdl_wait();
    const int h = blockIdx.x, j = threadIdx.x;
    const int C = NH * (2 * kKD + kVD);
    const int row_len = C + NH * kVD + 2 * NH;
    const size_t slot_size = static_cast<size_t>(NH) * kKD * kVD;
    const size_t sb = static_cast<size_t>(h) * kKD * kVD + j;
    const int cq = h * kKD + j, ck = NH * kKD + h * kKD + j, cv = 2 * NH * kKD + h * kVD + j;
    const uint32_t slot = ld_dep(params + 3) % 3u;

    float s[kKD];
#pragma unroll
    for (int i = 0; i < kKD; ++i) s[i] = ld_dep(state + slot * slot_size + sb + static_cast<size_t>(i) * kVD);
    auto load_win = [&](int c) {
        const float* b = conv_state + (static_cast<size_t>(slot) * C + c) * 3;
        return make_float3(ld_dep(b), ld_dep(b + 1), ld_dep(b + 2));
    };
    float3 wq = load_win(cq), wk = load_win(ck), wv = load_win(cv);
    const float4 tq = __ldg(conv_w + cq), tk = __ldg(conv_w + ck), tv = __ldg(conv_w + cv);
    auto conv = [](float3& w, float4 t, float x) {
        const float y = silu_f(t.x * w.x + t.y * w.y + t.z * w.z + t.w * x);
        w = make_float3(w.y, w.z, x);
        return y;
    };
    auto store = [&](uint32_t sl) {
#pragma unroll
        for (int i = 0; i < kKD; ++i) state[sl * slot_size + sb + static_cast<size_t>(i) * kVD] = s[i];
        const float3 ws[3] = {wq, wk, wv};
        const int cs[3] = {cq, ck, cv};
        for (int u = 0; u < 3; ++u) {
            float* b = conv_state + (static_cast<size_t>(sl) * C + cs[u]) * 3;
            b[0] = ws[u].x;
            b[1] = ws[u].y;
            b[2] = ws[u].z;
        }
    };
    const float na = __ldg(neg_a + h), dtb = __ldg(dt_bias + h), gn = __ldg(gate_norm + j);

    for (int mt = 0; mt < m; ++mt) {
        const float* row = proj + static_cast<size_t>(mt) * row_len;
        float q = conv(wq, tq, ld_dep(row + cq));
        float k = conv(wk, tk, ld_dep(row + ck));
        const float v = conv(wv, tv, ld_dep(row + cv));
        const float2 n = cta_sum2(q * q, k * k, red);
        q *= rsqrtf(n.x + 1e-6f) * rsqrtf(static_cast<float>(kKD));
        k *= rsqrtf(n.y + 1e-6f);
        qs[j] = q;
        ks[j] = k;
        __syncthreads();

        const float b = ld_dep(row + C + NH * kVD + h);
        const float a = ld_dep(row + C + NH * kVD + NH + h) + dtb;
        const float sp = a > 20.0f ? a : logf(1.0f + expf(a));
        const float decay = expf(na * sp);
        const float beta = 1.0f / (1.0f + expf(-b));
        float sk = 0.0f, sq = 0.0f, kq = 0.0f;
#pragma unroll
        for (int i = 0; i < kKD; ++i) {
            sk += s[i] * ks[i];
            sq += s[i] * qs[i];
            kq += ks[i] * qs[i];
        }
        const float delta = (v - decay * sk) * beta;
        float o = decay * sq + delta * kq;
        const volatile float* ksv = ks;  // read again: holding all 128 values across both loops would spill
#pragma unroll
        for (int i = 0; i < kKD; ++i) s[i] = decay * s[i] + ksv[i] * delta;

        const float z = ld_dep(row + C + h * kVD + j);
        const float ms = cta_sum2(o * o, 0.0f, red).x / static_cast<float>(kVD);
        o *= rsqrtf(ms + eps) * gn * silu_f(z);
        out[static_cast<size_t>(mt) * NH * kVD + h * kVD + j] = o;
        if (spec) store((slot + 1u + static_cast<uint32_t>(mt)) % 3u);
        __syncthreads();  // qs / ks are rewritten by the next token
    }
    if (!spec) store(slot);
}

}  // namespace
}  // namespace w4a8

using namespace w4a8;

extern "C" {

W4A8_API w4a8_status w4a8_deltanet(const float* proj, const float* conv_w, float* conv_state, float* state, float* out,
                                   const float* neg_a, const float* dt_bias, const float* gate_norm,
                                   const uint32_t* params, int32_t nh, int32_t m, float eps, int32_t spec,
                                   void* stream) {
    if (!proj || !conv_w || !conv_state || !state || !out || !neg_a || !dt_bias || !gate_norm || !params)
        return set_error(W4A8_EINVAL, "w4a8_deltanet: NULL pointer");
    if (nh < 1 || nh > 1024) return set_error(W4A8_EINVAL, "w4a8_deltanet: heads %d", nh);
    if (m < 1 || m > W4A8_GEMV_MAX_M) return set_error(W4A8_EINVAL, "w4a8_deltanet: m=%d", m);
    if (reinterpret_cast<uintptr_t>(conv_w) & 15) return set_error(W4A8_EINVAL, "w4a8_deltanet: conv_w not 16-byte aligned");
    return launch_pdl("w4a8_deltanet", deltanet_kernel, dim3(nh), dim3(kVD), 0, static_cast<cudaStream_t>(stream), proj,
                      reinterpret_cast<const float4*>(conv_w), conv_state, state, out, neg_a, dt_bias, gate_norm, params,
                      static_cast<int>(nh), static_cast<int>(m), eps, static_cast<int>(spec != 0));
}

}  // extern "C"
