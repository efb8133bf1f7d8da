// Activation quantization (optionally fused with RMSNorm) and the standalone argmax.
//
// quant: quant.wgsl:19-62.  One CTA of 256 threads per row (token).  Every float
// operation is spelled out (explicit _rn intrinsics, fixed reduction tree) so the
// CPU restatement in the oracle reproduces the output bit for bit:
//   sum of squares: thread t accumulates fma(x, x, acc) over its float4s in order
//   (x, y, z, w), elements t*4 + 1024*i; then a butterfly over the warp (xor 16..1);
//   then warp totals are added in warp order.
//   scale = 1 / sqrt(sum / k + eps); v = (x * scale) * norm_w.
//   per group (GROUP32) or per row (TOKEN): dx = amax / 127, inv = amax > 0 ? 1/dx : 0,
//   xq = rint(v * inv), xs = (dx, dx * sum xq) or dx.
// argmax: argmax.wgsl:14-43 with the packed-key reduction (common.cuh).
#include "launch.cuh"

namespace w4a8 {

constexpr int kQuantThreads = 256;

__device__ __forceinline__ float block_sum_fixed(float v, float* red) {
    // butterfly within the warp: every lane ends with the same bits
    for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(kFull, v, off));
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < kQuantThreads / 32; ++w) t = __fadd_rn(t, red[w]);
    __syncthreads();
    return t;
}

__device__ __forceinline__ float block_max(float v, float* red) {
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, off));
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < kQuantThreads / 32; ++w) t = fmaxf(t, red[w]);
    __syncthreads();
    return t;
}

template <bool NORM>
__device__ __forceinline__ void load8(const float* xr, const float* nw, int i, float scale, float e[8]) {
    const float4 a = ld_dep(reinterpret_cast<const float4*>(xr + i));
    const float4 b = ld_dep(reinterpret_cast<const float4*>(xr + i + 4));
    e[0] = a.x; e[1] = a.y; e[2] = a.z; e[3] = a.w;
    e[4] = b.x; e[5] = b.y; e[6] = b.z; e[7] = b.w;
    if (NORM) {
        const float4 na = __ldg(reinterpret_cast<const float4*>(nw + i));
        const float4 nb = __ldg(reinterpret_cast<const float4*>(nw + i + 4));
        const float n[8] = {na.x, na.y, na.z, na.w, nb.x, nb.y, nb.z, nb.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) e[j] = __fmul_rn(__fmul_rn(e[j], scale), n[j]);
    }
}

template <bool NORM, int ACT>
__global__ void __launch_bounds__(kQuantThreads) quant_kernel(const float* x, const float* __restrict__ nw,
                                                              float eps, int k, int8_t* __restrict__ xq,
                                                              float* __restrict__ xs) {
    __shared__ float red[kQuantThreads / 32];
    pdl_launch_dependents();
    pdl_wait();
    const int row = blockIdx.x;
    const float* xr = x + static_cast<size_t>(row) * k;
    const int tid = threadIdx.x;

    float scale = 1.0f;
    if (NORM) {
        float ss = 0.0f;
        for (int i = tid * 4; i < k; i += kQuantThreads * 4) {
            const float4 v = ld_dep(reinterpret_cast<const float4*>(xr + i));
            ss = __fmaf_rn(v.x, v.x, ss);
            ss = __fmaf_rn(v.y, v.y, ss);
            ss = __fmaf_rn(v.z, v.z, ss);
            ss = __fmaf_rn(v.w, v.w, ss);
        }
        const float tot = block_sum_fixed(ss, red);
        scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(k)), eps)));
    }

    // Each thread owns 8 consecutive inputs; 4 threads make a group of 32.
    float dx_tok = 0.0f, inv_tok = 0.0f;
    if (ACT == W4A8_ACT_TOKEN) {
        float amax = 0.0f;
        for (int i = tid * 8; i < k; i += kQuantThreads * 8) {
            float e[8];
            load8<NORM>(xr, nw, i, scale, e);
#pragma unroll
            for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(e[j]));
        }
        amax = block_max(amax, red);
        dx_tok = __fdiv_rn(amax, 127.0f);
        inv_tok = amax > 0.0f ? __fdiv_rn(1.0f, dx_tok) : 0.0f;
        if (tid == 0) xs[row] = dx_tok;
    }

    // k % 32 == 0, so a group's 4 threads are always all in range together; the
    // loop bound is uniform per quad.
    for (int i = tid * 8; i < ((k + 255) / 256) * 256; i += kQuantThreads * 8) {
        const bool in = i < k;
        float e[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (in) load8<NORM>(xr, nw, i, scale, e);
        float dx = dx_tok, inv = inv_tok;
        if (ACT == W4A8_ACT_GROUP32) {
            float amax = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(e[j]));
            amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 2));
            dx = __fdiv_rn(amax, 127.0f);
            inv = amax > 0.0f ? __fdiv_rn(1.0f, dx) : 0.0f;
        }
        int sum = 0;
        uint32_t packed[2] = {0u, 0u};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int qv = static_cast<int>(rintf(__fmul_rn(e[j], inv)));
            sum += qv;
            packed[j >> 2] |= (static_cast<uint32_t>(qv) & 0xffu) << (8 * (j & 3));
        }
        if (in) *reinterpret_cast<uint2*>(xq + static_cast<size_t>(row) * k + i) = make_uint2(packed[0], packed[1]);
        if (ACT == W4A8_ACT_GROUP32) {
            sum += __shfl_xor_sync(kFull, sum, 1);
            sum += __shfl_xor_sync(kFull, sum, 2);
            if (in && (tid & 3) == 0) {
                const size_t gi = static_cast<size_t>(row) * (k / 32) + i / 32;
                reinterpret_cast<float2*>(xs)[gi] = make_float2(dx, __fmul_rn(dx, static_cast<float>(sum)));
            }
        }
    }
}

w4a8_status launch_quant(const float* x, const float* nw, float eps, int m, int k, int act, int8_t* xq, float* xs,
                         cudaStream_t st) {
    const dim3 g(m), b(kQuantThreads);
    const char* what = "w4a8 quant";
    if (nw) {
        if (act == W4A8_ACT_TOKEN) return launch_pdl(what, quant_kernel<true, W4A8_ACT_TOKEN>, g, b, 0, st, x, nw, eps, k, xq, xs);
        return launch_pdl(what, quant_kernel<true, W4A8_ACT_GROUP32>, g, b, 0, st, x, nw, eps, k, xq, xs);
    }
    if (act == W4A8_ACT_TOKEN) return launch_pdl(what, quant_kernel<false, W4A8_ACT_TOKEN>, g, b, 0, st, x, nw, eps, k, xq, xs);
    return launch_pdl(what, quant_kernel<false, W4A8_ACT_GROUP32>, g, b, 0, st, x, nw, eps, k, xq, xs);
}

// ---------------------------------------------------------------------------
constexpr int kArgmaxThreads = 1024;

__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const float* logits, int v,
                                                                const uint32_t* __restrict__ ids,
                                                                uint32_t* __restrict__ tok_out) {
    __shared__ unsigned long long red[kArgmaxThreads / 32];
    pdl_launch_dependents();
    pdl_wait();
    const float* lr = logits + static_cast<size_t>(blockIdx.x) * v;
    unsigned long long key = 0;
    for (int i = threadIdx.x; i < v; i += kArgmaxThreads) {
        const unsigned long long kk = argmax_key(ld_dep(lr + i), static_cast<uint32_t>(i));
        key = kk > key ? kk : key;
    }
    for (int off = 16; off > 0; off >>= 1) {
        const unsigned long long o = shfl_xor_u64(key, off);
        key = o > key ? o : key;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = key;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kArgmaxThreads / 32; ++w) key = red[w] > key ? red[w] : key;
        const uint32_t idx = key ? ~static_cast<uint32_t>(key & 0xffffffffu) : 0u;
        tok_out[blockIdx.x] = ids ? __ldg(ids + idx) : idx;
    }
}

w4a8_status launch_argmax(const float* logits, int m, int v, const uint32_t* ids, uint32_t* tok_out, cudaStream_t st) {
    return launch_pdl("w4a8 argmax", argmax_kernel, dim3(m), dim3(kArgmaxThreads), 0, st, logits, v, ids, tok_out);
}

}  // namespace w4a8
