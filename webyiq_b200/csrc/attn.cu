// Decode attention over an f16 KV cache, flash-decoding style, and the merge of its
// chunks into the int8 input of the o projection.
//
// Reference: crates/engine/src/shaders/attn.wgsl:41-115 (one workgroup per chunk of
// CH = 32 positions, kv head and token: scores of the GQ query heads sharing the kv
// head, a chunk-local softmax, the partial P V, written as (o[D], max, sum)) and
// attn_combine.wgsl:31-83 (per query head and token: the chunks merged, the optional
// sigmoid gate, then the per-32 int8 quantization of quant.wgsl).  Token m of a step
// sits at position pos + m (pos read on the device, so a captured graph replays for
// every position) and attends to positions 0 ..= pos + m; chunks past that exit at once.
//
// B200 view: decode attention reads the cache once per token (K and V, 4 bytes per
// position and dimension) and is HBM-bound; a CTA's K and V rows are read with
// 16-byte loads, each K row by the GQ threads of its position at once (one L1 line),
// and the query heads are staged once per CTA in padded shared-memory rows.  Both
// kernels start under programmatic dependent launch and read their inputs (q, the
// cache, the partials), which earlier kernels write, with coherent loads after the
// dependency wait.
#include <cuda_fp16.h>

#include "common.cuh"
#include "launch.cuh"

namespace w4a8 {

namespace {

constexpr int kCH = 32;           // positions per chunk (attn.wgsl CH)
constexpr int kAttnThreads = 256;

__device__ __forceinline__ float4 h4(uint2 u) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

__global__ void __launch_bounds__(kAttnThreads) attn_partial_kernel(const float* qkv, const uint2* kc, const uint2* vc,
                                                                   int H, int KVH, int D, int maxctx,
                                                                   const uint32_t* params, float* part) {
    extern __shared__ float sm[];
    pdl_launch_dependents();
    pdl_wait();
    const int gq = H / KVH, d4 = D / 4, qstride = D + 4;  // query rows padded by one float4
    const int chunk = blockIdx.x, kh = blockIdx.y % KVH, mt = blockIdx.y / KVH;
    const uint32_t pos = ld_dep(params);
    // positions 0 ..= pos + mt, never past the cache (a position at or past maxctx is
    // the caller's error; the reads stay inside the cache all the same)
    const int seq_len = min(static_cast<int>(min(pos, static_cast<uint32_t>(maxctx))) + mt + 1, maxctx);
    const int t0 = chunk * kCH;
    if (t0 >= seq_len) return;
    float* qs = sm;                         // [gq][D + 4]
    float* ps = qs + gq * qstride;          // [gq][CH]
    float* ms = ps + gq * kCH;              // [gq][2]
    const int tid = threadIdx.x;

    const float4* q4 = reinterpret_cast<const float4*>(qkv + (static_cast<size_t>(mt) * (H + 2 * KVH) + kh * gq) * D);
    for (int i = tid; i < gq * d4; i += kAttnThreads)
        *reinterpret_cast<float4*>(qs + (i / d4) * qstride + 4 * (i % d4)) = ld_dep(q4 + i);
    __syncthreads();

    // scores: consecutive threads share a position (its K row is read once into L1)
    // and differ in query head
    const float scale = rsqrtf(static_cast<float>(D));
    for (int e = tid; e < gq * kCH; e += kAttnThreads) {
        const int h = e % gq, tt = e / gq;
        float s = -3.0e38f;
        if (t0 + tt < seq_len) {
            const uint2* kr = kc + (static_cast<size_t>(kh) * maxctx + t0 + tt) * d4;
            const float* qh = qs + h * qstride;
            s = 0.0f;
            for (int i = 0; i < d4; ++i) {
                const float4 k = h4(ld_dep(kr + i));
                const float4 q = *reinterpret_cast<const float4*>(qh + 4 * i);
                s += q.x * k.x + q.y * k.y + q.z * k.z + q.w * k.w;
            }
            s *= scale;
        }
        ps[h * kCH + tt] = s;
    }
    __syncthreads();
    if (tid < gq) {
        float mx = -3.0e38f;
        for (int i = 0; i < kCH; ++i) mx = fmaxf(mx, ps[tid * kCH + i]);
        float l = 0.0f;
        for (int i = 0; i < kCH; ++i) l += expf(ps[tid * kCH + i] - mx);
        ms[2 * tid] = mx;
        ms[2 * tid + 1] = l;
    }
    __syncthreads();
    for (int e = tid; e < gq * kCH; e += kAttnThreads) ps[e] = expf(ps[e] - ms[2 * (e / kCH)]);
    __syncthreads();

    const int n = min(kCH, seq_len - t0);
    const int nch = maxctx / kCH;
    for (int e = tid; e < gq * d4; e += kAttnThreads) {
        const int h = e / d4, dv = e % d4;
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        const uint2* vb = vc + (static_cast<size_t>(kh) * maxctx + t0) * d4 + dv;
        for (int i = 0; i < n; ++i) {
            const float p = ps[h * kCH + i];
            const float4 v = h4(ld_dep(vb + static_cast<size_t>(i) * d4));
            acc.x += p * v.x;
            acc.y += p * v.y;
            acc.z += p * v.z;
            acc.w += p * v.w;
        }
        float* base = part + ((static_cast<size_t>(mt) * H + kh * gq + h) * nch + chunk) * (D + 2);
        base[4 * dv] = acc.x;
        base[4 * dv + 1] = acc.y;
        base[4 * dv + 2] = acc.z;
        base[4 * dv + 3] = acc.w;
        if (dv == 0) {
            base[D] = ms[2 * h];
            base[D + 1] = ms[2 * h + 1];
        }
    }
}

// One CTA per (query head, token), D / 2 threads: thread j owns dims 2j and 2j + 1.
__global__ void attn_combine_kernel(const float* part, int H, int KVH, int D, int maxctx, const uint32_t* params,
                                    const float* gsrc, int8_t* xq, float2* xs, float* o_out) {
    extern __shared__ float o[];  // [D] head output, then [D / 32] group scales
    float* gs = o + D;
    pdl_launch_dependents();
    pdl_wait();
    const int h = blockIdx.x, mt = blockIdx.y, lid = threadIdx.x;
    const int nch = maxctx / kCH;
    const uint32_t pos = min(ld_dep(params), static_cast<uint32_t>(maxctx));
    const int n = min((static_cast<int>(pos) + mt + kCH) / kCH, nch);  // chunks covering 0 ..= pos + mt
    const float* hb = part + (static_cast<size_t>(mt) * H + h) * nch * (D + 2);

    float mx = -3.0e38f;
    for (int c = 0; c < n; ++c) mx = fmaxf(mx, ld_dep(hb + static_cast<size_t>(c) * (D + 2) + D));
    float l = 0.0f, a0 = 0.0f, a1 = 0.0f;
    for (int c = 0; c < n; ++c) {
        const float* cb = hb + static_cast<size_t>(c) * (D + 2);
        const float w = expf(ld_dep(cb + D) - mx);
        l += w * ld_dep(cb + D + 1);
        const float2 pv = ld_dep(reinterpret_cast<const float2*>(cb) + lid);
        a0 += w * pv.x;
        a1 += w * pv.y;
    }
    a0 /= l;
    a1 /= l;
    if (gsrc) {
        const float2 g =
            ld_dep(reinterpret_cast<const float2*>(gsrc + static_cast<size_t>(mt) * 2 * (H + KVH) * D + h * 2 * D + D) + lid);
        a0 /= 1.0f + expf(-g.x);
        a1 /= 1.0f + expf(-g.y);
    }
    o[2 * lid] = a0;
    o[2 * lid + 1] = a1;
    if (o_out) reinterpret_cast<float2*>(o_out + (static_cast<size_t>(mt) * H + h) * D)[lid] = make_float2(a0, a1);
    __syncthreads();

    // the head's groups of 32 (quant.wgsl format): dx = amax / 127, xq = rint(o / dx)
    if (lid < D / 32) {
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(o[lid * 32 + i]));
        gs[lid] = __fdiv_rn(amax, 127.0f);
    }
    __syncthreads();
    if (lid < D / 32) {
        const float dx = gs[lid];
        const float inv = dx > 0.0f ? __fdiv_rn(1.0f, dx) : 0.0f;
        int8_t* dst = xq + (static_cast<size_t>(mt) * H + h) * D + lid * 32;
        int sum = 0;
        for (int i = 0; i < 32; i += 4) {
            int q[4];
            for (int u = 0; u < 4; ++u) {
                q[u] = static_cast<int>(rintf(__fmul_rn(o[lid * 32 + i + u], inv)));
                sum += q[u];
            }
            *reinterpret_cast<uint32_t*>(dst + i) = (static_cast<uint32_t>(q[0]) & 0xffu) |
                                                     ((static_cast<uint32_t>(q[1]) & 0xffu) << 8) |
                                                     ((static_cast<uint32_t>(q[2]) & 0xffu) << 16) |
                                                     ((static_cast<uint32_t>(q[3]) & 0xffu) << 24);
        }
        xs[(static_cast<size_t>(mt) * H + h) * (D / 32) + lid] = make_float2(dx, __fmul_rn(dx, static_cast<float>(sum)));
    }
}

w4a8_status check_attn(const char* what, int H, int KVH, int D, int maxctx, int m, const void* params) {
    if (H < 1 || KVH < 1 || H % KVH || H / KVH > 16)
        return set_error(W4A8_EINVAL, "%s: H=%d KVH=%d (query heads a multiple of the kv heads, at most 16 per kv head)",
                         what, H, KVH);
    if (D < 32 || D > 1024 || D % 32)
        return set_error(W4A8_EINVAL, "%s: head dim %d (a multiple of 32, at most 1024)", what, D);
    if (maxctx < kCH || maxctx % kCH) return set_error(W4A8_EINVAL, "%s: maxctx %d (a multiple of 32)", what, maxctx);
    if (m < 1 || m > W4A8_GEMV_MAX_M) return set_error(W4A8_EINVAL, "%s: m=%d", what, m);
    if (!params) return set_error(W4A8_EINVAL, "%s: NULL params", what);
    return W4A8_OK;
}

}  // namespace
}  // namespace w4a8

using namespace w4a8;

extern "C" {

W4A8_API w4a8_status w4a8_attn_decode(const float* qkv, const void* kc, const void* vc, int32_t H, int32_t KVH,
                                      int32_t D, int32_t maxctx, const uint32_t* params, int32_t m, int32_t chunks,
                                      float* part, void* stream) {
    const w4a8_status c = check_attn("w4a8_attn_decode", H, KVH, D, maxctx, m, params);
    if (c != W4A8_OK) return c;
    if (!qkv || !kc || !vc || !part) return set_error(W4A8_EINVAL, "w4a8_attn_decode: NULL pointer");
    if (((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc)) & 15) ||
        (reinterpret_cast<uintptr_t>(part) & 7))
        return set_error(W4A8_EINVAL, "w4a8_attn_decode: qkv, kc, vc must be 16-byte aligned, part 8-byte aligned");
    if (chunks < 1 || chunks > maxctx / kCH)
        return set_error(W4A8_EINVAL, "w4a8_attn_decode: chunks=%d (1 .. maxctx / 32)", chunks);
    static FuncAttr attr;
    const int gq = H / KVH;
    const size_t smem = (static_cast<size_t>(gq) * (D + 4) + gq * kCH + 2 * gq) * 4;
    const w4a8_status a = ensure_smem(attn_partial_kernel, attr, smem, -1, "w4a8_attn_decode");
    if (a != W4A8_OK) return a;
    return launch_pdl("w4a8_attn_decode", attn_partial_kernel, dim3(chunks, KVH * m), dim3(kAttnThreads), smem,
                      static_cast<cudaStream_t>(stream), qkv, static_cast<const uint2*>(kc),
                      static_cast<const uint2*>(vc), static_cast<int>(H), static_cast<int>(KVH), static_cast<int>(D),
                      static_cast<int>(maxctx), params, part);
}

W4A8_API w4a8_status w4a8_attn_combine(const float* part, int32_t H, int32_t KVH, int32_t D, int32_t maxctx,
                                       const uint32_t* params, int32_t m, const float* gsrc, int8_t* xq, float* xs,
                                       float* o_out, void* stream) {
    const w4a8_status c = check_attn("w4a8_attn_combine", H, KVH, D, maxctx, m, params);
    if (c != W4A8_OK) return c;
    if (!part || !xq || !xs) return set_error(W4A8_EINVAL, "w4a8_attn_combine: NULL pointer");
    if (((reinterpret_cast<uintptr_t>(part) | reinterpret_cast<uintptr_t>(xs)) & 7) ||
        (reinterpret_cast<uintptr_t>(xq) & 3) || (gsrc && (reinterpret_cast<uintptr_t>(gsrc) & 7)) ||
        (o_out && (reinterpret_cast<uintptr_t>(o_out) & 7)))
        return set_error(W4A8_EINVAL, "w4a8_attn_combine: part, xs, gsrc, o_out must be 8-byte aligned, xq 4-byte");
    static FuncAttr attr;
    const size_t smem = (static_cast<size_t>(D) + D / 32) * 4;
    const w4a8_status a = ensure_smem(attn_combine_kernel, attr, smem, -1, "w4a8_attn_combine");
    if (a != W4A8_OK) return a;
    return launch_pdl("w4a8_attn_combine", attn_combine_kernel, dim3(H, m), dim3(D / 2), smem,
                      static_cast<cudaStream_t>(stream), part, static_cast<int>(H), static_cast<int>(KVH),
                      static_cast<int>(D), static_cast<int>(maxctx), params, gsrc, xq, reinterpret_cast<float2*>(xs),
                      o_out);
}

}  // extern "C"
