// W4A8 GEMV family: y = W x for 1..16 tokens, the group-dot test hook, and the
// lm_head GEMV with fused argmax.  One template, three epilogues.
//
// Work split (B200 view): the GEMV streams the packed weights from HBM once, so
// the kernel is built around keeping enough 16-byte weight loads in flight.  A
// warp is cut into 32/LPR row-groups of LPR lanes (LPR = 8, 16 or 32, picked from
// k so every lane owns about 8 chunks of a row); each row-group owns one output row
// (two weight rows for SWIGLU) and its lanes walk the row in 16-byte chunks
// (32 weights) with stride LPR, so one load instruction of the warp reads
// LPR*16 contiguous bytes of each of its rows.  The reduction over a row is
// log2(LPR) shuffles, shared by all rows of the warp.
//
// Reference: gemv_q4q8.wgsl:36-131 (per-group math at :68, modes at :122-129),
// argmax.wgsl:14-43 for the fused argmax.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace w4a8 {

enum GemvOut { OUT_Y = 0, OUT_DOTS = 1, OUT_ARGMAX = 2 };

struct GemvParams {
    const uint4* q;        // [rows, k/32] 16-byte chunks
    const void* s;         // scales, see w4a8.h
    const int8_t* xq;      // [m, k]
    const float* xs;       // [m] (TOKEN) or [m, k/32, 2] (GROUP32)
    float* y;              // OUT_Y: output; OUT_ARGMAX: logits or null
    int* dots;             // OUT_DOTS: [m, n_out, k/G]
    unsigned int* counter;           // OUT_ARGMAX workspace: CTAs done
    unsigned long long* ws_best;     // OUT_ARGMAX workspace: running max key per token
    unsigned long long* best_key;    // OUT_ARGMAX: [m]
    unsigned int* tok_out;           // OUT_ARGMAX: [m] or null
    const unsigned int* ids;         // OUT_ARGMAX: [vocab] or null
    int n_out;      // output rows (stored rows / 2 for SWIGLU)
    int k;
    int m;
    int lpr;        // lanes per row: 8, 16 or 32
    int row_offset; // OUT_ARGMAX: global id of row 0
};

constexpr int kGemvMaxWarps = 8;

template <int G, bool HAS_MIN, int ACT, int MODE, int MT, int OUT>
__global__ void __launch_bounds__(kGemvMaxWarps * 32)
gemv_kernel(const GemvParams p) {
    constexpr int U = 8;                     // chunks per lane per pass
    constexpr int NR = (MODE == W4A8_SWIGLU) ? 2 : 1;
    constexpr bool EXACT = (ACT == W4A8_ACT_TOKEN);
    using Acc = typename std::conditional<EXACT, long long, float>::type;

    const int lane = threadIdx.x & 31;
    const int lpr = p.lpr;
    const int lig = lane & (lpr - 1);        // lane in row-group
    const int warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    const int rgw = 32 / lpr;                // row-groups per warp
    const int orow = (blockIdx.x * nwarps + warp) * rgw + lane / lpr;
    const bool row_ok = orow < p.n_out;
    const int KC = p.k >> 5;                 // chunks per row
    const int KG = p.k / G;                  // groups per row

    const uint4* wrow[NR];
    int srow[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        const int rr = row_ok ? orow + r * p.n_out : 0;
        wrow[r] = p.q + static_cast<size_t>(rr) * KC;
        srow[r] = rr * KG;
    }

    Acc acc[NR][MT];
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[r][t] = Acc(0);

    // The next kernel in the stream may be scheduled as soon as every CTA of this
    // one is resident; it only prefetches weights before its own pdl_wait().
    pdl_launch_dependents();

    for (int c0 = 0; c0 < KC; c0 += lpr * U) {
        // Weights and scales first: they do not depend on the previous kernel.
        uint4 wv[NR][U];
        uint32_t sv[NR][U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = c0 + lig + lpr * u;
            const bool ok = row_ok && c < KC;
            const int g = (c * 32) / G;
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                wv[r][u] = ok ? ldg_stream(wrow[r] + c) : make_uint4(0, 0, 0, 0);
                if (HAS_MIN)
                    sv[r][u] = ok ? __ldg(static_cast<const uint32_t*>(p.s) + srow[r] + g) : 0u;
                else
                    sv[r][u] = ok ? static_cast<uint32_t>(__ldg(static_cast<const unsigned short*>(p.s) + srow[r] + g)) : 0u;
            }
        }
        if (c0 == 0) pdl_wait();  // activations (and y for ADD) come from the previous kernel

#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = c0 + lig + lpr * u;
            const bool ok = row_ok && c < KC;
            uint32_t lo[NR][4], hi[NR][4];
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                lo[r][0] = lo_nibbles(wv[r][u].x); hi[r][0] = hi_nibbles(wv[r][u].x);
                lo[r][1] = lo_nibbles(wv[r][u].y); hi[r][1] = hi_nibbles(wv[r][u].y);
                lo[r][2] = lo_nibbles(wv[r][u].z); hi[r][2] = hi_nibbles(wv[r][u].z);
                lo[r][3] = lo_nibbles(wv[r][u].w); hi[r][3] = hi_nibbles(wv[r][u].w);
            }
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                int dotv = 0;  // OUT_DOTS: this chunk's dot for token t
                if (t < p.m && ok) {
                    const uint4* xp = reinterpret_cast<const uint4*>(p.xq + static_cast<size_t>(t) * p.k) + 2 * c;
                    const uint4 xa = __ldg(xp);
                    const uint4 xb = __ldg(xp + 1);
                    const int X = chunk_sum(xa, xb);
#pragma unroll
                    for (int r = 0; r < NR; ++r) {
                        const int I = chunk_dot(lo[r], hi[r], xa, xb);
                        if (OUT == OUT_DOTS) {
                            dotv = HAS_MIN ? I : I - 8 * X;
                        } else if (EXACT) {
                            if (HAS_MIN) {
                                const Fix16 s = fix16(sv[r][u] & 0xffffu);
                                const Fix16 mn = fix16(sv[r][u] >> 16);
                                acc[r][t] += shl64(s.mant * I, s.sh) + shl64(mn.mant * X, mn.sh);
                            } else {
                                const Fix16 s = fix16(sv[r][u]);
                                acc[r][t] += shl64(s.mant * (I - 8 * X), s.sh);
                            }
                        } else {
                            const float2 d = __ldg(reinterpret_cast<const float2*>(p.xs) +
                                                   static_cast<size_t>(t) * KC + c);
                            if (HAS_MIN) {
                                const float s = __half2float(__ushort_as_half(static_cast<unsigned short>(sv[r][u] & 0xffffu)));
                                const float mn = __half2float(__ushort_as_half(static_cast<unsigned short>(sv[r][u] >> 16)));
                                acc[r][t] += s * d.x * static_cast<float>(I) + mn * d.y;
                            } else {
                                const float s = __half2float(__ushort_as_half(static_cast<unsigned short>(sv[r][u])));
                                acc[r][t] += s * d.x * static_cast<float>(I - 8 * X);
                            }
                        }
                    }
                }
                if (OUT == OUT_DOTS && t < p.m) {
                    // G = 128: the 4 chunks of a group sit on 4 neighbouring lanes
                    if (G == 128) {
                        dotv += __shfl_xor_sync(kFull, dotv, 1);
                        dotv += __shfl_xor_sync(kFull, dotv, 2);
                    }
                    if (ok && (G == 32 || (lig & 3) == 0))
                        p.dots[(static_cast<size_t>(t) * p.n_out + orow) * KG + (c * 32) / G] = dotv;
                }
            }
        }
    }
    if (OUT == OUT_DOTS) return;

    // Sum over the lanes of the row-group (exact in the int64 path).
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
        for (int t = 0; t < MT; ++t)
            for (int off = lpr >> 1; off > 0; off >>= 1) {
                if (EXACT)
                    acc[r][t] += shfl_xor_i64(acc[r][t], off);
                else
                    acc[r][t] += __shfl_xor_sync(kFull, acc[r][t], off);
            }

    float val[NR][MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        float dx = 1.0f;
        if (EXACT && t < p.m) dx = __ldg(p.xs + t);
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            if (EXACT)
                val[r][t] = fix_to_float(static_cast<long long>(acc[r][t]), dx);
            else
                val[r][t] = static_cast<float>(acc[r][t]);
        }
    }

    if (OUT == OUT_Y) {
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            if (row_ok && t < p.m && lig == (t & (lpr - 1))) {
                float* yp = p.y + static_cast<size_t>(t) * p.n_out + orow;
                if (MODE == W4A8_STORE)
                    *yp = val[0][t];
                else if (MODE == W4A8_ADD)
                    *yp = __fadd_rn(*yp, val[0][t]);
                else
                    *yp = silu_mul(val[0][t], val[NR - 1][t]);
            }
        }
        return;
    }

    // OUT_ARGMAX
    __shared__ unsigned long long s_key[kGemvMaxWarps][MT];
    __shared__ bool s_last;
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        if (p.y != nullptr && row_ok && t < p.m && lig == (t & (lpr - 1)))
            p.y[static_cast<size_t>(t) * p.n_out + orow] = val[0][t];
        unsigned long long key = (row_ok && t < p.m) ? argmax_key(val[0][t], static_cast<uint32_t>(p.row_offset + orow)) : 0ull;
        for (int off = lpr; off < 32; off <<= 1) {
            const unsigned long long o = shfl_xor_u64(key, off);
            key = o > key ? o : key;
        }
        if (lane == 0) s_key[warp][t] = key;
    }
    __syncthreads();
    if (threadIdx.x < p.m) {
        unsigned long long key = 0;
        for (int w = 0; w < nwarps; ++w) {
            const unsigned long long o = s_key[w][threadIdx.x];
            key = o > key ? o : key;
        }
        if (key) atomicMax(p.ws_best + threadIdx.x, key);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int done = atomicAdd(p.counter, 1u);
        s_last = (done == gridDim.x - 1);
    }
    __syncthreads();
    if (s_last) {
        __threadfence();
        if (threadIdx.x < p.m) {
            const unsigned long long key = atomicExch(p.ws_best + threadIdx.x, 0ull);
            p.best_key[threadIdx.x] = key;
            if (p.tok_out) {
                const uint32_t idx = key ? ~static_cast<uint32_t>(key & 0xffffffffu) : 0u;
                p.tok_out[threadIdx.x] = p.ids ? __ldg(p.ids + idx) : idx;
            }
        }
        if (threadIdx.x == 0) *p.counter = 0u;
    }
}

// Host-side launch of one instantiation (defined in gemv_*.cu).
w4a8_status launch_gemv(const GemvParams& p, int group, bool has_min, int act, int mode, int out,
                        int nwarps, int grid, cudaStream_t stream);

}  // namespace w4a8
