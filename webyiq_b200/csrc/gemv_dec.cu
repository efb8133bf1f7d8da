// Decode GEMV: one or two tokens, group-128 weights, per-token int8 activations
// (or f32 activations quantized here), y = W x [+ y] or SWIGLU, for the
// projection shapes of a decode step (a few MB of weights per call).
//
// Reference: gemv_q4q8.wgsl:36-131 (per-group math at :68, modes at :122-129) and
// quant.wgsl for the fused per-token quantization.  Numerics: the exact per-token
// path of w4a8.h (int64 sum over groups of fix16(s) * (I - 8 X) [+ fix16(min) * X],
// then ((float)acc * 2^-24) * dx), bit-identical to the other GEMV kernels.
//
// Why this shape (B200 view).  A decode step is a chain of such calls, each waiting
// for the previous one (griddepcontrol.wait), so what counts is the time from that
// wait to the last store, not bandwidth: the weights (which do not depend on the
// previous kernel) are fetched before the wait, and after it the CTA meets one
// barrier (two with fused quant).
//  - One CTA per SM (two of consecutive calls fit on an SM, so the next call's
//    copies run while this one computes) owns a balanced contiguous row range.
//    Its rows are copied into shared memory with per-thread cp.async pieces, and
//    each thread waits for its own pieces before the dependency wait: bulk copies
//    issued by a dependent grid before griddepcontrol.wait complete only after the
//    previous grid has finished.  The CTA's scale span travels the same way, and
//    each lane decodes its groups' scales to (mantissa, shift) before the wait: a
//    plain load still in flight at the wait would hold up the activation loads.
//  - L lanes share a row (L = 8, 16 or 32) and each owns GPL whole 128-groups: the
//    exact int32 group dot from its 4 x GPL 16-byte chunks (dp4a, low and high
//    nibbles in separate accumulators), the group's int64 scale step, then log2(L)
//    shuffles add the row; the row's first lane writes y.  Chunks are read in a
//    per-lane rotated order so the 8 lanes of a shared-memory phase hit distinct
//    bank groups (rows are stored unpadded).
//  - The activations the lane meets stay in registers (32 x GPL per token), read
//    from a copy of the row staged once per CTA in shared memory with its group
//    sums.  Int8 activations are copied there with one coalesced, coherent 16-byte
//    load per piece (they are written by the previous kernel while this one is
//    already resident, so never through the read-only path); fused quant writes the
//    row there itself (one pass over the f32 row, the absmax exchanged by a shared
//    atomicMax, group sums from warp shuffles).
#include <cuda_fp16.h>

#include "gemv.cuh"
#include "launch.cuh"
#include "tma.cuh"

namespace w4a8 {

int sm_count();
unsigned int* device_error_word();  // gemv_mma.cu

namespace {

constexpr int kDecMaxPass = 4;                 // row passes per CTA (scale registers)
// fused quant: float4s of x a thread holds per token (12 in the 128-thread CTAs,
// so that K = 6144 fits them)
constexpr int dec_vpt(int m, int threads) { return m == 1 ? (threads <= 128 ? 12 : 8) : 4; }

// CTAs per SM.  DEEP (one token, when its rows fit 72 KB): three CTAs, so the CTAs
// of the next two calls are resident and copying their weights while this one
// computes; 256 threads with one group per lane (K <= 4096), 128 with two (~130
// registers).  Otherwise two CTAs: 384 threads for one token and one group per
// lane, which covers more rows per CTA, 256 for the rest.
template <int MT, int GPL, bool DEEP>
struct DecCfg {
    static constexpr int threads = DEEP ? (MT * GPL == 1 ? 256 : 128) : (MT * GPL == 1 ? 384 : 256);
    static constexpr int blocks = DEEP ? 3 : 2;  // registers: 3 x 256 x 80 or 3 x 128 x 130; 2 x 384 x 80
};
constexpr size_t kDecSmemDeep = 72 * 1024;     // three CTAs per SM
constexpr size_t kDecSmemBudget = 100 * 1024;  // two CTAs per SM

struct DecParams {
    const unsigned char* q;  // [rows][k/2]
    const void* s;           // [rows][k/128] u16 f16 (symmetric) or u32 (scale | min << 16)
    const int8_t* xq;        // [m][k]
    const float* xs;         // [m] per-token dx
    const float* xf32;       // [m][k] f32 activations to quantize here (FQ), else null
    const float* nw;         // FQ with NORM: RMSNorm weights [k]
    float eps;
    float* y;                // [m][y_stride]
    int n_out, k, m, y_stride;
    int L;         // lanes per row
    int rows_max;  // rows of the largest CTA range
    int sc_off;    // shared-memory offset of the scale spans (per half: sc_half bytes)
    int sc_half;
    unsigned int* err;  // device error word
};

__device__ __forceinline__ int pack_fix(uint32_t h) {
    const Fix16 f = fix16(h);
    return (f.mant << 8) | f.sh;
}

template <bool HAS_MIN, int MODE, int MT, int GPL, bool FQ, bool NORM, bool DEEP>
__global__ void __launch_bounds__(DecCfg<MT, GPL, DEEP>::threads, DecCfg<MT, GPL, DEEP>::blocks) gemv_dec_kernel(const DecParams p) {
    constexpr bool SWI = MODE == W4A8_SWIGLU;
    constexpr int NH = SWI ? 2 : 1;  // weight rows per output row (gate, up)
    constexpr int kSteps = 4 * GPL;  // 16-byte chunks per lane per row
    constexpr int T = DecCfg<MT, GPL, DEEP>::threads;
    constexpr int NW = T / 32;
    extern __shared__ __align__(128) unsigned char smem[];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = p.k, KG = K >> 7, KC = K >> 5, RB = K >> 1;
    const int L = p.L, lsh = __ffs(L) - 1;
    const int rb = static_cast<int>(static_cast<long long>(blockIdx.x) * p.n_out / gridDim.x);
    const int re = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * p.n_out / gridDim.x);
    const int nrow = re - rb;
    const size_t hstride = static_cast<size_t>(p.rows_max) * RB;

    pdl_launch_dependents();
    // ---- before the dependency wait: this CTA's weight rows and the lane's scales ----
    for (int i = warp; i < NH * nrow; i += NW) {
        const int h = SWI ? (i >= nrow) : 0;
        const int r = i - h * nrow;
        const unsigned char* src = p.q + (static_cast<size_t>(rb + r) + static_cast<size_t>(h) * p.n_out) * RB;
        unsigned char* dst = smem + h * hstride + static_cast<size_t>(r) * RB;
        for (int c = lane; c < KC; c += 32) cp_async16(dst + c * 16, src + c * 16);
    }
    // the scale span of the CTA's rows (per half), widened to 16-byte boundaries
    const int sbytes = HAS_MIN ? 4 : 2;
    size_t sbase[NH];
#pragma unroll
    for (int h = 0; h < NH; ++h) {
        const size_t b0 = (static_cast<size_t>(rb) + static_cast<size_t>(h) * p.n_out) * KG * sbytes;
        const size_t b1 = b0 + static_cast<size_t>(nrow) * KG * sbytes;
        const size_t a0 = b0 & ~static_cast<size_t>(15), a1 = (b1 + 15) & ~static_cast<size_t>(15);
        sbase[h] = b0 - a0;
        const unsigned char* src = static_cast<const unsigned char*>(p.s) + a0;
        unsigned char* dst = smem + p.sc_off + h * p.sc_half;
        for (int i = tid; i < static_cast<int>((a1 - a0) >> 4); i += T) cp_async16(dst + i * 16, src + i * 16);
    }
    cp_async_commit();

    const int j = lane & (L - 1);  // the lane's span of a row: groups [j*GPL, j*GPL + GPL)
    const int ph = lane & 7;       // position in its 16-byte shared-memory phase
    // rotation: step c reads chunk (c%4 + rc) % 4 of group j*GPL + (c/4 + rg) % GPL
    const int rg = (GPL % 2 == 0) ? (ph >> 2) & 1 : 0;
    const int rc = (GPL % 2 == 0) ? (ph & 3) : ((ph >> 1) & 3);
    int gidx[GPL];
    bool gin[GPL];
#pragma unroll
    for (int g = 0; g < GPL; ++g) {
        gidx[g] = j * GPL + (g + rg) % GPL;
        gin[g] = gidx[g] < KG;
    }
    int coff[kSteps];  // byte offset of step c's chunk in the packed row
#pragma unroll
    for (int c = 0; c < kSteps; ++c) coff[c] = (gidx[c / 4] * 4 + (c % 4 + rc) % 4) * 16;

    const int rpw = 32 >> lsh;  // rows a warp takes per pass
    const int npass = (nrow + NW * rpw - 1) / (NW * rpw);
    // The activations towards L2: a prefetch returns no data, so a line the previous
    // kernel still writes is read afresh after the wait; a line it does not write
    // (an input copied in long before) then comes from L2 instead of DRAM.
    {
        const char* xb0 = FQ ? reinterpret_cast<const char*>(p.xf32) : reinterpret_cast<const char*>(p.xq);
        const int lines = (p.m * K * (FQ ? 4 : 1) + 127) >> 7;
        for (int i = tid; i < lines; i += T) asm volatile("prefetch.global.L2 [%0];" ::"l"(xb0 + (static_cast<size_t>(i) << 7)));
        if (!FQ && tid == 0) asm volatile("prefetch.global.L2 [%0];" ::"l"(p.xs));
    }
    __shared__ unsigned int s_amax[2];  // fused quant: per-token absmax as float bits
    __shared__ float s_dx[2];
    __shared__ uint64_t s_xbar;         // int8 activations: their bulk copy landed
    if (FQ && tid < 2) s_amax[tid] = 0u;
    if (!FQ && tid == 0) {
        mbar_init(&s_xbar, 1);
        mbar_init_fence();
    }
    cp_async_wait_upto(0);  // this thread's pieces have landed
    __syncthreads();        // and everyone's
    // decoded scales (and mins) of this lane's groups, [pass][h][g]
    int sfx[kDecMaxPass][NH][GPL], mfx[kDecMaxPass][NH][GPL];
#pragma unroll
    for (int ps = 0; ps < kDecMaxPass; ++ps) {
        const int rl = (ps * NW + warp) * rpw + (lane >> lsh);
#pragma unroll
        for (int h = 0; h < NH; ++h)
#pragma unroll
            for (int g = 0; g < GPL; ++g) {
                sfx[ps][h][g] = mfx[ps][h][g] = 0;
                if (ps < npass && rl < nrow && gin[g]) {
                    const unsigned char* sp =
                        smem + p.sc_off + h * p.sc_half + sbase[h] + (static_cast<size_t>(rl) * KG + gidx[g]) * sbytes;
                    if (HAS_MIN) {
                        const uint32_t w = *reinterpret_cast<const uint32_t*>(sp);
                        sfx[ps][h][g] = pack_fix(w & 0xffffu);
                        mfx[ps][h][g] = pack_fix(w >> 16);
                    } else {
                        sfx[ps][h][g] = pack_fix(*reinterpret_cast<const unsigned short*>(sp));
                    }
                }
            }
    }
    pdl_wait();  // activations (and y for ADD) come from the previous kernel

    // ---- activations ----
    // Fused quant stages the quantized rows once per CTA in shared memory, per token:
    // the first 16 bytes of every 32-byte chunk, then the second 16 bytes (so the
    // lanes' rotated chunk reads are conflict-free), and the group sums X[KG].
    const int xrow = K + ((KG * 4 + 15) & ~15);  // bytes per token (16-byte multiple)
    unsigned char* xsm = smem + p.sc_off + NH * p.sc_half;
    auto xhalf = [&](int t, int h, int ci) -> unsigned char* {  // 16-byte half h of chunk ci
        return xsm + static_cast<size_t>(t) * xrow + h * (K / 2) + ci * 16;
    };
    auto xgrp = [&](int t) -> int* { return reinterpret_cast<int*>(xsm + static_cast<size_t>(t) * xrow + K); };
    float dx[MT];
    if (FQ) {
        // per-token quantization (quant.wgsl with one scale per token), exactly as
        // w4a8_quant computes it: amax, dx = amax / 127, inv = 1 / dx (0 for a zero
        // row), rint(x * inv).  One pass over x: each thread keeps its float4s in
        // registers across the amax exchange.  A warp's 32 neighbouring float4s are
        // one 128-group, so the group sums come from warp shuffles.
        constexpr int VPT = dec_vpt(MT, T);
        // With the norm, the first 256 threads hold x as the quant kernel's 256
        // threads do (float4 t + 256 j), so the sum of squares is added in the same
        // order and the RMS scale has the same bits.
        constexpr int XS = NORM ? 256 : T;  // stride of a thread's float4s
        const bool holder = !NORM || tid < 256;
        float4 v[MT][VPT];
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            const float4* src = reinterpret_cast<const float4*>(p.xf32 + static_cast<size_t>(t) * K);
#pragma unroll
            for (int u = 0; u < VPT; ++u) {
                const int i = tid + u * XS;
                v[t][u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (holder && t < p.m && i < K / 4) v[t][u] = ld_dep(src + i);
            }
        }
        if (NORM) {
            // scale = 1 / sqrt(sum(x^2) / k + eps): per-thread fma chain in element
            // order, a butterfly within each warp, then the 8 warp totals in order
            __shared__ float s_ss[2][8];
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                float ss = 0.0f;
#pragma unroll
                for (int u = 0; u < VPT; ++u) {
                    ss = __fmaf_rn(v[t][u].x, v[t][u].x, ss);
                    ss = __fmaf_rn(v[t][u].y, v[t][u].y, ss);
                    ss = __fmaf_rn(v[t][u].z, v[t][u].z, ss);
                    ss = __fmaf_rn(v[t][u].w, v[t][u].w, ss);
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(kFull, ss, off));
                if (lane == 0 && warp < 8) s_ss[t][warp] = ss;
            }
            __syncthreads();
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                float tot = 0.0f;
                for (int w8 = 0; w8 < 8; ++w8) tot = __fadd_rn(tot, s_ss[t][w8]);
                const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(K)), p.eps)));
                const float4* nw4 = reinterpret_cast<const float4*>(p.nw);
#pragma unroll
                for (int u = 0; u < VPT; ++u) {
                    const int i = tid + u * XS;
                    if (!holder || t >= p.m || i >= K / 4) continue;
                    const float4 n = __ldg(nw4 + i);
                    v[t][u].x = __fmul_rn(__fmul_rn(v[t][u].x, sc), n.x);
                    v[t][u].y = __fmul_rn(__fmul_rn(v[t][u].y, sc), n.y);
                    v[t][u].z = __fmul_rn(__fmul_rn(v[t][u].z, sc), n.z);
                    v[t][u].w = __fmul_rn(__fmul_rn(v[t][u].w, sc), n.w);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            float a = 0.0f;
#pragma unroll
            for (int u = 0; u < VPT; ++u)
                a = fmaxf(fmaxf(a, fabsf(v[t][u].x)), fmaxf(fmaxf(fabsf(v[t][u].y), fabsf(v[t][u].z)), fabsf(v[t][u].w)));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) a = fmaxf(a, __shfl_xor_sync(kFull, a, off));
            if (lane == 0 && t < p.m) atomicMax(&s_amax[t], __float_as_uint(a));
        }
        __syncthreads();
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            if (t >= p.m) continue;
            const float a = __uint_as_float(s_amax[t]);
            const float inv = a > 0.0f ? __fdiv_rn(1.0f, __fdiv_rn(a, 127.0f)) : 0.0f;
#pragma unroll
            for (int u = 0; u < VPT; ++u) {
                const int i = tid + u * XS;  // float4 index: elements 4i..4i+3
                if (u * XS >= K / 4) break;   // warp-uniform (K / 4 is a multiple of 32)
                const int q0 = static_cast<int>(rintf(__fmul_rn(v[t][u].x, inv)));
                const int q1 = static_cast<int>(rintf(__fmul_rn(v[t][u].y, inv)));
                const int q2 = static_cast<int>(rintf(__fmul_rn(v[t][u].z, inv)));
                const int q3 = static_cast<int>(rintf(__fmul_rn(v[t][u].w, inv)));
                int X = 0;
                if (holder && i < K / 4) {
                    *reinterpret_cast<uint32_t*>(xhalf(t, (i >> 2) & 1, i >> 3) + (i & 3) * 4) =
                        (static_cast<uint32_t>(q0) & 0xffu) | ((static_cast<uint32_t>(q1) & 0xffu) << 8) |
                        ((static_cast<uint32_t>(q2) & 0xffu) << 16) | ((static_cast<uint32_t>(q3) & 0xffu) << 24);
                    X = q0 + q1 + q2 + q3;
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) X += __shfl_xor_sync(kFull, X, off);
                if (lane == 0 && holder && i < K / 4) xgrp(t)[i >> 5] = X;
            }
            if (tid == 0) s_dx[t] = __fdiv_rn(a, 127.0f);
        }
    }
    uint4 xa[MT][kSteps], xb[MT][kSteps];
    int Xg[MT][GPL];
    if (!FQ) {
        // int8 activations: staged once per CTA in shared memory, in the layout the
        // fused quant writes, with the group sums.  The rows come in by one bulk copy
        // issued after the dependency wait: it goes through the TMA unit, not behind
        // the weight copies that the next calls' CTAs on this SM have queued at the
        // load/store unit.  Then one 16-byte shared-memory read per piece.
        const int pieces = K >> 4;  // 16-byte pieces per token; 8 per 128-group
        unsigned char* raw = xsm + static_cast<size_t>(p.m) * xrow;  // [m][K], after the staging rows
        if (tid == 0) {
            mbar_expect_tx(&s_xbar, static_cast<uint32_t>(p.m * K));
            tma_bulk_load(raw, p.xq, static_cast<uint32_t>(p.m * K), &s_xbar);
        }
        if (tid < MT) s_dx[tid] = tid < p.m ? ld_dep(p.xs + tid) : 0.0f;
        if (!mbar_wait(&s_xbar, 0)) {
            atomicOr(p.err, DEV_ERR_TMA_TIMEOUT);
            mbar_wait(&s_xbar, 0);  // once more (bounded), so the copy is not in flight at exit
        }
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            if (t >= p.m) break;
            const uint4* src = reinterpret_cast<const uint4*>(raw + static_cast<size_t>(t) * K);
            for (int base = warp * 32; base < pieces; base += T) {  // whole warps: the shuffles below
                const int i = base + lane;
                const bool in = i < pieces;
                const uint4 v = in ? src[i] : make_uint4(0, 0, 0, 0);
                if (in) *reinterpret_cast<uint4*>(xhalf(t, i & 1, i >> 1)) = v;
                const uint32_t ones = 0x01010101u;
                int X = dp4a(ones, v.x, dp4a(ones, v.y, dp4a(ones, v.z, dp4a(ones, v.w, 0))));
                X += __shfl_xor_sync(kFull, X, 1);
                X += __shfl_xor_sync(kFull, X, 2);
                X += __shfl_xor_sync(kFull, X, 4);
                if (in && (i & 7) == 0) xgrp(t)[i >> 3] = X;
            }
        }
    }
    {
        __syncthreads();
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            dx[t] = t < p.m ? s_dx[t] : 0.0f;
#pragma unroll
            for (int g = 0; g < GPL; ++g) Xg[t][g] = (t < p.m && gin[g]) ? xgrp(t)[gidx[g]] : 0;
#pragma unroll
            for (int c = 0; c < kSteps; ++c) {
                xa[t][c] = xb[t][c] = make_uint4(0, 0, 0, 0);
                if (t < p.m && gin[c / 4]) {
                    const int ci = coff[c] >> 4;  // chunk index in the row
                    xa[t][c] = *reinterpret_cast<const uint4*>(xhalf(t, 0, ci));
                    xb[t][c] = *reinterpret_cast<const uint4*>(xhalf(t, 1, ci));
                }
            }
        }
    }

    // ---- row passes ----
#pragma unroll
    for (int ps = 0; ps < kDecMaxPass; ++ps) {
        if (ps >= npass) break;
        const int rl = (ps * NW + warp) * rpw + (lane >> lsh);
        const bool rin = rl < nrow;
        long long acc[NH][MT];
#pragma unroll
        for (int h = 0; h < NH; ++h) {
            const unsigned char* row = smem + h * hstride + static_cast<size_t>(rin ? rl : 0) * RB;
            uint4 w[kSteps];
#pragma unroll
            for (int c = 0; c < kSteps; ++c)
                w[c] = (rin && gin[c / 4]) ? *reinterpret_cast<const uint4*>(row + coff[c]) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                acc[h][t] = 0;
#pragma unroll
                for (int g = 0; g < GPL; ++g) {
                    const uint32_t ml = 0x0F0F0F0Fu, mh = 0xF0F0F0F0u;
                    int lo = 0, hi = 0;
#pragma unroll
                    for (int c = 4 * g; c < 4 * g + 4; ++c) {
                        lo = dp4a_us(w[c].x & ml, xa[t][c].x, lo);
                        hi = dp4a_us(w[c].x & mh, xa[t][c].y, hi);
                        lo = dp4a_us(w[c].y & ml, xa[t][c].z, lo);
                        hi = dp4a_us(w[c].y & mh, xa[t][c].w, hi);
                        lo = dp4a_us(w[c].z & ml, xb[t][c].x, lo);
                        hi = dp4a_us(w[c].z & mh, xb[t][c].y, hi);
                        lo = dp4a_us(w[c].w & ml, xb[t][c].z, lo);
                        hi = dp4a_us(w[c].w & mh, xb[t][c].w, hi);
                    }
                    const int I = lo + (hi >> 4);  // hi is an exact multiple of 16
                    const int sf = sfx[ps][h][g];
                    if (HAS_MIN) {
                        const int mf = mfx[ps][h][g];
                        acc[h][t] += shl64((sf >> 8) * I, sf & 0xff) + shl64((mf >> 8) * Xg[t][g], mf & 0xff);
                    } else {
                        acc[h][t] += shl64((sf >> 8) * (I - 8 * Xg[t][g]), sf & 0xff);
                    }
                }
            }
        }
        for (int off = 1; off < L; off <<= 1)
#pragma unroll
            for (int h = 0; h < NH; ++h)
#pragma unroll
                for (int t = 0; t < MT; ++t) acc[h][t] += shfl_xor_i64(acc[h][t], off);
        if (j == 0 && rin) {
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                if (t >= p.m) continue;
                float v = fix_to_float(acc[0][t], dx[t]);
                float* yp = p.y + static_cast<size_t>(t) * p.y_stride + rb + rl;
                if (SWI)
                    *yp = silu_mul(v, fix_to_float(acc[NH - 1][t], dx[t]));
                else if (MODE == W4A8_ADD)
                    *yp = __fadd_rn(*yp, v);
                else
                    *yp = v;
            }
        }
    }
}

// Lanes per row and groups per lane: the smallest L in {8, 16, 32} covering the row
// with GPL * MT <= 2 groups' activations in registers; L = 0 when none does.
struct DecShape {
    int L, gpl;
};
DecShape dec_shape(int kg, int m) {
    for (int gpl = 1; gpl <= (m == 1 ? 2 : 1); ++gpl)
        for (int L = 8; L <= 32; L <<= 1)
            if (kg <= L * gpl) return {L, gpl};
    return {0, 0};
}

struct DecPlan {
    DecShape sh;
    bool deep;  // three CTAs per SM
    int ctas, rows_max, threads;
    int sc_off, sc_half;
    size_t smem;
};

// The plan for CTAs of `threads` threads; whether it fits `budget` bytes of shared
// memory, kDecMaxPass row passes and the fused quant's registers.
bool dec_fit(const GemvParams& g, bool has_min, int mode, int threads, size_t budget, DecPlan& pl) {
    pl.threads = threads;
    const int sms = sm_count();
    pl.ctas = g.n_out < sms ? g.n_out : sms;
    pl.rows_max = (g.n_out + pl.ctas - 1) / pl.ctas;
    const int nh = mode == W4A8_SWIGLU ? 2 : 1;
    const int sbytes = has_min ? 4 : 2;
    pl.sc_off = nh * pl.rows_max * (g.k / 2);
    pl.sc_half = ((pl.rows_max * (g.k / 128) * sbytes + 15) & ~15) + 16;  // + the widening to 16 bytes
    pl.smem = static_cast<size_t>(pl.sc_off) + static_cast<size_t>(nh) * pl.sc_half +
              static_cast<size_t>(g.m) * (g.k + (((g.k / 128) * 4 + 15) & ~15)) +  // activation staging
              (g.xf32 ? 0 : static_cast<size_t>(g.m) * g.k);                        // and its bulk copy
    const int rows_per_pass = (pl.threads / 32) * (32 / pl.sh.L);
    const int npass = (pl.rows_max + rows_per_pass - 1) / rows_per_pass;
    const int xs = g.norm_w ? 256 : pl.threads;  // the threads that hold x (the norm's partition)
    const bool vpt_ok = !g.xf32 || (g.k / 4 + xs - 1) / xs <= dec_vpt(g.m, threads);
    return pl.smem <= budget && npass <= kDecMaxPass && vpt_ok;
}

bool dec_plan(const GemvParams& g, bool has_min, int mode, DecPlan& pl) {
    if (g.m < 1 || g.m > 2 || g.k % 128 != 0 || g.n_out < 1) return false;
    pl.sh = dec_shape(g.k / 128, g.m);
    if (pl.sh.L == 0) return false;
    const bool one = g.m * pl.sh.gpl == 1;
    // three CTAs per SM for one token (with two groups a lane: 128 threads, and not
    // with the norm, whose partition of x needs 256)
    pl.deep = g.m == 1 && (one || !g.norm_w) &&
              dec_fit(g, has_min, mode, one ? DecCfg<1, 1, true>::threads : DecCfg<1, 2, true>::threads, kDecSmemDeep, pl);
    if (pl.deep) return true;
    return dec_fit(g, has_min, mode, one ? DecCfg<1, 1, false>::threads : DecCfg<2, 1, false>::threads, kDecSmemBudget, pl);
}

template <bool HAS_MIN, int MODE, int MT, int GPL, bool FQ, bool NORM, bool DEEP>
w4a8_status dec_inst(const DecParams& p, const DecPlan& pl, cudaStream_t st) {
    // set on first use per device: static shared memory counts against the default 48 KB too
    static FuncAttr attr;
    auto kernel = gemv_dec_kernel<HAS_MIN, MODE, MT, GPL, FQ, NORM, DEEP>;
    const w4a8_status a = ensure_smem(kernel, attr, pl.smem, 100, "w4a8 gemv (decode)");
    if (a != W4A8_OK) return a;
    return launch_pdl("w4a8 gemv (decode)", kernel, dim3(pl.ctas), dim3(DecCfg<MT, GPL, DEEP>::threads), pl.smem, st, p);
}

template <bool HAS_MIN, int MODE, bool FQ, bool NORM>
w4a8_status dec_shape_dispatch(const DecParams& p, const DecPlan& pl, cudaStream_t st) {
    if (p.m == 1 && pl.sh.gpl == 1)
        return pl.deep ? dec_inst<HAS_MIN, MODE, 1, 1, FQ, NORM, true>(p, pl, st)
                       : dec_inst<HAS_MIN, MODE, 1, 1, FQ, NORM, false>(p, pl, st);
    if (p.m == 1)
        return pl.deep && !NORM ? dec_inst<HAS_MIN, MODE, 1, 2, FQ, false, true>(p, pl, st)
                                : dec_inst<HAS_MIN, MODE, 1, 2, FQ, NORM, false>(p, pl, st);
    return dec_inst<HAS_MIN, MODE, 2, 1, FQ, NORM, false>(p, pl, st);
}

template <bool HAS_MIN, bool FQ, bool NORM = false>
w4a8_status dec_mode_dispatch(const DecParams& p, const DecPlan& pl, int mode, cudaStream_t st) {
    if (mode == W4A8_STORE) return dec_shape_dispatch<HAS_MIN, W4A8_STORE, FQ, NORM>(p, pl, st);
    if (mode == W4A8_ADD) return dec_shape_dispatch<HAS_MIN, W4A8_ADD, FQ, NORM>(p, pl, st);
    return dec_shape_dispatch<HAS_MIN, W4A8_SWIGLU, FQ, NORM>(p, pl, st);
}

}  // namespace

// Whether the decode GEMV covers this call: group 128, per-token activations, the
// y output, one or two tokens, and a per-CTA row range that fits shared memory.
bool gemv_dec_covers(const GemvParams& g, int group, int act, int mode, int out) {
    if (group != 128 || act != W4A8_ACT_TOKEN || out != OUT_Y) return false;
    DecPlan pl;
    return dec_plan(g, true, mode, pl);  // the larger (u32) scale span
}

w4a8_status launch_gemv_dec(const GemvParams& g, bool has_min, int mode, cudaStream_t st) {
    DecPlan pl;
    if (!dec_plan(g, has_min, mode, pl)) return set_error(W4A8_EINVAL, "w4a8 gemv (decode): call not covered");
    DecParams p{};
    p.q = reinterpret_cast<const unsigned char*>(g.q);
    p.s = g.s;
    p.xq = g.xq;
    p.xs = g.xs;
    p.xf32 = g.xf32;
    p.nw = g.norm_w;
    p.eps = g.eps;
    p.y = g.y;
    p.n_out = g.n_out;
    p.k = g.k;
    p.m = g.m;
    p.y_stride = g.y_stride;
    p.L = pl.sh.L;
    p.rows_max = pl.rows_max;
    p.sc_off = pl.sc_off;
    p.sc_half = pl.sc_half;
    p.err = device_error_word();
    if (!p.err) return set_error(W4A8_ECUDA, "w4a8 gemv (decode): device error word unavailable");
    if (!g.xf32 && (reinterpret_cast<uintptr_t>(g.xq) & 15) != 0)
        return set_error(W4A8_EINVAL, "w4a8 gemv (decode): xq not 16-byte aligned");
    if (g.xf32 && g.norm_w)
        return has_min ? dec_mode_dispatch<true, true, true>(p, pl, mode, st)
                       : dec_mode_dispatch<false, true, true>(p, pl, mode, st);
    if (g.xf32) return has_min ? dec_mode_dispatch<true, true>(p, pl, mode, st) : dec_mode_dispatch<false, true>(p, pl, mode, st);
    return has_min ? dec_mode_dispatch<true, false>(p, pl, mode, st) : dec_mode_dispatch<false, false>(p, pl, mode, st);
}

}  // namespace w4a8
