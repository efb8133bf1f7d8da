// W4A8 GEMV family: y = W x for 1..4 tokens per launch, the group-dot test hook,
// and the lm_head GEMV with fused argmax.  One template, three epilogues.
//
// Work split (B200 view).  The GEMV streams the packed weights from HBM exactly
// once, so the kernel is shaped like a copy kernel with a little integer math:
//  - Persistent CTAs (2 per SM) own balanced contiguous ranges of output rows.  A
//    range is walked in rounds; the rows of a round are one contiguous span of
//    16-byte chunks (32 weights each; two spans for SWIGLU).
//  - The CTA has T = KC * floor(256 / KC) threads (KC = chunks per row), so thread
//    t always owns chunk column c = t % KC: in a round it loads column c of rows
//    t / KC + j * (T / KC), j < U, with 16-byte non-allocating loads into
//    registers, every warp instruction moving 512 contiguous bytes.  Round 0 is
//    requested before griddepcontrol.wait, i.e. while the previous kernel still
//    runs, and round r+1 before round r is summed.
//  - Because the column is fixed, each thread reads its 32 activation bytes per
//    token from global once, right after the wait: no staging, no barrier.
//  - Per chunk: 8 dp4a (the high nibbles are used in place, x16, through an
//    unsigned-by-signed dp4a), then the 4 chunks of a 128-group (4 neighbouring
//    lanes) are summed by two shuffles and scaled once; the group terms are summed
//    over the warp's 32 columns by shuffles and stored per (row, warp segment);
//    one thread per row adds the segments in a fixed order, so results never
//    depend on timing.
//
// Reference: gemv_q4q8.wgsl:36-131 (per-group math at :68, modes at :122-129),
// argmax.wgsl:14-43 for the fused argmax.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace w4a8 {

enum GemvOut { OUT_Y = 0, OUT_DOTS = 1, OUT_ARGMAX = 2 };

constexpr int kGemvMaxThreads = 256;
#ifndef W4A8_GEMV_U
#define W4A8_GEMV_U 7
#endif
#ifndef W4A8_GEMV_MINB1
#define W4A8_GEMV_MINB1 4
#endif
constexpr int kGemvU = W4A8_GEMV_U;  // chunks (rows) per thread per round (8 for SWIGLU)
__host__ __device__ constexpr int gemv_u(int nr) { return nr == 2 ? 8 : kGemvU; }
constexpr int kGemvMaxMT = 4;    // tokens per launch; more tokens = more launches
constexpr int kGemvMaxKC = 256;  // k <= 8192

struct XchgArgs;  // xchg.cuh

struct GemvParams {
    const uint4* q;        // [rows, k/32] 16-byte chunks
    const void* s;         // scales, see w4a8.h
    const int8_t* xq;      // [m, k]
    const float* xs;       // [m] (TOKEN) or [m, k/32, 2] (GROUP32)
    const float* xf32;     // tensor-core GEMV only: [m, k] f32 activations quantized per token inside
    const float* norm_w;   // decode GEMV with fused quant only: RMSNorm weights [k] (or null)
    float eps;             // and its epsilon
    float* y;              // OUT_Y: output; OUT_ARGMAX: logits or null
    int* dots;             // OUT_DOTS: [m, n_out, k/G]
    unsigned int* counter;           // OUT_ARGMAX workspace: CTAs done
    unsigned long long* ws_best;     // OUT_ARGMAX workspace: running max key per token
    unsigned long long* best_key;    // OUT_ARGMAX: [m]
    unsigned int* tok_out;           // OUT_ARGMAX: [m] or null
    const unsigned int* ids;         // OUT_ARGMAX: [vocab] or null
    int n_out;      // output rows (stored rows / 2 for SWIGLU)
    int k;
    int m;          // tokens in this launch (<= kGemvMaxMT)
    int y_stride;   // token stride of y (n_out of the full call)
    int row_offset; // OUT_ARGMAX: global id of row 0
    const XchgArgs* xchg;  // OUT_ARGMAX, streaming kernel only: merge the keys over peers in the last CTA (or null)
};

// Segment = the lanes whose group terms are summed by shuffles before they are
// stored: 8 neighbouring lanes (two 128-groups, or eight 32-groups) when a row
// has a multiple of 8 chunks, else the 4 chunks of a group (G=128) or one chunk.
__host__ __device__ inline int gemv_seg(int kc, int cpg) { return kc % 8 == 0 ? 8 : cpg; }

// Working threads (a multiple of kc); the CTA is rounded up to whole warps and the
// extra threads only join the shuffles.
__host__ __device__ inline int gemv_workers(int kc) { return kc * (kGemvMaxThreads / kc); }
__host__ __device__ inline int gemv_threads(int kc) { return (gemv_workers(kc) + 31) & ~31; }

// Shared memory: the segment terms of one round, [m][NR][rows][nseg] (8-byte).
__host__ __device__ inline size_t gemv_smem_bytes(int m, int k, int group, int nr) {
    const int kc = k / 32;
    const int rows = (gemv_workers(kc) / kc) * (gemv_u(nr) / nr);
    const int nseg = kc / gemv_seg(kc, group / 32);
    return static_cast<size_t>(m) * nr * rows * nseg * 8;
}

// dp4a with unsigned bytes in a and signed bytes in b.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Dot of one chunk (4 weight words) with 32 int8 activations (xa, xb).  Low nibbles
// are weights 8i..8i+3 and meet xa/xb words 0, 2, 4, 6; high nibbles, weights
// 8i+4..8i+7, meet words 1, 3, 5, 7 and are used in place (16x their value), so
// the chunk dot is lo + (hi16 >> 4), exact (|hi16| < 2^17).
__device__ __forceinline__ int chunk_dot16(const uint4& w, const uint4& xa, const uint4& xb) {
    const uint32_t ml = 0x0F0F0F0Fu, mh = 0xF0F0F0F0u;
    int lo = 0, hi = 0;
    lo = dp4a_us(w.x & ml, xa.x, lo);
    hi = dp4a_us(w.x & mh, xa.y, hi);
    lo = dp4a_us(w.y & ml, xa.z, lo);
    hi = dp4a_us(w.y & mh, xa.w, hi);
    lo = dp4a_us(w.z & ml, xb.x, lo);
    hi = dp4a_us(w.z & mh, xb.y, hi);
    lo = dp4a_us(w.w & ml, xb.z, lo);
    hi = dp4a_us(w.w & mh, xb.w, hi);
    return lo + (hi >> 4);
}

// Bulk prefetch of [p, p + bytes) into L2 by the copy engine (16-byte multiples).
__device__ __forceinline__ void l2_prefetch_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

template <int MT>
struct GemvLaunchBounds {
    static constexpr int min_blocks = MT == 1 ? W4A8_GEMV_MINB1 : 2;
};

template <int G, bool HAS_MIN, int ACT, int MODE, int MT, int OUT>
__global__ void __launch_bounds__(kGemvMaxThreads, GemvLaunchBounds<MT>::min_blocks)
gemv_kernel(const GemvParams p) {
    constexpr int NR = (MODE == W4A8_SWIGLU) ? 2 : 1;
    constexpr bool EXACT = (ACT == W4A8_ACT_TOKEN);
    constexpr int CPG = G / 32;      // chunks per group (1 or 4)
    constexpr int U = gemv_u(NR);
    constexpr int UH = U / NR;       // rows per half per thread-round
    using Term = typename std::conditional<EXACT, long long, float>::type;
    extern __shared__ __align__(16) unsigned char smem[];

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int T = blockDim.x;
    const int KC = p.k >> 5;
    const int KG = p.k / G;
    const int m = p.m;
    const int c = tid % KC;             // this thread's chunk column
    const bool worker = tid < gemv_workers(KC);
    const int rpj = gemv_workers(KC) / KC;  // rows per j
    const int rr = rpj * UH;            // output rows per round
    const int seg = gemv_seg(KC, CPG);  // lanes per stored segment
    const int nseg = KC / seg;
    const int g = c / CPG;              // group of the column
    const bool lead = worker && (lane % seg) == 0;
    Term* red = reinterpret_cast<Term*>(smem);  // [m][NR][rr][nseg]

    const int rb = static_cast<int>(static_cast<long long>(blockIdx.x) * p.n_out / gridDim.x);
    const int re = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * p.n_out / gridDim.x);
    const int rounds = (re - rb + rr - 1) / rr;
    const int r0t = tid / KC;  // this thread's first row within a round

    // weights of a round: registers, requested early
    uint4 wv[U];
    auto load = [&](int o0) {
        const int o1 = min(o0 + rr, re);
#pragma unroll
        for (int j = 0; j < U; ++j) {
            const int row = o0 + r0t + (j % UH) * rpj;
            const size_t grow = static_cast<size_t>(row) + (j >= UH ? static_cast<size_t>(p.n_out) : 0);
            wv[j] = (worker && row < o1) ? ldg_stream(p.q + grow * KC + c) : make_uint4(0, 0, 0, 0);
        }
    };
    // scales of a round: asked of L2 in bulk early, read when the round is computed
    const int sb = HAS_MIN ? 4 : 2;
    auto prefetch_scales = [&](int o0) {
        if (tid != 0) return;
        const int o1 = min(o0 + rr, re);
        for (int h = 0; h < NR; ++h) {
            const size_t b0 = ((static_cast<size_t>(o0) + static_cast<size_t>(h) * p.n_out) * KG) * sb;
            const size_t b1 = ((static_cast<size_t>(o1) + static_cast<size_t>(h) * p.n_out) * KG) * sb;
            const size_t a0 = (b0 + 15) & ~static_cast<size_t>(15), a1 = b1 & ~static_cast<size_t>(15);
            if (a1 > a0) l2_prefetch_bulk(static_cast<const unsigned char*>(p.s) + a0, static_cast<uint32_t>(a1 - a0));
        }
    };
    // weights of a later round: asked of L2 in bulk (one instruction per span)
    auto prefetch_weights = [&](int o0) {
        if (tid != 0 || o0 >= re) return;
        const int o1 = min(o0 + rr, re);
        for (int h = 0; h < NR; ++h) {
            const uint4* a = p.q + (static_cast<size_t>(o0) + static_cast<size_t>(h) * p.n_out) * KC;
            l2_prefetch_bulk(a, static_cast<uint32_t>(static_cast<size_t>(o1 - o0) * KC * 16));
        }
    };
    auto scale_of = [&](int o0, int j) -> uint32_t {
        const int row = o0 + r0t + (j % UH) * rpj;
        const size_t e = (static_cast<size_t>(row) + (j >= UH ? static_cast<size_t>(p.n_out) : 0)) * KG + g;
        return HAS_MIN ? __ldg(static_cast<const uint32_t*>(p.s) + e)
                       : static_cast<uint32_t>(__ldg(static_cast<const unsigned short*>(p.s) + e));
    };

    // The next kernel in the stream may be scheduled as soon as every CTA of this
    // one is resident; it only requests weights before its own pdl_wait().
    pdl_launch_dependents();
    if (rounds > 0) {
        prefetch_scales(rb);
        if (rounds > 1) {
            prefetch_weights(rb + rr);
            prefetch_scales(rb + rr);
        }
        load(rb);
    }
    pdl_wait();  // activations (and y for ADD) come from the previous kernel

    // this thread's activation column, its chunk sum and its group sum, per token
    uint4 xa[MT], xb[MT];
    int Xg[MT];
    float dx[MT], dxs[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        xa[t] = xb[t] = make_uint4(0, 0, 0, 0);
        dx[t] = dxs[t] = 0.0f;
        if (t < m) {
            const uint4* xp = reinterpret_cast<const uint4*>(p.xq + static_cast<size_t>(t) * p.k) + 2 * c;
            xa[t] = ld_dep(xp);
            xb[t] = ld_dep(xp + 1);
            if (EXACT) {
                dx[t] = ld_dep(p.xs + t);
            } else {
                const float2 d = ld_dep(reinterpret_cast<const float2*>(p.xs) + static_cast<size_t>(t) * KC + c);
                dx[t] = d.x;
                dxs[t] = d.y;
            }
        }
        int X = chunk_sum(xa[t], xb[t]);
        if (CPG == 4 && (EXACT || OUT == OUT_DOTS)) {
            X += __shfl_xor_sync(kFull, X, 1);
            X += __shfl_xor_sync(kFull, X, 2);
        }
        Xg[t] = X;  // group sum (exact path) or chunk sum (per-32 path)
    }

    unsigned long long best[MT];  // OUT_ARGMAX: running best key per token (row threads)
#pragma unroll
    for (int t = 0; t < MT; ++t) best[t] = 0ull;

    for (int r = 0; r < rounds; ++r) {
        const int o0 = rb + r * rr;
        const int o1 = min(o0 + rr, re);
        if (r + 2 < rounds) {
            prefetch_weights(o0 + 2 * rr);
            prefetch_scales(o0 + 2 * rr);
        }
        uint32_t sv[U];
#pragma unroll
        for (int j = 0; j < U; ++j) {
            const int rl = r0t + (j % UH) * rpj;
            sv[j] = (worker && o0 + rl < o1 && (EXACT ? (c % CPG) == 0 : true)) ? scale_of(o0, j) : 0u;
        }
        // group terms of every chunk, summed over the segment
#pragma unroll
        for (int j = 0; j < U; ++j) {
            const int rl = r0t + (j % UH) * rpj;
            const bool ok = worker && o0 + rl < o1;
            const uint32_t sc = sv[j];
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                if (t >= m) break;
                int I = chunk_dot16(wv[j], xa[t], xb[t]);
                Term term;
                if (EXACT || OUT == OUT_DOTS) {
                    if (CPG == 4) {
                        I += __shfl_xor_sync(kFull, I, 1);
                        I += __shfl_xor_sync(kFull, I, 2);
                    }
                    if (OUT == OUT_DOTS) {
                        if (ok && (c % CPG) == 0)
                            p.dots[(static_cast<size_t>(t) * p.n_out + o0 + rl) * KG + g] = HAS_MIN ? I : I - 8 * Xg[t];
                        continue;
                    }
                    long long v = 0;
                    if ((c % CPG) == 0) {  // one lane of the group scales it
                        if (HAS_MIN) {
                            const Fix16 s = fix16(sc & 0xffffu), mn = fix16(sc >> 16);
                            v = shl64(s.mant * I, s.sh) + shl64(mn.mant * Xg[t], mn.sh);
                        } else {
                            const Fix16 s = fix16(sc);
                            v = shl64(s.mant * (I - 8 * Xg[t]), s.sh);
                        }
                    }
                    term = static_cast<Term>(v);
                } else {
                    // per-32 activation scales: one f32 term per chunk (gemv_q4q8.wgsl:68)
                    const uint32_t sw = sc;
                    const float s = __half2float(__ushort_as_half(static_cast<unsigned short>(sw & 0xffffu)));
                    float f;
                    if (HAS_MIN) {
                        const float mn = __half2float(__ushort_as_half(static_cast<unsigned short>(sw >> 16)));
                        f = s * dx[t] * static_cast<float>(I) + mn * dxs[t];
                    } else {
                        f = s * dx[t] * static_cast<float>(I - 8 * Xg[t]);
                    }
                    if (CPG == 4) {
                        f += __shfl_xor_sync(kFull, f, 1);
                        f += __shfl_xor_sync(kFull, f, 2);
                    }
                    term = static_cast<Term>((lane & (CPG - 1)) == 0 ? f : 0.0f);
                }
                // sum the segment's group terms (lanes CPG apart)
                if (seg == 8) {
                    for (int off = CPG; off < 8; off <<= 1) {
                        if (EXACT)
                            term += shfl_xor_i64(static_cast<long long>(term), off);
                        else
                            term += __shfl_xor_sync(kFull, term, off);
                    }
                }
                if (ok && lead)
                    red[((static_cast<size_t>(t) * NR + j / UH) * rr + rl) * nseg + c / seg] = term;
            }
        }
        // request the next round before this round's rows are summed
        if (r + 1 < rounds) load(o0 + rr);
        if (OUT == OUT_DOTS) continue;
        __syncthreads();

        // one thread per (token, row): add the segments in order
        const int nrow = o1 - o0;
        for (int i = tid; i < m * nrow; i += T) {
            const int t = i / nrow, rl = i - t * nrow;
            float val[NR];
#pragma unroll
            for (int h = 0; h < NR; ++h) {
                const Term* rp = red + ((static_cast<size_t>(t) * NR + h) * rr + rl) * nseg;
                Term a = rp[0];
                for (int s = 1; s < nseg; ++s) a += rp[s];
                float d = 1.0f;
#pragma unroll
                for (int tt = 0; tt < MT; ++tt)
                    if (tt == t) d = dx[tt];
                val[h] = EXACT ? fix_to_float(static_cast<long long>(a), d) : static_cast<float>(a);
            }
            const int row = o0 + rl;
            if (OUT == OUT_Y) {
                float* yp = p.y + static_cast<size_t>(t) * p.y_stride + row;
                if (MODE == W4A8_STORE)
                    *yp = val[0];
                else if (MODE == W4A8_ADD)
                    *yp = __fadd_rn(*yp, val[0]);
                else
                    *yp = silu_mul(val[0], val[NR - 1]);
            } else {
                if (p.y != nullptr) p.y[static_cast<size_t>(t) * p.y_stride + row] = val[0];
                const unsigned long long key = argmax_key(val[0], static_cast<uint32_t>(p.row_offset + row));
#pragma unroll
                for (int tt = 0; tt < MT; ++tt)
                    if (tt == t) best[tt] = key > best[tt] ? key : best[tt];
            }
        }
        __syncthreads();  // `red` is rewritten by the next round
    }

    if (OUT != OUT_ARGMAX) return;

    // CTA max of the running keys, one atomicMax per token, then the last CTA to
    // finish publishes the result and re-zeroes the workspace.
    __shared__ unsigned long long s_key[kGemvMaxThreads / 32][MT];
    __shared__ bool s_last;
    const int warp = tid >> 5, nwarps = (T + 31) >> 5;
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        unsigned long long key = best[t];
        for (int off = 1; off < 32; off <<= 1) {
            const unsigned long long o = shfl_xor_u64(key, off);
            key = o > key ? o : key;
        }
        if (lane == 0) s_key[warp][t] = key;
    }
    __syncthreads();
    if (tid < m) {
        unsigned long long key = 0;
        for (int w = 0; w < nwarps; ++w) {
            const unsigned long long o = s_key[w][tid];
            key = o > key ? o : key;
        }
        if (key) atomicMax(p.ws_best + tid, key);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned int done = atomicAdd(p.counter, 1u);
        s_last = (done == gridDim.x - 1);
    }
    __syncthreads();
    if (s_last) {
        __threadfence();
        if (tid < m) {
            const unsigned long long key = atomicExch(p.ws_best + tid, 0ull);
            p.best_key[tid] = key;
            if (p.tok_out) {
                const uint32_t idx = key ? ~static_cast<uint32_t>(key & 0xffffffffu) : 0u;
                p.tok_out[tid] = p.ids ? __ldg(p.ids + idx) : idx;
            }
        }
        if (tid == 0) *p.counter = 0u;
    }
}

// Host-side launch of the instantiation matching (group, has_min, act, mode, out, m).
w4a8_status launch_gemv(const GemvParams& p, int group, bool has_min, int act, int mode, int out,
                        cudaStream_t stream);

}  // namespace w4a8
