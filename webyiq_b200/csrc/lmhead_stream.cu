// lm_head GEMV with fused argmax for group-128 weights and per-token activations,
// written as a streaming kernel: the vocabulary matrix (262 MB at 248,320 x 2048)
// is read once from HBM, so the kernel is built to keep HBM busy rather than
// around a per-round CTA barrier.
//
// Reference: head_ops (graph.rs:476-486) = lm_head GEMV (gemv_q4q8.wgsl:36-131) +
// argmax (argmax.wgsl:14-43).  Numerics are the exact per-token path of w4a8.h
// (int64 sum of fix16(s) * (I - 8 X) per row, then ((float)acc * 2^-24) * dx), so
// keys and tokens are bit-identical to the other GEMV kernels and to the oracle.
//
// Layout of the work (one CTA per SM, persistent on a contiguous range of rows):
//  - Rows [o0, o0 + R) of the weights are one contiguous span, and so are their
//    scales: one bulk copy each per stage into a ring of kStages stages (about 64 KB
//    of weights per stage).  Thread 0 fills the ring before the kernel waits for
//    the previous one (the weights do not depend on it); after that the last warp
//    to finish a stage refills its slot, so there is no producer warp and all 16
//    warps have 128 registers a thread.
//  - The consumers are integer-issue bound (a 64 KB stage arrives about every
//    1.5 us per SM at full HBM rate), so every lane does only useful work: L lanes
//    share a row and each owns GPL whole 128-groups of it.  A lane forms the exact
//    int32 group dot of its 4 x GPL 16-byte chunks with dp4a (low and high nibbles
//    in separate accumulators, combined once per group), applies the group's exact
//    scale step in int64, and the L lanes add their int64 sums by log2(L)
//    shuffles.  The lane's activation chunks stay in registers for the whole
//    kernel (32 x GPL registers per token).
//  - Bank conflicts: the rows are copied as they lie in HBM (no padding), so each
//    lane walks its chunks in a rotated order that sends the 8 lanes of every
//    16-byte shared-memory phase to 8 distinct 16-byte bank groups; the rotation
//    stays inside a group, so the group of each step is a per-lane constant.
//  - A warp releases a stage with one shared atomic; no CTA-wide barrier runs per
//    stage.  At the end the CTA's best key per token goes through the same
//    workspace protocol as w4a8_lmhead_argmax (atomicMax, done counter, the last
//    CTA publishes and re-zeroes).  For a vocabulary shard of the column-split
//    lm_head (w4a8_lmhead_argmax_xchg) the last CTA instead merges the keys with
//    the peers over NVLink (xchg.cuh), so the sharded call is one kernel.
// Every wait is bounded; a wait that gives up sets the device error word.
#include <cuda_fp16.h>

#include "gemv.cuh"
#include "launch.cuh"
#include "tma.cuh"
#include "xchg.cuh"

namespace w4a8 {

int sm_count();                     // capi.cu
unsigned int* device_error_word();  // gemv_mma.cu

namespace {

constexpr int kStages = 3;
constexpr int kConsumers = 16;                   // warps, all consumers
constexpr int kThreads = kConsumers * 32;
constexpr uint32_t kStageTarget = 64 * 1024;     // weight bytes per stage (at most)
constexpr int kMaxRows = 128;                    // rows per stage (at most)

struct StreamParams {
    const unsigned char* q;  // [n][k/2]
    const unsigned char* s;  // [n][kg] u16 (symmetric) or u32 (scale, min)
    const int8_t* xq;        // [m][k]
    const float* xs;         // [m] per-token dx
    float* logits;           // [m][n] or null
    unsigned int* counter;
    unsigned long long* ws_best;
    unsigned long long* best_key;
    unsigned int* tok_out;
    const unsigned int* ids;
    unsigned int* err;
    int n, k, m, row_offset;
    int rows_per_stage;    // R, a multiple of 8
    uint32_t stage_bytes;  // R * k/2 + the scale span, 128-byte multiple
    XchgArgs xchg;         // world > 0: the last CTA merges the keys over the peers (xchg.cuh)
};

// Lanes per row (L) and groups per lane (GPL) for kg groups per row and mt tokens:
// the smallest L in {8, 16, 32} whose lanes cover the row with GPL * mt <= 2 (the
// activation registers a lane holds); L = 0 when none does.
struct SpanShape {
    int L, gpl;
};
__host__ __device__ inline SpanShape span_shape(int kg, int mt) {
    const int gmax = mt == 1 ? 2 : 1;
    for (int L = 8; L <= 32; L <<= 1)
        if (kg <= L * gmax) return {L, (kg + L - 1) / L};
    return {0, 0};
}

// Rows per stage: as many as fit kStageTarget, a multiple of one CTA pass
// (kConsumers * 32 / L rows) when at least one pass fits, else a multiple of 8.
inline int stream_rows(int k, int L) {
    int r = static_cast<int>(2 * kStageTarget / static_cast<uint32_t>(k));
    r = r > kMaxRows ? kMaxRows : r;
    const int pass = kConsumers * 32 / L;
    if (r >= pass) return r - r % pass;
    return r < 8 ? 8 : (r & ~7);
}

template <bool HAS_MIN, int MT, int L, int GPL>
__global__ void __launch_bounds__(kThreads, 1) lmhead_stream_kernel(const StreamParams p) {
    constexpr int kSteps = 4 * GPL;  // 16-byte chunks per lane per row
    constexpr int kRowsPerWarp = 32 / L;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t full[kStages];
    __shared__ int s_done[kStages];  // warps that finished the slot, over all its uses
    __shared__ int s_issued;         // stages whose copies were issued
    __shared__ unsigned long long s_key[kConsumers][MT];
    __shared__ bool s_last;
    __shared__ volatile int s_abort;
    __shared__ unsigned int s_xseq;  // the exchange's sequence number (shards of a column-split head)

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = p.k, KG = K >> 7;
    const int sb = HAS_MIN ? 4 : 2;
    const int R = p.rows_per_stage;
    const uint32_t wbytes = static_cast<uint32_t>(R) * static_cast<uint32_t>(K / 2);
    // CTA row range: whole blocks of 8 rows (so every copy is 16-byte aligned)
    const int nblk = p.n / 8;
    const int rb = static_cast<int>(static_cast<long long>(blockIdx.x) * nblk / gridDim.x) * 8;
    const int re = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * nblk / gridDim.x) * 8;
    const int nst = (re - rb + R - 1) / R;

    // Copies stage i (rows rb + i*R ...) into its ring slot; one thread issues it.
    auto issue = [&](int i) {
        const int s = i % kStages;
        const int o0 = rb + i * R, nrow = min(R, re - o0);
        const uint32_t wb = static_cast<uint32_t>(nrow) * static_cast<uint32_t>(K / 2);
        const uint32_t scb = static_cast<uint32_t>(nrow) * static_cast<uint32_t>(KG * sb);
        unsigned char* st = smem + static_cast<size_t>(s) * p.stage_bytes;
        mbar_expect_tx(&full[s], wb + scb);
        tma_bulk_load(st + wbytes, p.s + static_cast<size_t>(o0) * KG * sb, scb, &full[s]);
        tma_bulk_load(st, p.q + static_cast<size_t>(o0) * (K / 2), wb, &full[s]);
    };

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            s_done[s] = 0;
        }
        s_abort = 0;
        mbar_init_fence();
        const int first = nst < kStages ? nst : kStages;
        for (int i = 0; i < first; ++i) issue(i);
        s_issued = first;
    }
    __syncthreads();
    pdl_launch_dependents();

    {
        const int cw = warp;
        const int j = lane % L;   // this lane's span of the row: groups [j*GPL, j*GPL + GPL)
        const int ph = lane & 7;  // position in its 16-byte shared-memory phase
        // rotation: step c reads chunk (c%4 + rc) % 4 of group j*GPL + (c/4 + rg) % GPL
        const int rg = (GPL % 2 == 0) ? (ph >> 2) & 1 : 0;
        const int rc = (GPL % 2 == 0) ? (ph & 3) : ((ph >> 1) & 3);
        int gidx[GPL];  // the group of slot g (steps 4g..4g+3)
        bool gin[GPL];  // false past the row's end
#pragma unroll
        for (int g = 0; g < GPL; ++g) {
            gidx[g] = j * GPL + (g + rg) % GPL;
            gin[g] = gidx[g] < KG;
        }
        int coff[kSteps];  // byte offset of step c's chunk in the packed row
#pragma unroll
        for (int c = 0; c < kSteps; ++c) coff[c] = (gidx[c / 4] * 4 + (c % 4 + rc) % 4) * 16;

        pdl_wait();  // the activations come from the previous kernel
        if (p.xchg.world > 0 && tid == 0) s_xseq = xchg_next_seq(p.xchg);  // off the merge's critical path
        uint4 xa[MT][kSteps], xb[MT][kSteps];
        int Xg[MT][GPL];
        float dx[MT];
        unsigned long long best[MT];
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            best[t] = 0ull;
            dx[t] = t < p.m ? ld_dep(p.xs + t) : 0.0f;
#pragma unroll
            for (int g = 0; g < GPL; ++g) Xg[t][g] = 0;
#pragma unroll
            for (int c = 0; c < kSteps; ++c) {
                xa[t][c] = xb[t][c] = make_uint4(0, 0, 0, 0);
                if (t < p.m && gin[c / 4]) {
                    const uint4* xp = reinterpret_cast<const uint4*>(p.xq + static_cast<size_t>(t) * K + coff[c] * 2);
                    xa[t][c] = ld_dep(xp);
                    xb[t][c] = ld_dep(xp + 1);
                }
                Xg[t][c / 4] += chunk_sum(xa[t][c], xb[t][c]);  // the group's activation sum
            }
        }
        for (int i = 0; i < nst; ++i) {
            const int s = i % kStages, u = i / kStages;
            const bool ok = !s_abort && mbar_wait(&full[s], u & 1);
            if (!__all_sync(kFull, ok)) {
                if (lane == 0) {
                    s_abort = 1;
                    atomicOr(p.err, DEV_ERR_TMA_TIMEOUT);
                }
                break;
            }
            const int o0 = rb + i * R, nrow = min(R, re - o0);
            const unsigned char* st = smem + static_cast<size_t>(s) * p.stage_bytes;
            const unsigned char* sc = st + wbytes;
            for (int rw = cw * kRowsPerWarp; rw < nrow; rw += kConsumers * kRowsPerWarp) {
                const int rl = rw + lane / L;
                const bool rin = rl < nrow;
                const unsigned char* row = st + static_cast<size_t>(rin ? rl : 0) * (K / 2);
                uint4 w[kSteps];
#pragma unroll
                for (int c = 0; c < kSteps; ++c)
                    w[c] = (rin && gin[c / 4]) ? *reinterpret_cast<const uint4*>(row + coff[c]) : make_uint4(0, 0, 0, 0);
                uint32_t sv[GPL];
#pragma unroll
                for (int g = 0; g < GPL; ++g) {
                    const size_t e = static_cast<size_t>(rl) * KG + gidx[g];
                    sv[g] = 0u;
                    if (rin && gin[g])
                        sv[g] = HAS_MIN ? reinterpret_cast<const uint32_t*>(sc)[e]
                                        : static_cast<uint32_t>(reinterpret_cast<const unsigned short*>(sc)[e]);
                }
                long long acc[MT];
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    acc[t] = 0;
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
                        if (HAS_MIN) {
                            const Fix16 fs = fix16(sv[g] & 0xffffu), fm = fix16(sv[g] >> 16);
                            acc[t] += shl64(fs.mant * I, fs.sh) + shl64(fm.mant * Xg[t][g], fm.sh);
                        } else {
                            const Fix16 fs = fix16(sv[g]);
                            acc[t] += shl64(fs.mant * (I - 8 * Xg[t][g]), fs.sh);
                        }
                    }
                }
#pragma unroll
                for (int off = 1; off < L; off <<= 1)
#pragma unroll
                    for (int t = 0; t < MT; ++t) acc[t] += shfl_xor_i64(acc[t], off);
                if (j == 0 && rin) {
#pragma unroll
                    for (int t = 0; t < MT; ++t) {
                        if (t < p.m) {
                            const float v = fix_to_float(acc[t], dx[t]);
                            const int grow = o0 + rl;
                            if (p.logits) p.logits[static_cast<size_t>(t) * p.n + grow] = v;
                            const unsigned long long key = argmax_key(v, static_cast<uint32_t>(p.row_offset + grow));
                            best[t] = key > best[t] ? key : best[t];
                        }
                    }
                }
            }
            // release the slot; the last warp out refills it with stage i + kStages
            __syncwarp();
            if (lane == 0) {
                __threadfence_block();  // this warp's reads of the slot come before the count
                const int done = atomicAdd(&s_done[s], 1) + 1;
                if (done == (u + 1) * kConsumers && i + kStages < nst) {
                    __threadfence_block();
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    issue(i + kStages);
                    atomicMax(&s_issued, i + kStages + 1);
                }
            }
        }
        // the warp's best key per token (the row leaders hold the candidates)
#pragma unroll
        for (int t = 0; t < MT; ++t) {
#pragma unroll
            for (int off = L; off < 32; off <<= 1) {
                const unsigned long long o = __shfl_xor_sync(kFull, best[t], off);
                best[t] = o > best[t] ? o : best[t];
            }
            if (lane == 0) s_key[cw][t] = best[t];
        }
    }
    __syncthreads();
    const bool aborted = s_abort;
    if (aborted && tid == 0) {
        // no copy may still be landing when the CTA exits
        for (int j = s_issued > kStages ? s_issued - kStages : 0; j < s_issued; ++j)
            mbar_wait(&full[j % kStages], (j / kStages) & 1);
    }

    // CTA max, one atomicMax per token, the last CTA publishes and re-zeroes.  A CTA
    // whose wait gave up adds no key but is still counted, so the workspace is left
    // zeroed for the next call whatever happened in this one.
    if (!aborted && tid < p.m) {
        unsigned long long key = 0;
        for (int w = 0; w < kConsumers; ++w) {
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
        if (p.xchg.world > 0) {
            // the shard's key goes straight into the exchange with the peers, so a
            // sharded call is this one kernel
            __shared__ unsigned long long s_own[MT];
            if (tid < p.m) s_own[tid] = atomicExch(p.ws_best + tid, 0ull);
            if (tid == 0) *p.counter = 0u;
            __syncthreads();
            xchg_merge(p.xchg, p.m, s_xseq, s_own, p.best_key, p.tok_out, p.ids, p.err);
            return;
        }
        if (tid < p.m) {
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

template <bool HAS_MIN, int MT, int L, int GPL>
w4a8_status launch_inst(const StreamParams& p, cudaStream_t st) {
    static FuncAttr attr;
    auto kernel = lmhead_stream_kernel<HAS_MIN, MT, L, GPL>;
    const size_t smem = static_cast<size_t>(kStages) * p.stage_bytes;
    const w4a8_status a = ensure_smem(kernel, attr, smem, -1, "w4a8 lm_head (stream)");
    if (a != W4A8_OK) return a;
    int ctas = sm_count();
    const int nblk = p.n / 8;
    if (ctas > nblk) ctas = nblk;
    return launch_pdl("w4a8 lm_head (stream)", kernel, dim3(ctas), dim3(kThreads), smem, st, p);
}

template <bool HAS_MIN>
w4a8_status launch_shape(const StreamParams& p, SpanShape sh, cudaStream_t st) {
    if (p.m == 1) {
        if (sh.L == 8) return sh.gpl == 1 ? launch_inst<HAS_MIN, 1, 8, 1>(p, st) : launch_inst<HAS_MIN, 1, 8, 2>(p, st);
        if (sh.L == 16) return launch_inst<HAS_MIN, 1, 16, 2>(p, st);
        return launch_inst<HAS_MIN, 1, 32, 2>(p, st);
    }
    if (sh.L == 8) return launch_inst<HAS_MIN, 2, 8, 1>(p, st);
    if (sh.L == 16) return launch_inst<HAS_MIN, 2, 16, 1>(p, st);
    return launch_inst<HAS_MIN, 2, 32, 1>(p, st);
}

}  // namespace

// Whether the streaming lm_head covers this call (otherwise the dp4a GEMV runs it):
// group 128, per-token activations, one or two tokens, whole 8-row blocks, rows of
// at most 64 groups (32 for two tokens), 16-byte aligned scales.
bool lmhead_stream_covers(const GemvParams& g, int group, int act) {
    if (group != 128 || act != W4A8_ACT_TOKEN || g.m < 1 || g.m > 2 || g.n_out % 8 != 0 || g.k % 128 != 0) return false;
    if (span_shape(g.k / 128, g.m).L == 0) return false;
    return (reinterpret_cast<uintptr_t>(g.s) & 15) == 0;
}

w4a8_status launch_lmhead_stream(const GemvParams& g, bool has_min, cudaStream_t st) {
    StreamParams p{};
    p.q = reinterpret_cast<const unsigned char*>(g.q);
    p.s = static_cast<const unsigned char*>(g.s);
    p.xq = g.xq;
    p.xs = g.xs;
    p.logits = g.y;
    p.counter = g.counter;
    p.ws_best = g.ws_best;
    p.best_key = g.best_key;
    p.tok_out = g.tok_out;
    p.ids = g.ids;
    p.err = device_error_word();
    if (!p.err) return set_error(W4A8_ECUDA, "w4a8 lm_head: device error word unavailable");
    p.n = g.n_out;
    p.k = g.k;
    p.m = g.m;
    p.row_offset = g.row_offset;
    if (g.xchg) p.xchg = *g.xchg;
    const SpanShape sh = span_shape(g.k / 128, g.m);
    if (sh.L == 0) return set_error(W4A8_EINVAL, "w4a8 lm_head (stream): k=%d not covered", g.k);
    p.rows_per_stage = stream_rows(g.k, sh.L);
    const uint32_t sb = has_min ? 4 : 2;
    const uint32_t wb = static_cast<uint32_t>(p.rows_per_stage) * static_cast<uint32_t>(g.k / 2);
    const uint32_t scb = static_cast<uint32_t>(p.rows_per_stage) * static_cast<uint32_t>(g.k / 128) * sb;
    p.stage_bytes = (wb + scb + 127u) & ~127u;
    return has_min ? launch_shape<true>(p, sh, st) : launch_shape<false>(p, sh, st);
}

}  // namespace w4a8
