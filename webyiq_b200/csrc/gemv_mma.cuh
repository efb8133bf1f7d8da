// W4A8 GEMV on the warp-level integer tensor cores (mma.sync m16n8k32, u8 x s8),
// for group-128 weights with per-token int8 activations: y = W x for up to 8
// tokens per launch, the group-dot test hook and the lm_head GEMV with fused
// argmax.
//
// Why this shape (B200 view).  The GEMV streams packed weights from HBM once; the
// SM must turn every 16 weight bytes into dot products with as few instructions
// and as short dependency chains as possible, so that the post-wait critical
// path (activations in, math, outputs out) is short.  The packed words go into
// the tensor core unchanged:
//  - A packed word i holds weights 8i..8i+3 in its low nibbles and 8i+4..8i+7 in
//    its high nibbles (tools/convert.py:7-11).  w & 0x0F0F0F0F is the first four
//    as u8 bytes; w & 0xF0F0F0F0 is the other four times 16, still u8.  Each goes
//    into the tensor core against the raw int8 activation word it meets, in two
//    accumulators, and the exact int32 group dot is D_lo + (D_hi16 >> 4).  (The
//    int4 mma forms would take the packed words as they are, but they run far
//    slower than the int8 form on sm_100.)
//  - A = 16 weight rows x 32 k, B = 32 k x 8 tokens.  Lane (g, t) = (lane/4,
//    lane%4) loads 16 contiguous bytes (k-words 4t..4t+3 of a 128-group) of rows g
//    and g+8; per group that is two low-nibble and two high-nibble mma.  The D
//    fragment holds the group dots of rows g, g+8 for tokens 2t, 2t+1, and the
//    exact per-group scale step runs in the lanes that own those rows.
//  - A CTA (one per SM, persistent) owns a balanced contiguous row range, walked
//    in rounds of RT 16-row tiles; its warps are RT x KS (tile, K-slice) tasks of
//    up to 4 groups, so every lane holds at most 8 x 16 weight bytes, requested
//    before griddepcontrol.wait.  K-slice partial sums meet in shared memory and
//    are added in slice order (int64: exact anyway).
//
// Reference: gemv_q4q8.wgsl:36-131 (per-group math at :68, modes at :122-129),
// argmax.wgsl:14-43 for the fused argmax.  Numerics: the exact per-token path of
// w4a8.h, y = ((float)(sum_g fix(s)*(I - 8X) [+ fix(min)*X]) * 2^-24) * dx.
#pragma once

#include "gemv.cuh"
#include "tma.cuh"

namespace w4a8 {

constexpr int kMmaMaxWarps = 16;
constexpr int kMmaGPS = 4;      // groups per K-slice task
constexpr int kMmaTokens = 8;   // tokens of one mma block (the mma N)
constexpr int kMmaMaxTokens = 16;  // tokens per launch: the 8-token kernel runs two blocks over one weight pass
constexpr int kMmaMaxStages = 3;

// Set (atomicOr) by a kernel whose bounded wait gave up; read and cleared by
// w4a8_device_error.  Defined here: only gemv_mma.cu includes this header.
__device__ unsigned int g_w4a8_dev_error = 0;

struct MmaParams {
    const uint4* q;        // [rows, k/32] 16-byte chunks
    const void* s;         // scales: u16 f16 (symmetric) or u32 (scale, min)
    const int8_t* xq;      // [m, k]
    const float* xs;       // [m] per-token dx
    const float* xf32;     // [m, k] f32 activations to quantize here (xq, xs unused), or null
    float* y;              // OUT_Y output; OUT_ARGMAX logits or null
    int* dots;             // OUT_DOTS [m, n_out, k/128]
    unsigned int* counter;
    unsigned long long* ws_best;
    unsigned long long* best_key;
    unsigned int* tok_out;
    const unsigned int* ids;
    int n_out;      // output rows
    int k;
    int m;          // tokens (<= 8)
    int y_stride;
    int row_offset;
    int rt;         // tiles per round
    int ks;         // K-slices
    int stages;     // weight stages in shared memory
};

// Padded shared-memory row stride for k/2 weight bytes: stride = 80 (mod 128) makes
// the 32 lanes' 16-byte A-operand reads (rows gq, columns tq) hit every bank
// exactly 4 times, the minimum for 512 bytes.
__host__ __device__ inline int mma_row_stride(int k) {
    const int b = k / 2;
    return b + ((80 - b % 128) % 128 + 128) % 128;
}

// Shared memory: weight stages [S][rt*16 rows][stride], their scales
// [S][rt*16 rows][k/128] (rows in the order they are copied), activation operands
// [KG][m][4][8 words] (the 32 bytes lane-quarter t meets), per-group activation
// sums [KG][m], K-slice partial sums [rt][ks][16][m] (int64).
struct MmaSmem {
    size_t stage, stage_bytes, sc, sc_bytes, xf, xg, dx, red, bar, total;
};
__host__ __device__ inline MmaSmem mma_smem_plan(int m, int k, int rt, int ks, int stages, int sb) {
    MmaSmem s{};
    const size_t kg = static_cast<size_t>(k) / 128;
    auto up = [](size_t v) { return (v + 127) & ~static_cast<size_t>(127); };
    s.stage = 0;
    s.stage_bytes = static_cast<size_t>(rt) * 16 * mma_row_stride(k);
    s.sc = up(s.stage + stages * s.stage_bytes);        // scales [S][rt*16 rows][kg] (gate | up)
    s.sc_bytes = up(static_cast<size_t>(rt) * 16 * kg * sb);
    s.xf = up(s.sc + stages * s.sc_bytes);
    s.xg = s.xf + kg * m * 4 * 32;
    s.dx = up(s.xg + kg * m * 4);                       // per-token dx [8]
    s.red = up(s.dx + kMmaMaxTokens * 4);
    s.bar = up(s.red + static_cast<size_t>(rt) * ks * 16 * m * 8);
    s.total = s.bar + kMmaMaxStages * 8;
    return s;
}

__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One token: 64 registers, so the next kernel's CTA fits beside this one and its
// weight copies start while this one finishes.  More tokens: room for the epilogue,
// unless PAIR: at most 12 warps and 80 registers, so that two CTAs (this call's and
// the next one's) share an SM whenever the shared-memory plan fits twice.
constexpr int kMmaPairWarps = 12;
// dynamic shared bytes of a PAIR CTA: two of them, with their static arrays (< 512
// bytes) and the 1 KB the runtime reserves a CTA, fit in an SM's 228 KB
constexpr size_t kMmaPairSmem = 228 * 1024 / 2 - 1024 - 512;
template <int MT, bool PAIR>
struct MmaBounds {
    static constexpr int threads = PAIR ? kMmaPairWarps * 32 : kMmaMaxWarps * 32;
    static constexpr int min_blocks = (MT == 1 || PAIR) ? 2 : 1;
};

// FQ: the activations arrive as f32 (p.xf32) and are quantized per token here.
template <bool HAS_MIN, int MODE, int OUT, int MT, bool FQ, bool PAIR = false>
__global__ void __launch_bounds__(MmaBounds<MT, PAIR>::threads, MmaBounds<MT, PAIR>::min_blocks)
gemv_mma_kernel(const MmaParams p) {
    constexpr bool SWI = (MODE == W4A8_SWIGLU);
    constexpr int TR = SWI ? 8 : 16;  // output rows per tile
    extern __shared__ __align__(128) unsigned char smem[];

    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int gq = lane >> 2, tq = lane & 3;  // mma group / thread-in-group
    const int KC = p.k >> 5, KG = p.k >> 7;
    // MT: compile-time bound on the tokens of one mma block; the 8-token kernel takes
    // up to 16 tokens as two blocks that share each staged weight round
    const int m = MT == kMmaTokens ? min(p.m, kMmaMaxTokens) : min(MT, p.m);
    const int nblk = (m + kMmaTokens - 1) / kMmaTokens;
    const int rt = p.rt, ks = p.ks, S = p.stages;
    const int tile = warp / ks, slice = warp - tile * ks;  // this warp's task
    const bool active = tile < rt;
    const int g0 = static_cast<int>(static_cast<long long>(slice) * KG / ks);
    const int g1 = static_cast<int>(static_cast<long long>(slice + 1) * KG / ks);
    const int ng = g1 - g0;  // <= kMmaGPS (host guarantees)
    const int stride = mma_row_stride(p.k);
    // B column c carries token c % MT of the groups in slot c / CW (zeros for the
    // other groups), so the D registers of lane (gq, tq) accumulate ONE group per
    // accumulator set and the lanes of a quad share the per-group scale steps.
    constexpr int CW = MT >= 2 ? MT : 2;   // B columns per slot
    constexpr int NSLOT = 8 / CW;          // slots = groups per accumulator set (4, 4, 2, 1)
    constexpr int NSET = kMmaGPS / NSLOT;  // accumulator sets (1, 1, 2, 4)
    const int bslot = gq / CW, btok = gq % MT;  // B column gq
    const int dslot = (2 * tq) / CW;            // D columns 2tq, 2tq+1
    const int sb = HAS_MIN ? 4 : 2;
    const MmaSmem sp = mma_smem_plan(m, p.k, rt, ks, S, sb);
    // scales travel with the weights when a row of them is a whole number of
    // 16-byte units (k % 1024 == 0 symmetric, k % 512 == 0 with mins)
    const bool scale_tma = ((KG * sb) & 15) == 0;
    float* sdx = reinterpret_cast<float*>(smem + sp.dx);
    uint32_t* xf = reinterpret_cast<uint32_t*>(smem + sp.xf);
    int* xg = reinterpret_cast<int*>(smem + sp.xg);
    long long* red = reinterpret_cast<long long*>(smem + sp.red);

    const int rb = static_cast<int>(static_cast<long long>(blockIdx.x) * p.n_out / gridDim.x);
    const int re = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * p.n_out / gridDim.x);
    const int rows_round = rt * TR;
    const int rounds = (re - rb + rows_round - 1) / rows_round;

    // Every thread copies 16-byte pieces of round r into stage `slot` as one commit
    // group (cp.async: copies issued before griddepcontrol.wait then land while the
    // previous kernel still runs); a warp takes whole rows into their padded
    // shared-memory rows (A rows 0-7 gate / 8-15 up for SWIGLU).
    auto issue = [&](int r, int slot) {
        const int o0 = rb + r * rows_round;
        const int nrow = min(rows_round, re - o0);
        const int ncopy = (SWI ? 2 : 1) * nrow;
        const int nwarps = static_cast<int>(blockDim.x >> 5);
        unsigned char* st = smem + sp.stage + static_cast<size_t>(slot) * sp.stage_bytes;
        for (int i = warp; i < ncopy; i += nwarps) {
            const int h = SWI ? (i >= nrow) : 0;
            const int ri = i - h * nrow;
            const int srow = SWI ? (ri / 8) * 16 + (ri % 8) + 8 * h : ri;
            const uint4* src = p.q + (static_cast<size_t>(o0 + ri) + static_cast<size_t>(h) * p.n_out) * KC;
            unsigned char* dst = st + static_cast<size_t>(srow) * stride;
            for (int c = lane; c < KC; c += 32) cp_async16(dst + c * 16, src + c);
        }
        if (scale_tma) {  // [h][row][KG]: gate (or all) rows, then up rows
            const int srow_bytes = KG * sb, pieces = nrow * srow_bytes / 16;
            unsigned char* sdst = smem + sp.sc + static_cast<size_t>(slot) * sp.sc_bytes;
            for (int h = 0; h < (SWI ? 2 : 1); ++h) {
                const uint4* ssrc = reinterpret_cast<const uint4*>(
                    static_cast<const unsigned char*>(p.s) +
                    (static_cast<size_t>(o0) + static_cast<size_t>(h) * p.n_out) * srow_bytes);
                uint4* d = reinterpret_cast<uint4*>(sdst + static_cast<size_t>(h) * rows_round * srow_bytes);
                for (int i = tid; i < pieces; i += blockDim.x) cp_async16(d + i, ssrc + i);
            }
        }
        cp_async_commit();
    };
    // this thread's pieces of round r have landed (rounds up to r + S - 1 are issued)
    auto wait_round = [&](int r) { cp_async_wait_upto(min(r + S - 1, rounds - 1) - r); };
    auto prefetch_scales = [&](int r) {  // the fallback: the round's scale span towards L2
        if (scale_tma || tid != 0 || r >= rounds) return;
        const int o0 = rb + r * rows_round, o1 = min(o0 + rows_round, re);
        const size_t sb = HAS_MIN ? 4 : 2;
        for (int h = 0; h < (SWI ? 2 : 1); ++h) {
            const size_t r0 = static_cast<size_t>(o0) + static_cast<size_t>(h) * p.n_out;
            const size_t b0 = r0 * KG * sb, b1 = (r0 + (o1 - o0)) * KG * sb;
            const size_t a0 = (b0 + 15) & ~static_cast<size_t>(15), a1 = b1 & ~static_cast<size_t>(15);
            if (a1 > a0) l2_prefetch_bulk(static_cast<const unsigned char*>(p.s) + a0, static_cast<uint32_t>(a1 - a0));
        }
    };
    // stored rows behind A rows gq and gq+8 of this warp's tile in round r
    auto lane_rows = [&](int r, int& ra, int& rc, bool& oka, bool& okc) {
        const int t0 = rb + r * rows_round + tile * TR;
        ra = t0 + gq;
        rc = SWI ? t0 + gq + p.n_out : t0 + gq + 8;
        oka = active && t0 + gq < re;
        okc = active && (SWI ? t0 + gq < re : t0 + gq + 8 < re);
    };
    uint32_t sa[NSET], sc[NSET];  // scales of this lane's groups (set a: group a * NSLOT + dslot)
    auto load_scales = [&](int r) {  // the fallback when scales are not staged by TMA
        if (scale_tma) return;
        int ra, rc;
        bool oka, okc;
        lane_rows(r, ra, rc, oka, okc);
#pragma unroll
        for (int a = 0; a < NSET; ++a) {
            const int j = a * NSLOT + dslot;
            const size_t ea = static_cast<size_t>(ra) * KG + g0 + j, ec = static_cast<size_t>(rc) * KG + g0 + j;
            uint32_t& sj = sa[a];
            uint32_t& cj = sc[a];
            sj = cj = 0u;
            if (j < ng && oka)
                sj = HAS_MIN ? __ldg(static_cast<const uint32_t*>(p.s) + ea)
                                : static_cast<uint32_t>(__ldg(static_cast<const unsigned short*>(p.s) + ea));
            if (j < ng && okc)
                cj = HAS_MIN ? __ldg(static_cast<const uint32_t*>(p.s) + ec)
                                : static_cast<uint32_t>(__ldg(static_cast<const unsigned short*>(p.s) + ec));
        }
    };

    // Fused quant: per-token absmax, as float bits (non-negative, so they order
    // as unsigned integers), filled by shared-memory atomicMax.
    __shared__ unsigned int s_amax_bits[kMmaMaxTokens];
    __shared__ uint4 s_xzero[2];  // the activations a B column meets outside its slot
    if (tid < 2) s_xzero[tid] = make_uint4(0, 0, 0, 0);
    if (FQ && tid < kMmaMaxTokens) s_amax_bits[tid] = 0u;

    // Weights first: they do not depend on the previous kernel.  Each thread waits
    // for its own pieces of round 0 before the dependency wait.
    for (int r = 0; r < S && r < rounds; ++r) issue(r, r);
    if (rounds > 0) wait_round(0);
    prefetch_scales(0);
    prefetch_scales(1);
    pdl_launch_dependents();
    pdl_wait();  // activations (and y for ADD) come from the previous kernel

    load_scales(0);
    // Activation operands and group sums.  Work item (g, t, tq): the 32 bytes
    // x[t][128g + 32tq ..] that lane-quarter tq of the mma meets, stored as
    // [g][t][tq][8 words]; the quarter sums of a group are added by shuffles
    // (items of one (g, t) are 4 neighbouring threads).
    if (FQ) {
        // Per-token quantization fused in (quant.wgsl with one scale per token):
        // amax over the row, dx = amax / 127, inv = 1 / dx (0 for a zero row) and
        // rint(x * inv), exactly as w4a8_quant computes them, so the result equals
        // w4a8_quant followed by this GEMV bit for bit.  Every CTA quantizes the
        // rows it needs (they come from L2).  When every work item has a thread
        // (the decode case), the item's 32 inputs stay in registers across the
        // absmax exchange: one pass over x.
        __syncthreads();  // s_amax_bits zeroed
        const int nitem = KG * m * 4;
        // 32 inputs of item i -> int8 words in xf, their sum returned
        auto put = [&](int i, const float (&e)[32], float inv) -> int {
            int X = 0;
            uint32_t wd[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const int q0 = static_cast<int>(rintf(__fmul_rn(e[4 * c], inv)));
                const int q1 = static_cast<int>(rintf(__fmul_rn(e[4 * c + 1], inv)));
                const int q2 = static_cast<int>(rintf(__fmul_rn(e[4 * c + 2], inv)));
                const int q3 = static_cast<int>(rintf(__fmul_rn(e[4 * c + 3], inv)));
                X += q0 + q1 + q2 + q3;
                wd[c] = (static_cast<uint32_t>(q0) & 0xffu) | ((static_cast<uint32_t>(q1) & 0xffu) << 8) |
                        ((static_cast<uint32_t>(q2) & 0xffu) << 16) | ((static_cast<uint32_t>(q3) & 0xffu) << 24);
            }
            uint4* dst = reinterpret_cast<uint4*>(xf + static_cast<size_t>(i) * 8);
            dst[0] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
            dst[1] = make_uint4(wd[4], wd[5], wd[6], wd[7]);
            return X;
        };
        auto load = [&](int i, float (&e)[32]) -> int {  // returns the item's token
            const int tq2 = i & 3, t = (i >> 2) % m, g = (i >> 2) / m;
            const float4* src =
                reinterpret_cast<const float4*>(p.xf32 + static_cast<size_t>(t) * p.k + g * 128 + tq2 * 32);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const float4 v = ld_dep(src + c);
                e[4 * c] = v.x;
                e[4 * c + 1] = v.y;
                e[4 * c + 2] = v.z;
                e[4 * c + 3] = v.w;
            }
            return t;
        };
        auto local_max = [](const float (&e)[32]) -> float {
            float a = 0.0f;
#pragma unroll
            for (int c = 0; c < 32; ++c) a = fmaxf(a, fabsf(e[c]));
            return a;
        };
        auto inv_of = [&](int t) -> float {
            const float a = __uint_as_float(s_amax_bits[t]);
            return a > 0.0f ? __fdiv_rn(1.0f, __fdiv_rn(a, 127.0f)) : 0.0f;
        };
        if (nitem <= static_cast<int>(blockDim.x)) {
            float e[32];
            int t = 0;
            if (tid < nitem) {
                t = load(tid, e);
                atomicMax(&s_amax_bits[t], __float_as_uint(local_max(e)));
            }
            __syncthreads();
            int X = 0;
            if (tid < nitem) X = put(tid, e, inv_of(t));
            X += __shfl_xor_sync(kFull, X, 1);
            X += __shfl_xor_sync(kFull, X, 2);
            if (tid < nitem && (tid & 3) == 0) xg[tid >> 2] = X;  // [g][t]
        } else {
            for (int i = tid; i < nitem; i += blockDim.x) {
                float e[32];
                const int t = load(i, e);
                atomicMax(&s_amax_bits[t], __float_as_uint(local_max(e)));
            }
            __syncthreads();
            for (int i0 = 0; i0 < nitem; i0 += blockDim.x) {
                const int i = i0 + tid;
                int X = 0;
                if (i < nitem) {
                    float e[32];
                    const int t = load(i, e);
                    X = put(i, e, inv_of(t));
                }
                X += __shfl_xor_sync(kFull, X, 1);
                X += __shfl_xor_sync(kFull, X, 2);
                if (i < nitem && (i & 3) == 0) xg[i >> 2] = X;  // [g][t]
            }
        }
        if (OUT != OUT_DOTS && tid < m) sdx[tid] = __fdiv_rn(__uint_as_float(s_amax_bits[tid]), 127.0f);
    } else {
        if (OUT != OUT_DOTS && tid < m) sdx[tid] = ld_dep(p.xs + tid);  // the dots hook has no xs
        // Up to four items a thread are requested before any is used, so that a
        // pass costs one round trip, not one per item (one token: one item a thread).
        constexpr int kIt = MT == 1 ? 1 : 4;
        const int nitem = KG * m * 4;
        for (int i0 = 0; i0 < nitem; i0 += kIt * blockDim.x) {
            uint4 u[kIt], v[kIt];
#pragma unroll
            for (int b = 0; b < kIt; ++b) {
                const int i = i0 + b * blockDim.x + tid;
                if (i < nitem) {
                    const int tq2 = i & 3, t = (i >> 2) % m, g = (i >> 2) / m;
                    const uint4* src = reinterpret_cast<const uint4*>(p.xq + static_cast<size_t>(t) * p.k + g * 128 + tq2 * 32);
                    u[b] = ld_dep(src);
                    v[b] = ld_dep(src + 1);
                }
            }
#pragma unroll
            for (int b = 0; b < kIt; ++b) {
                const int i = i0 + b * blockDim.x + tid;
                int X = 0;
                if (i < nitem) {
                    uint4* dst = reinterpret_cast<uint4*>(xf + static_cast<size_t>(i) * 8);
                    dst[0] = u[b];
                    dst[1] = v[b];
                    X = chunk_sum(u[b], v[b]);
                }
                X += __shfl_xor_sync(kFull, X, 1);
                X += __shfl_xor_sync(kFull, X, 2);
                if (i < nitem && (i & 3) == 0) xg[i >> 2] = X;  // [g][t]
            }
        }
    }
    __syncthreads();

    unsigned long long best[MT];  // OUT_ARGMAX: running best key per token (finalizing threads)
#pragma unroll
    for (int t = 0; t < MT; ++t) best[t] = 0ull;

    for (int r = 0; r < rounds; ++r) {
        const int slot = r % S;
        if (r > 0) {  // round 0 landed before the dependency wait
            wait_round(r);
            __syncthreads();
        }
        prefetch_scales(r + 2);
        int ra, rc;
        bool oka, okc;
        lane_rows(r, ra, rc, oka, okc);
        const unsigned char* st = smem + sp.stage + static_cast<size_t>(slot) * sp.stage_bytes;
        const unsigned char* scs = smem + sp.sc + static_cast<size_t>(slot) * sp.sc_bytes;
        // staged scale rows of A rows gq and gq+8 (index [h][row in round][g])
        const int ria = SWI ? tile * TR + gq : tile * 16 + gq;
        const int ric = SWI ? rows_round + ria : ria + 8;
        const unsigned char* rowa = st + static_cast<size_t>(tile * 16 + gq) * stride + tq * 16;
        const unsigned char* rowc = rowa + static_cast<size_t>(8) * stride;
        for (int tb = 0; tb < nblk; ++tb) {  // token blocks of 8 (one unless MT == 8 and m > 8)
        const int tb0 = tb * kMmaTokens, mb = m - tb0;  // this block's first token, tokens left
        // two accumulators per set (by group parity) when a set takes several
        // groups, so that the dependent mma chains stay short
        constexpr int NSUB = NSLOT > 1 ? 2 : 1;
        int dl[NSET][NSUB][4], dh[NSET][NSUB][4];
#pragma unroll
        for (int a = 0; a < NSET; ++a)
#pragma unroll
            for (int u = 0; u < NSUB; ++u)
#pragma unroll
                for (int e = 0; e < 4; ++e) dl[a][u][e] = dh[a][u][e] = 0;
        // the exact per-group scale step of this lane's groups of set a; element e:
        // A row gq (e < 2) or gq+8, D column 2tq + (e & 1) = token (2tq + (e & 1)) % MT
        long long acc[4] = {0, 0, 0, 0};
        auto finish = [&](int a) {
            const int jj = a * NSLOT + dslot;
            if (jj >= ng) return;
            const int gg = g0 + jj;
            // the raw scale words of rows gq and gq+8 for this group
            uint32_t s2[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (scale_tma) {
                    const size_t si = static_cast<size_t>(h == 0 ? ria : ric) * KG + gg;
                    s2[h] = HAS_MIN ? reinterpret_cast<const uint32_t*>(scs)[si]
                                    : static_cast<uint32_t>(reinterpret_cast<const unsigned short*>(scs)[si]);
                } else {
                    s2[h] = h == 0 ? sa[a] : sc[a];
                }
            }
            // fix(s) = mant * 2^sh as one int64 per row, so that a step is one wide
            // multiply-add: D * (mant << sh) == (mant * D) << sh exactly (|mant * D| <
            // 2^28, |result| < 2^58)
            long long fsc[2] = {0, 0}, fmn[2] = {0, 0};
            if (OUT != OUT_DOTS) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const Fix16 fs = fix16(HAS_MIN ? (s2[h] & 0xffffu) : s2[h]);
                    fsc[h] = shl64(fs.mant, fs.sh);
                    if (HAS_MIN) {
                        const Fix16 fm = fix16(s2[h] >> 16);
                        fmn[h] = shl64(fm.mant, fm.sh);
                    }
                }
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (MT == 1 && (e & 1)) continue;  // both D columns hold token 0
                const int t = MT == 1 ? 0 : (2 * tq + (e & 1)) % MT;
                if (t >= mb) continue;
                int lo = dl[a][0][e], hi = dh[a][0][e];
                if (NSUB == 2) {
                    lo += dl[a][NSUB - 1][e];
                    hi += dh[a][NSUB - 1][e];
                }
                const int I = lo + (hi >> 4);  // hi = 16 * high-nibble dot, exact
                const int X = xg[gg * m + tb0 + t];
                if (OUT == OUT_DOTS) {
                    const bool ok = e < 2 ? oka : okc;
                    const int row = e < 2 ? ra : rc;
                    if (ok) p.dots[(static_cast<size_t>(tb0 + t) * p.n_out + row) * KG + gg] = HAS_MIN ? I : I - 8 * X;
                } else if (HAS_MIN) {
                    acc[e] += static_cast<long long>(I) * fsc[e >> 1] + static_cast<long long>(X) * fmn[e >> 1];
                } else {
                    acc[e] += static_cast<long long>(I - 8 * X) * fsc[e >> 1];
                }
            }
        };
        // one group a set (8 tokens): each set is finished right after its mma, so
        // that its accumulators die early (four live sets would spill); otherwise
        // all sets after the last mma
        constexpr bool EARLY = NSLOT == 1;
#pragma unroll
        for (int j = 0; j < kMmaGPS; ++j) {
            if (j >= ng) break;
            const int g = g0 + j;
            uint4 wa = make_uint4(0, 0, 0, 0), wc = make_uint4(0, 0, 0, 0);
            if (active) {
                wa = *reinterpret_cast<const uint4*>(rowa + g * 64);
                wc = *reinterpret_cast<const uint4*>(rowc + g * 64);
            }
            // B column gq: token btok's activations if group j is in its slot
            const bool mine = (j % NSLOT) == bslot && btok < mb;
            const uint4* xp = mine ? reinterpret_cast<const uint4*>(xf + ((static_cast<size_t>(g) * m + tb0 + btok) * 4 + tq) * 8)
                                   : s_xzero;
            const uint4 x0 = xp[0];  // activations of k-words 0, 1 (low 4, high 4 each)
            const uint4 x1 = xp[1];  // k-words 2, 3
            const uint32_t ml = 0x0F0F0F0Fu, mh = 0xF0F0F0F0u;
            int (&sl)[4] = dl[j / NSLOT][j % NSUB];
            int (&sh)[4] = dh[j / NSLOT][j % NSUB];
            // k-words w0, w1 of rows gq (wa) and gq+8 (wc); A k-slots 0-3 / 16-19
            // of this lane meet B words 0 / 1 of the same lane
            mma_u8s8(sl, wa.x & ml, wc.x & ml, wa.y & ml, wc.y & ml, x0.x, x0.z);
            mma_u8s8(sl, wa.z & ml, wc.z & ml, wa.w & ml, wc.w & ml, x1.x, x1.z);
            mma_u8s8(sh, wa.x & mh, wc.x & mh, wa.y & mh, wc.y & mh, x0.y, x0.w);
            mma_u8s8(sh, wa.z & mh, wc.z & mh, wa.w & mh, wc.w & mh, x1.y, x1.w);
            if (EARLY) finish(j);
        }
        if (!EARLY) {
#pragma unroll
            for (int a = 0; a < NSET; ++a) finish(a);
        }
        // lanes of a quad holding the same rows and tokens (other groups) add up
        if (OUT != OUT_DOTS && MT <= 4) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (MT == 1 && (e & 1)) continue;
                if (MT <= 2) acc[e] += shfl_xor_i64(acc[e], 1);
                acc[e] += shfl_xor_i64(acc[e], 2);
            }
        }
        const bool writer = MT <= 2 ? tq == 0 : (MT == 4 ? tq < 2 : true);
        if (OUT != OUT_DOTS && active && writer) {  // K-slice partial sums: red[tile][slice][A row][token]
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (MT == 1 && (e & 1)) continue;
                const int t = MT == 1 ? 0 : (2 * tq + (e & 1)) % MT;
                const int arow = gq + (e >= 2 ? 8 : 0);
                if (t < mb) red[((static_cast<size_t>(tile) * ks + slice) * 16 + arow) * m + tb0 + t] = acc[e];
            }
        }
        }  // token blocks
        if (r + 1 < rounds) load_scales(r + 1);
        __syncthreads();  // every warp is done with stage `slot` and has stored its sums
        if (r + S < rounds) issue(r + S, slot);
        if (OUT == OUT_DOTS) continue;
        // one thread per (output row, token): add the slices in order
        const int nout = min(rows_round, re - (rb + r * rows_round));
        for (int i = tid; i < nout * m; i += blockDim.x) {
            const int t = i % m, orow = i / m;  // output row within the round
            const int tl = orow / TR, rw = orow - tl * TR;
            long long a0 = 0, a1 = 0;
            for (int s2 = 0; s2 < ks; ++s2) {
                a0 += red[((static_cast<size_t>(tl) * ks + s2) * 16 + rw) * m + t];
                if (SWI) a1 += red[((static_cast<size_t>(tl) * ks + s2) * 16 + rw + 8) * m + t];
            }
            const float dx = sdx[t];
            const float v0 = fix_to_float(a0, dx);
            const int row = rb + r * rows_round + orow;
            if (OUT == OUT_Y) {
                float* yp = p.y + static_cast<size_t>(t) * p.y_stride + row;
                if (MODE == W4A8_STORE)
                    *yp = v0;
                else if (MODE == W4A8_ADD)
                    *yp = __fadd_rn(*yp, v0);
                else
                    *yp = silu_mul(v0, fix_to_float(a1, dx));
            } else {
                if (p.y != nullptr) p.y[static_cast<size_t>(t) * p.y_stride + row] = v0;
                const unsigned long long key = argmax_key(v0, static_cast<uint32_t>(p.row_offset + row));
#pragma unroll
                for (int tt = 0; tt < MT; ++tt)
                    if (tt == t) best[tt] = key > best[tt] ? key : best[tt];
            }
        }
        __syncthreads();  // `red` is rewritten by the next round
    }

    if (OUT != OUT_ARGMAX) return;

    // Max per token over the CTA, one atomicMax per token, and the last CTA to
    // finish publishes the result and re-zeroes the workspace.
    __shared__ unsigned long long s_key[kMmaMaxWarps][MT];
    __shared__ bool s_last;
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
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) key = s_key[w][tid] > key ? s_key[w][tid] : key;
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

}  // namespace w4a8
