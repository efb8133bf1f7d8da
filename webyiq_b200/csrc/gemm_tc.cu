// W4A8 prefill GEMM on the 5th-generation tensor cores: tcgen05.mma kind::i8 with
// the accumulators in tensor memory (TMEM), for group-128 symmetric int4 weights
// and per-token int8 activations:
//
//     y[m, n] = dx[m] * sum_g s[n, g] * I[m, n, g],   I = sum_{k in g} (q[n,k] - 8) * xq[m, k]
//
// Reference: gemm_q4q8.wgsl:46-121 (the tiled prefill GEMM; its per-group math is
// the GEMV's, gemv_q4q8.wgsl:29-34,68, and the output modes are those of
// gemv_q4q8.wgsl:122-129).  The per-group int32 dots I are exact; the scale step
// is fp32 (y within 1e-6 relative of the exact path), not the bit-exact int64
// step of the GEMV kernels.
//
// Why this shape (B200 view).
//  - Weight rows are the MMA M (128, one TMEM lane per row) and tokens the MMA N
//    (128 columns).  The per-group scale s[n, g] is then a per-lane constant, so
//    the epilogue thread that owns a row multiplies every column it reads by one
//    register.
//  - The int4 -> int8 step writes 16*(q-8) into each byte: the nibble q^8 (the
//    4-bit two's complement of q-8) lands in the high half of the byte, so its
//    sign extends for free; the factor 16 is folded into the scale (exact).  One
//    packed word becomes two int8 words in three logic operations.
//  - The scale step needs the group's int32 dots as floats.  Each TMEM
//    accumulator is pre-set to the bits of 1.5*2^23 and the MMA adds the group's
//    dots onto it (|16 I| < 2^22), so the accumulator read back as a float is
//    exactly 1.5*2^23 + 16 I; one packed subtract and one packed FMA per two
//    values finish the step, and writing the bias back re-arms the buffer.
//  - Four TMEM buffers of 128 columns (all 512) hold consecutive groups, so the
//    tensor core runs up to four groups ahead of the epilogue.  Shared memory
//    holds four stages of the pipeline: the packed weight tile (TMA), its int8
//    expansion (written by the dequant warps in the 128-byte-swizzled K-major
//    layout the MMA descriptor names) and the activation tile (TMA, 128-byte
//    swizzle).  Each CTA is persistent over tiles; the last tile's output stores
//    overlap the next tile's first MMAs.
//
// Warp roles (12 warps, 168 registers each): warp 0 lane 0 is the scheduler, a
// loop that issues TMA copies and MMAs as soon as their barriers allow (non-
// blocking tests, so neither waits behind the other); warps 1-3 expand int4 to
// int8; warps 4-11 are the epilogue (two halves of 64 columns; warp % 4 is the
// TMEM lane quadrant a warp may read).  Every wait is bounded; a wait that gives
// up sets the device error word, and all roles then leave their loops.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <mutex>

#include "common.cuh"
#include "launch.cuh"
#include "tma.cuh"

namespace w4a8 {

int sm_count();                    // capi.cu
unsigned int* device_error_word();  // gemv_mma.cu

namespace {

constexpr int kRows = 128;  // weight rows per tile (MMA M)
constexpr int kTok = 128;   // tokens per tile (MMA N)
constexpr int kLoadStages = 6;  // packed weight + activation tiles (TMA ring)
constexpr int kAStages = 3;     // int8 weight tiles (expansion ring)
constexpr int kBufs = 4;        // TMEM group accumulators of kTok columns
constexpr uint32_t kTmemCols = kBufs * kTok;
constexpr int kDeqWarp0 = 1, kDeqWarps = 3;
constexpr int kDeqThreads = kDeqWarps * 32;
constexpr int kEpiWarp0 = 4, kEpiWarps = 8;
constexpr int kThreads = (kEpiWarp0 + kEpiWarps) * 32;  // 384: 168 registers per thread
constexpr uint32_t kBias = 0x4B400000u;  // bits of 1.5 * 2^23
constexpr float kBiasF = 12582912.0f;

constexpr uint32_t kXBytes = kTok * 128;   // activation tile: kTok rows x 128 k
constexpr uint32_t kABytes = kRows * 128;  // int8 weight tile: kRows x 128 k
constexpr uint32_t kPBytes = kRows * 64;   // packed weight tile: kRows x 64 bytes
constexpr uint32_t kOffX = 0;
constexpr uint32_t kOffP = kOffX + kLoadStages * kXBytes;
constexpr uint32_t kOffA = kOffP + kLoadStages * kPBytes;
constexpr uint32_t kOffXchg = kOffA + kAStages * kABytes;
constexpr uint32_t kXchgBytes = 2 * 64 * 64 * 4;  // SWIGLU: up-half values of both column halves

__host__ __device__ constexpr uint32_t bar_offset(bool swiglu) { return kOffXchg + (swiglu ? kXchgBytes : 0); }
__host__ __device__ constexpr size_t smem_bytes(bool swiglu) { return 1024 + bar_offset(swiglu) + 256; }
static_assert(smem_bytes(true) <= 227 * 1024, "shared memory plan exceeds 227 KB");

struct TcParams {
    const uint16_t* s;  // [rows][kg] f16 scales
    const float* dx;    // [m] per-token activation scale
    float* y;           // [m][y_stride]
    int* dots;          // group-dot hook: [m][rows][kg]
    unsigned int* err;  // device error word
    int rows;           // weight rows (2 * n_out for SWIGLU)
    int n_out;
    int m, kg, y_stride;
    int row_tiles, tok_tiles;
};

// --- tcgen05 / TMA primitives -------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

// K-major operand in the 128-byte swizzle: rows of 128 bytes, 8-row atoms 1024
// bytes apart (stride byte offset), start address advanced by 32 bytes per k-step.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);  // start address
    d |= static_cast<uint64_t>(1) << 16;                         // leading byte offset (unused here)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;                 // stride byte offset
    d |= static_cast<uint64_t>(1) << 46;                         // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2) << 61;                         // 128-byte swizzle
    return d;
}

// kind::i8 instruction descriptor: s32 accumulate, signed A and B, both K-major.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kTok >> 3) << 17) |
                            (static_cast<uint32_t>(kRows >> 4) << 24);

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, 1, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 32 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Writes the bias into 32 consecutive columns of this thread's lane.
__device__ __forceinline__ void tmem_bias32(uint32_t taddr) {
    const uint32_t b = kBias;
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
        "%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
        "r"(b)
        : "memory");
}

// Barrier over the 128 threads of one epilogue column half (an mbarrier, so the
// wait is bounded like every other wait here).
__device__ __forceinline__ bool half_sync(uint64_t* bar, uint32_t& phase, volatile int* abort_flag,
                                          unsigned int* err) {
    mbar_arrive(bar);
    const bool ok = mbar_wait(bar, phase & 1);
    ++phase;
    if (!ok) {
        *abort_flag = 1;
        atomicOr(err, DEV_ERR_GEMM_TIMEOUT);
    }
    return ok;
}

// 16 * (q - 8) for the four low nibbles / the four high nibbles of a packed word.
__device__ __forceinline__ uint32_t expand_lo(uint32_t w) { return ((w ^ 0x88888888u) << 4) & 0xF0F0F0F0u; }
__device__ __forceinline__ uint32_t expand_hi(uint32_t w) { return (w ^ 0x88888888u) & 0xF0F0F0F0u; }

// A bounded wait that turns a timeout into the error word and the abort flag.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, unsigned int* err) {
    if (mbar_wait(bar, parity)) return true;
    *abort_flag = 1;
    atomicOr(err, DEV_ERR_GEMM_TIMEOUT);
    return false;
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

template <int MODE, bool DOTS>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                   const TcParams p) {
    constexpr bool SWI = (MODE == W4A8_SWIGLU);
    constexpr int kOutRows = SWI ? 64 : kRows;  // output rows per tile
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + bar_offset(SWI));  // TMA landed
    uint64_t* empty = full + kLoadStages;   // MMA done with the load stage
    uint64_t* aready = empty + kLoadStages; // int8 tile written
    uint64_t* aempty = aready + kAStages;   // MMA done with the int8 tile
    uint64_t* accf = aempty + kAStages;     // group accumulator complete
    uint64_t* acce = accf + kBufs;          // group accumulator read and re-biased
    uint64_t* done = acce + kBufs;
    uint64_t* xbar = done + 1;  // SWIGLU exchange, one per column half
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kLoadStages; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        for (int s = 0; s < kAStages; ++s) {
            mbar_init(aready + s, kDeqThreads);
            mbar_init(aempty + s, 1);
        }
        for (int b = 0; b < kBufs; ++b) {
            mbar_init(accf + b, 1);
            mbar_init(acce + b, kEpiWarps * 32);
        }
        mbar_init(done, 1);
        mbar_init(xbar, 128);
        mbar_init(xbar + 1, 128);
        *abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 0) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();
    pdl_wait();

    const int tiles = p.row_tiles * p.tok_tiles;
    const int kg = p.kg;

    if (warp == 0) {
        // ---- scheduler: TMA copies up to kLoadStages groups ahead, MMAs in order ----
        if (lane == 0) {
            const int my_tiles = blockIdx.x < tiles ? (tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
            const uint32_t total = static_cast<uint32_t>(my_tiles) * kg;
            uint32_t tj = 0, mj = 0;  // next group to copy / to multiply
            int tg = 0, tt = blockIdx.x;  // group and tile of tj
            long long idle_since = clock64();
            while (mj < total) {
                bool progress = false;
                while (tj < total) {
                    const uint32_t s = tj % kLoadStages, u = tj / kLoadStages;
                    if (!mbar_test(empty + s, (u & 1) ^ 1)) break;
                    const int n0 = (tt / p.tok_tiles) * kOutRows, m0 = (tt % p.tok_tiles) * kTok;
                    mbar_expect_tx(full + s, kPBytes + kXBytes);
                    unsigned char* pk = smem + kOffP + s * kPBytes;
                    if (SWI) {
                        tma_load_2d(pk, &tm_w, tg * 64, n0, full + s);
                        tma_load_2d(pk + 64 * 64, &tm_w, tg * 64, p.n_out + n0, full + s);
                    } else {
                        tma_load_2d(pk, &tm_w, tg * 64, n0, full + s);
                    }
                    tma_load_2d(smem + kOffX + s * kXBytes, &tm_x, tg * 128, m0, full + s);
                    ++tj;
                    if (++tg == kg) {
                        tg = 0;
                        tt += gridDim.x;
                    }
                    progress = true;
                }
                if (mj < tj) {
                    const uint32_t s = mj % kLoadStages, u = mj / kLoadStages;
                    const uint32_t sa = mj % kAStages, ua = mj / kAStages;
                    const uint32_t b = mj % kBufs, v = mj / kBufs;
                    if (mbar_test(aready + sa, ua & 1) && mbar_test(full + s, u & 1) && mbar_test(acce + b, v & 1)) {
                        tc_fence_after();
                        const uint32_t a_addr = smem_u32(smem + kOffA + sa * kABytes);
                        const uint32_t x_addr = smem_u32(smem + kOffX + s * kXBytes);
                        const uint32_t d = tmem + b * kTok;
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            mma_i8(d, sw128_desc(a_addr + 32 * kk), sw128_desc(x_addr + 32 * kk), kIdesc);
                        tc_commit(empty + s);
                        tc_commit(aempty + sa);
                        tc_commit(accf + b);
                        ++mj;
                        progress = true;
                    }
                }
                if (progress) {
                    idle_since = clock64();
                } else if (*abort_flag || clock64() - idle_since > kWaitLimitCycles) {
                    *abort_flag = 1;
                    atomicOr(p.err, DEV_ERR_GEMM_TIMEOUT);
                    break;
                }
            }
            // Every MMA issued completes, and no copy is still landing in shared
            // memory, before TMEM is released and the CTA exits.
            tc_commit(done);
            mbar_wait(done, 0);
            for (uint32_t i = tj > kLoadStages ? tj - kLoadStages : 0; i < tj; ++i)
                mbar_wait(full + i % kLoadStages, (i / kLoadStages) & 1);
        }
    } else if (warp < kEpiWarp0) {
        // ---- int4 -> int8 expansion into the swizzled K-major A tile ----
        const int dt = threadIdx.x - kDeqWarp0 * 32;
        uint32_t j = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            for (int g = 0; g < kg; ++g, ++j) {
                const uint32_t s = j % kLoadStages, u = j / kLoadStages;
                const uint32_t sa = j % kAStages, ua = j / kAStages;
                const bool w_ok = !*abort_flag && tc_wait(full + s, u & 1, abort_flag, p.err) &&
                                  tc_wait(aempty + sa, (ua & 1) ^ 1, abort_flag, p.err);
                if (!__all_sync(kFull, w_ok)) {
                    ok = false;
                    break;
                }
                const uint4* src = reinterpret_cast<const uint4*>(smem + kOffP + s * kPBytes);
                unsigned char* dst = smem + kOffA + sa * kABytes;
                for (int ci = dt; ci < kRows * 4; ci += kDeqThreads) {
                    // 16-byte chunk ci: row ci/4, k-words 4(ci%4)..+3 -> int8 chunks 2(ci%4), +1
                    const int r = ci >> 2, c = ci & 3;
                    const uint4 w = src[ci];
                    const uint4 o0 = make_uint4(expand_lo(w.x), expand_hi(w.x), expand_lo(w.y), expand_hi(w.y));
                    const uint4 o1 = make_uint4(expand_lo(w.z), expand_hi(w.z), expand_lo(w.w), expand_hi(w.w));
                    *reinterpret_cast<uint4*>(dst + r * 128 + (((2 * c) ^ (r & 7)) << 4)) = o0;
                    *reinterpret_cast<uint4*>(dst + r * 128 + (((2 * c + 1) ^ (r & 7)) << 4)) = o1;
                }
                fence_proxy_async();
                mbar_arrive(aready + sa);
            }
        }
    } else {
        // ---- epilogue: scale step per group, output per tile ----
        const int ew = warp - kEpiWarp0;
        const int quad = warp & 3, half = ew >> 2;
        const int lrow = quad * 32 + lane;  // TMEM lane = tile row of this thread
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16) + half * 64;
        for (int b = 0; b < kBufs; ++b) {
            tmem_bias32(lane_base + b * kTok);
            tmem_bias32(lane_base + b * kTok + 32);
        }
        tmem_wait_st();
        tc_fence_before();
        for (int b = 0; b < kBufs; ++b) mbar_arrive(acce + b);

        float* xchg = reinterpret_cast<float*>(smem + kOffXchg) + half * 64 * 64;
        const float2 nbias = make_float2(-kBiasF, -kBiasF);
        uint32_t xph = 0;
        uint32_t j = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            const int n0 = (t / p.tok_tiles) * kOutRows, m0 = (t % p.tok_tiles) * kTok;
            int row;
            bool row_ok;
            if (SWI) {
                const int o = n0 + (lrow & 63);
                row_ok = o < p.n_out;
                row = lrow < 64 ? o : p.n_out + o;
            } else {
                row = n0 + lrow;
                row_ok = row < p.rows;
            }
            const uint16_t* srow = p.s + static_cast<size_t>(row_ok ? row : 0) * kg;
            float2 acc[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] = make_float2(0.f, 0.f);
            float sc_next = row_ok ? __half2float(__ushort_as_half(__ldg(srow))) : 0.f;
            for (int g = 0; g < kg; ++g, ++j) {
                const float sc = sc_next * 0.0625f;  // the expansion's factor 16
                if (g + 1 < kg) sc_next = row_ok ? __half2float(__ushort_as_half(__ldg(srow + g + 1))) : 0.f;
                const uint32_t b = j % kBufs, v = j / kBufs;
                const bool w_ok = !*abort_flag && tc_wait(accf + b, v & 1, abort_flag, p.err);
                if (!__all_sync(kFull, w_ok)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const float2 sc2 = make_float2(sc, sc);
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    uint32_t r[32];
                    const uint32_t ta = lane_base + b * kTok + hh * 32;
                    tmem_ld32(ta, r);
                    tmem_wait_ld();
                    tmem_bias32(ta);
                    if (DOTS) {
                        if (row_ok) {
#pragma unroll
                            for (int i = 0; i < 32; ++i) {
                                const int m = m0 + half * 64 + hh * 32 + i;
                                if (m < p.m)
                                    p.dots[(static_cast<size_t>(m) * p.rows + row) * kg + g] =
                                        static_cast<int>(r[i] - kBias) >> 4;
                            }
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const float2 f = __fadd2_rn(make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])), nbias);
                            acc[hh * 16 + i] = __ffma2_rn(f, sc2, acc[hh * 16 + i]);
                        }
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(acce + b);
            }
            if (!ok || DOTS) continue;
            // Output: y[m, n] = acc * dx[m]; a warp stores 32 consecutive n per token.
            const int mbase = m0 + half * 64;
            if (SWI) {
                if (lrow >= 64) {
#pragma unroll
                    for (int i = 0; i < 64; ++i) {
                        const int m = mbase + i;
                        const float d = m < p.m ? __ldg(p.dx + m) : 0.f;
                        const float a = (i & 1) ? acc[i >> 1].y : acc[i >> 1].x;
                        xchg[i * 64 + (lrow - 64)] = a * d;
                    }
                }
                if (!half_sync(xbar + half, xph, abort_flag, p.err)) break;
                if (lrow < 64 && row_ok) {
                    const int n = n0 + lrow;
#pragma unroll
                    for (int i = 0; i < 64; ++i) {
                        const int m = mbase + i;
                        if (m < p.m) {
                            const float a = ((i & 1) ? acc[i >> 1].y : acc[i >> 1].x) * __ldg(p.dx + m);
                            p.y[static_cast<size_t>(m) * p.y_stride + n] = silu_mul(a, xchg[i * 64 + lrow]);
                        }
                    }
                }
                if (!half_sync(xbar + half, xph, abort_flag, p.err)) break;
            } else if (row_ok) {
#pragma unroll
                for (int i = 0; i < 64; ++i) {
                    const int m = mbase + i;
                    if (m < p.m) {
                        const float a = ((i & 1) ? acc[i >> 1].y : acc[i >> 1].x) * __ldg(p.dx + m);
                        float* dst = p.y + static_cast<size_t>(m) * p.y_stride + row;
                        if (MODE == W4A8_ADD)
                            *dst += a;
                        else
                            *dst = a;
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// --- host side ------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// Row-major byte matrix [outer][inner] with the given row stride, copied in boxes
// of box_inner x box_outer bytes.
w4a8_status encode_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t stride,
                      uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
    const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return set_error(W4A8_ECUDA, "w4a8_gemm: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {stride};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, elem,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(W4A8_ECUDA, "w4a8_gemm: tensor map encode failed (%d)", static_cast<int>(r));
    return W4A8_OK;
}

template <int MODE, bool DOTS>
w4a8_status launch_inst(const CUtensorMap& tw, const CUtensorMap& tx, const TcParams& p, cudaStream_t st) {
    static size_t configured = 0;  // dynamic shared memory set for this instantiation
    auto kernel = gemm_tc_kernel<MODE, DOTS>;
    const size_t smem = smem_bytes(MODE == W4A8_SWIGLU);
    if (smem > configured) {
        const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return set_error(W4A8_ECUDA, "w4a8_gemm: smem attribute: %s", cudaGetErrorString(e));
        configured = smem;
    }
    const int tiles = p.row_tiles * p.tok_tiles;
    const int sms = sm_count();
    const int grid = tiles < sms ? tiles : sms;
    return launch_pdl("w4a8_gemm (tcgen05)", kernel, dim3(grid), dim3(kThreads), smem, st, tw, tx, p);
}

}  // namespace

// Group-128 symmetric weights, per-token activations, k % 128 == 0 (checked by
// the caller).  dots != nullptr selects the group-dot hook (mode STORE, no y).
w4a8_status launch_gemm_tc(const w4a8_weight* w, const int8_t* xq, const float* dx, int m, int mode, float* y,
                           int* dots, cudaStream_t st) {
    const bool swi = mode == W4A8_SWIGLU;
    TcParams p{};
    p.s = static_cast<const uint16_t*>(w->s);
    p.dx = dx;
    p.y = y;
    p.dots = dots;
    p.err = device_error_word();
    if (!p.err) return set_error(W4A8_ECUDA, "w4a8_gemm: device error word unavailable");
    p.rows = w->n;
    p.n_out = swi ? w->n / 2 : w->n;
    p.m = m;
    p.kg = w->k / 128;
    p.y_stride = p.n_out;
    p.row_tiles = (p.n_out + (swi ? 63 : 127)) / (swi ? 64 : 128);
    p.tok_tiles = (m + kTok - 1) / kTok;
    CUtensorMap tw, tx;
    w4a8_status s = encode_2d(&tw, w->q, static_cast<uint64_t>(w->k / 2), static_cast<uint64_t>(w->n),
                              static_cast<uint64_t>(w->k / 2), 64, swi ? 64 : 128, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (s != W4A8_OK) return s;
    s = encode_2d(&tx, xq, static_cast<uint64_t>(w->k), static_cast<uint64_t>(m), static_cast<uint64_t>(w->k), 128,
                  kTok, CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != W4A8_OK) return s;
    if (dots) return launch_inst<W4A8_STORE, true>(tw, tx, p, st);
    if (mode == W4A8_ADD) return launch_inst<W4A8_ADD, false>(tw, tx, p, st);
    if (swi) return launch_inst<W4A8_SWIGLU, false>(tw, tx, p, st);
    return launch_inst<W4A8_STORE, false>(tw, tx, p, st);
}

}  // namespace w4a8
