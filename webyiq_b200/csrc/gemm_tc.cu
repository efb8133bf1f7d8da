// W4A8 prefill GEMM on the 5th-generation tensor cores: tcgen05.mma kind::i8 on
// SM pairs (cta_group::2) with the accumulators in tensor memory (TMEM), for
// group-128 symmetric int4 weights and per-token int8 activations:
//
//     y[m, n] = dx[m] * sum_g s[n, g] * I[m, n, g],   I = sum_{k in g} (q[n,k] - 8) * xq[m, k]
//
// Reference: gemm_q4q8.wgsl:46-121 (the tiled prefill GEMM; its per-group math is
// the GEMV's, gemv_q4q8.wgsl:29-34,68, and the output modes are those of
// gemv_q4q8.wgsl:122-129).  The per-group int32 dots I are exact; the scale step
// is f32 (y within 1e-6 relative of the exact path), not the bit-exact int64
// step of the GEMV kernels.
//
// Why this shape (B200 view).
//  - A cluster of two CTAs (two SMs) computes a tile of 256 weight rows x 128
//    tokens with one tcgen05.mma.cta_group::2 per 32-deep k-step (M = 256 rows,
//    N = 128 tokens).  Each SM holds 128 weight rows and HALF of the activation
//    tile (64 tokens); the pair's tensor cores share both halves.  So an SM
//    brings in 8 KB of packed weights and 8 KB of activations per 128-deep group
//    (16 KB, a third less than a one-SM 128 x 128 tile), which is what the L2 ->
//    SM path can sustain at tensor-core speed.
//  - Weight rows are the MMA M (one TMEM lane per row), tokens the MMA N: the
//    per-group scale s[n, g] is a per-lane constant in the epilogue.
//  - The packed weights arrive by TMA (a 3-D map of 4 groups x 128 rows x 64 B with
//    64-byte swizzle, so the row reads are conflict-free).  The expansion warps
//    expand each group ahead of its MMA into an int8 weight tile in TMEM (the
//    MMA's A operand): 16*(q-8) per byte, the nibble q^8 (the 4-bit
//    two's complement of q-8) in the high half of the byte, so its sign extends
//    for free; the factor 16 is folded into the scale (exact).  Keeping A in TMEM
//    spares shared-memory bandwidth, the other limit of this kernel.
//  - Activations come by TMA, four groups (4 x 8 KB) per copy through a 3-D
//    tensor map (k-inner 128 bytes, tokens, groups), so every group lands as its
//    own swizzled K-major block (the MMA's B operand).
//  - Each group's MMAs write their own TMEM accumulator (the first k-step
//    overwrites it), an exact int32 16 I.  The scale warps read it, release the
//    buffer at once and finish the scale step from registers (an exact int -> f32
//    conversion and one packed FMA per two values).  Three accumulator buffers of
//    128 columns and four int8 weight tiles of 32 columns fill TMEM's 512 columns.
//
// Warp roles per CTA (23 warps): 0 weight and activation TMA; 1 and 2 MMA issue
// (cluster rank 0 only), the even and the odd groups (a tcgen05.mma blocks its
// thread for about its own duration, and a barrier test or commit after it holds
// the thread up further, so a second issuing thread keeps the tensor core fed
// meanwhile); 1 also allocates TMEM; 3-6 weight expansion, one warp per TMEM lane
// quarter (warp % 4 is the quarter a warp may access), each thread expanding its
// whole tile row of a group into the TMEM weight tile, up to kABufs groups ahead
// of the scale step; 7-22 the scale step, four warps per lane quarter, each on its
// own 32 of the tile's 128 token columns.  Expansion and scale step run in
// separate warps so neither waits behind the other, and four scale warps per SM
// sub-partition hide the TMEM load latency of each other.
// The barrier the MMA waits on per group ("go": its int8 tile written and its
// accumulator released) lives in rank 0 and both CTAs arrive on it; the MMA's
// completions arrive on both CTAs' barriers (one multicast tcgen05.commit).  Every wait is bounded; a wait
// that gives up sets the device error word and all roles then leave their loops.
// Nothing here uses cluster multicast.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <mutex>

#include "common.cuh"
#include "launch.cuh"
#include "tma.cuh"

namespace w4a8 {

int sm_count();                     // capi.cu
unsigned int* device_error_word();  // gemv_mma.cu

namespace {

constexpr int kRows = 128;      // weight rows per CTA (half of the MMA M = 256)
constexpr int kTok = 128;       // tokens per tile (the MMA N); each CTA loads half
constexpr int kHalfTok = kTok / 2;
constexpr int kSG = 4;          // groups per pipeline stage (one weight and one activation copy)
constexpr int kStages = 3;
constexpr int kDBufs = 3;       // TMEM group accumulators of kTok columns
constexpr int kABufs = 4;       // TMEM int8 weight tiles of 32 columns (128 rows x 128 k)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemA = kDBufs * kTok;  // first column of the weight tiles
static_assert(kTmemA + kABufs * 32 <= kTmemCols, "TMEM plan exceeds 512 columns");
constexpr int kMmaWarps = 2;                 // MMA issue: warp 1 the even groups, warp 2 the odd ones
constexpr int kExpWarp0 = 1 + kMmaWarps, kExpWarps = 4;  // weight expansion: one warp per TMEM lane quarter
constexpr int kSclWarp0 = kExpWarp0 + kExpWarps;
constexpr int kSclPerQuad = 4;                          // scale warps per lane quarter
constexpr int kSclWarps = 4 * kSclPerQuad;
constexpr int kCW = kTok / kSclPerQuad;                 // token columns of one scale warp
static_assert(kCW == 32, "a scale warp reads its slice of an accumulator with one 32-column load");
constexpr int kThreads = (kSclWarp0 + kSclWarps) * 32;  // 736 (80 registers a thread)

constexpr uint32_t kWGroupBytes = kRows * 64;       // packed weights of one group (this CTA's rows)
constexpr uint32_t kXGroupBytes = kHalfTok * 128;   // activations of one group (this CTA's tokens)
constexpr uint32_t kStageBytes = kSG * (kWGroupBytes + kXGroupBytes);
constexpr uint32_t kOffW = 0;                       // [stage][group][128 rows][64 B], 64-byte swizzle
constexpr uint32_t kOffX = kStages * kSG * kWGroupBytes;  // [stage][group][64 tokens][128 B], 128-byte swizzle
constexpr uint32_t kOffXchg = kOffX + kStages * kSG * kXGroupBytes;
constexpr uint32_t kXchgBytes = kTok * 64 * 4;  // SWIGLU: up-row values of every column slice

__host__ __device__ constexpr uint32_t bar_offset(bool swiglu) { return kOffXchg + (swiglu ? kXchgBytes : 0); }
__host__ __device__ constexpr size_t smem_bytes(bool swiglu) { return 1024 + bar_offset(swiglu) + 512; }
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

// --- cluster / tcgen05 / TMA primitives -----------------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
// Arrival on a barrier of either CTA of the cluster (address from peer_addr).  The
// data it publishes is in tensor memory, ordered by the tcgen05 fences around the
// arrival and the wait, so the arrival keeps the default CTA-scope release: a
// cluster-scope release would also wait for this thread's outstanding global loads.
__device__ __forceinline__ void arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Pair-wide TMEM allocation: the same warp of both CTAs executes it.
__device__ __forceinline__ void tmem_alloc2(uint32_t* slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
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

// kind::i8 instruction descriptor: s32 accumulate, signed A and B, both K-major,
// M = 256 (the pair), N = kTok.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kTok >> 3) << 17) |
                            (static_cast<uint32_t>(256 >> 4) << 24);

// One k-step of the pair's MMA: A (this CTA's 128 weight rows, int8) from TMEM,
// B (this CTA's 64 tokens) from shared memory; acc = 0 overwrites the
// accumulator (the group's first k-step), acc = 1 adds to it.
__device__ __forceinline__ void mma_i8_pair_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                               uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::i8 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}
// Arrives on the barrier at this shared::cluster address (either CTA of the pair)
// once the MMAs issued so far complete.
__device__ __forceinline__ void tc_commit_to(uint32_t cluster_addr) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_addr)
                 : "memory");
}
// The same barrier in both CTAs, one instruction: the commit arrives at this
// shared-memory offset in every CTA of the mask (both CTAs of the pair).  This is
// a completion signal, not a load; nothing here loads with cluster multicast.
__device__ __forceinline__ void tc_commit_both(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                     smem_u32(bar)),
                 "h"(static_cast<unsigned short>(3))
                 : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
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

// 32 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

// 16 * (q - 8) for the four low nibbles / the four high nibbles of a packed word.
__device__ __forceinline__ uint32_t expand_lo(uint32_t w) { return ((w ^ 0x88888888u) << 4) & 0xF0F0F0F0u; }
__device__ __forceinline__ uint32_t expand_hi(uint32_t w) { return (w ^ 0x88888888u) & 0xF0F0F0F0u; }

// Bounded waits that turn a timeout into the error word and the abort flag.
struct Abort {
    volatile int* flag;
    unsigned int* err;
    __device__ bool fail() const {
        *flag = 1;
        atomicOr(err, DEV_ERR_GEMM_TIMEOUT);
        return false;
    }
    __device__ bool wait(uint64_t* bar, uint32_t parity) const { return mbar_wait(bar, parity) || fail(); }
    // Barrier over the 128 threads of one scale column slice (bounded, unlike a
    // named barrier).
    __device__ bool slice_sync(uint64_t* bar, uint32_t& phase) const {
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
        const bool ok = mbar_wait(bar, phase & 1);
        ++phase;
        return ok || fail();
    }
};

template <int MODE, bool DOTS>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                   const TcParams p) {
    constexpr bool SWI = (MODE == W4A8_SWIGLU);
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + bar_offset(SWI));  // stage copies landed (local)
    uint64_t* empty = full + kStages;     // MMA done with a stage (both)
    // "Go" for group j (ring of kABufs, rank 0; both CTAs arrive): its int8 weight
    // tile is in TMEM (the expansion warps' arrivals) and its accumulator buffer is
    // free (the scale warps' arrivals after group j - kDBufs), so the MMA thread
    // waits on one barrier per group.
    uint64_t* go = empty + kStages;
    // The MMAs of group j complete (both CTAs, one ring of kABufs): accumulator j
    // may be read, and weight tile j % kABufs may be rewritten for group j + kABufs.
    uint64_t* gdone = go + kABufs;
    uint64_t* done = gdone + kABufs;      // all MMAs complete (rank 0)
    uint64_t* xbar = done + 1;            // SWIGLU exchange, one per column slice (local)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + kSclPerQuad);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, kMmaWarps);  // one commit per MMA thread
        }
        for (int a = 0; a < kABufs; ++a) {
            mbar_init(go + a, 2 * (kExpWarps + kSclWarps));  // every expansion and scale warp of each CTA
            mbar_init(gdone + a, 1);
        }
        mbar_init(done, kMmaWarps);
        for (int c = 0; c < kSclPerQuad; ++c) mbar_init(xbar + c, 128);
        *abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 1) tmem_alloc2(tmem_slot, kTmemCols);
    tc_fence_before();
    cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();
    pdl_wait();

    const Abort ab{abort_flag, p.err};
    const int nclusters = gridDim.x / 2;
    const int cluster = blockIdx.x / 2;
    const int tiles = p.row_tiles * p.tok_tiles;
    const int my_tiles = cluster < tiles ? (tiles - 1 - cluster) / nclusters + 1 : 0;
    const int kg = p.kg;
    const int spt = (kg + kSG - 1) / kSG;  // stages per tile
    // First weight row of this CTA's 128 (SWIGLU: first gate row of its 64 outputs).
    auto row0_of = [&](int t) -> int {
        const int rt = t / p.tok_tiles;
        return SWI ? rt * 128 + static_cast<int>(rank) * 64 : rt * 256 + static_cast<int>(rank) * kRows;
    };

    if (warp == 0) {
        // ---- TMA: kSG groups of this CTA's packed weight rows and its 64 tokens per stage ----
        if (lane == 0) {
            uint32_t js = 0;
            bool ok = true;
            for (int i = 0; i < my_tiles && ok; ++i) {
                const int t = cluster + i * nclusters;
                const int r0 = row0_of(t);
                const int m0 = (t % p.tok_tiles) * kTok + static_cast<int>(rank) * kHalfTok;
                for (int st = 0; st < spt; ++st, ++js) {
                    const uint32_t s = js % kStages, u = js / kStages;
                    if (*abort_flag || !ab.wait(empty + s, (u & 1) ^ 1)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(full + s, kStageBytes);
                    unsigned char* w = smem + kOffW + s * kSG * kWGroupBytes;
                    if (SWI) {
                        tma_load_3d(w, &tm_w, 0, r0, st * kSG, full + s);
                        tma_load_3d(w + kSG * kWGroupBytes / 2, &tm_w, 0, p.n_out + r0, st * kSG, full + s);
                    } else {
                        tma_load_3d(w, &tm_w, 0, r0, st * kSG, full + s);
                    }
                    tma_load_3d(smem + kOffX + s * kSG * kXGroupBytes, &tm_x, 0, m0, st * kSG, full + s);
                }
            }
            // No copy may still be landing in shared memory when the CTA exits.
            for (uint32_t i = js > kStages ? js - kStages : 0; i < js; ++i)
                mbar_wait(full + i % kStages, (i / kStages) & 1);
        }
    } else if (warp <= kMmaWarps) {
        // ---- MMA issue (rank 0): four k-steps of 32 per group for the pair, the
        //      even groups from warp 1 and the odd ones from warp 2 ----
        // (Both CTAs' expansion warps saw the group's stage land before they
        // arrived on go, so go covers the activation tile halves too.)  A barrier
        // test or a commit right after MMAs holds up its thread for about 200 / 60
        // cycles, in which this thread's own MMAs drain; with two threads issuing
        // alternate groups, one thread's test and commit run while the other's MMAs
        // keep the tensor core busy.  Each thread commits only its own MMAs (a
        // commit tracks the MMAs its thread issued), so every group's completion
        // and every stage's release (count kMmaWarps) stay exact.
        if (rank == 0 && lane == 0) {
            const uint32_t par = static_cast<uint32_t>(warp - 1);  // this thread's groups: j % 2 == par
            uint32_t j = 0, js = 0;
            bool ok = true;
            for (int i = 0; i < my_tiles && ok; ++i) {
                for (int g = 0; g < kg; ++g, ++j) {
                    const uint32_t s = js % kStages;
                    if ((j & 1) == par) {
                        const uint32_t a = j % kABufs, ua = j / kABufs;
                        const uint32_t b = j % kDBufs;
                        if (!mbar_test(go + a, ua & 1) && (*abort_flag || !ab.wait(go + a, ua & 1))) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t x_addr = smem_u32(smem + kOffX + (s * kSG + g % kSG) * kXGroupBytes);
                        const uint32_t d = tmem + b * kTok;
                        const uint32_t at = tmem + kTmemA + a * 32;
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            mma_i8_pair_ts(d, at + kk * 8, sw128_desc(x_addr + 32 * kk), kIdesc, kk > 0);
                        tc_commit_both(gdone + a);
                    }
                    if (g % kSG == kSG - 1 || g == kg - 1) {
                        tc_commit_both(empty + s);  // this thread's MMAs of the stage (none: at once)
                        ++js;
                    }
                }
            }
            // Every MMA issued completes before TMEM is released.
            tc_commit_to(peer_addr(done, 0));
            if (warp == 1) mbar_wait(done, 0);
        }
    } else if (warp < kSclWarp0) {
        // ---- weight expansion: every group of every tile, in order, into TMEM weight
        //      tile jd % kABufs, as soon as its stage has landed and the MMAs that read
        //      the tile's previous contents have completed ----
        const int quad = warp & 3;
        const int lrow = quad * 32 + lane;  // TMEM lane = tile row of this thread
        const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
        const uint32_t go_rank0 = peer_addr(go, 0);
        const uint32_t total = static_cast<uint32_t>(my_tiles) * kg;
        const int sw = (lrow >> 1) & 3;  // the 64-byte swizzle of this row's chunks
        uint32_t sde = 0;                // running stage index
        int ge = 0;                      // group within the tile
        uint32_t seen = ~0u;             // the running stage whose landing this warp has seen
        int pend = -1;                   // the weight tile stored but not yet published
        // A tile is published (wait::st, fence, arrival on go) once the next group's
        // expansion is done, so each store completes while the warp works on the
        // next group instead of holding it up.  (A store reads its registers at
        // issue, so they are reused at once.)
        auto publish = [&](int a) {
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) arrive_cluster(go_rank0 + a * 8);
        };
        bool ok = true;
        for (uint32_t jd = 0; jd < total; ++jd) {
            const uint32_t s = sde % kStages, a = jd % kABufs, ua = jd / kABufs;
            bool w_ok = !*abort_flag;
            if (w_ok && sde != seen) {  // once per stage
                w_ok = ab.wait(full + s, (sde / kStages) & 1);
                seen = sde;
            }
            w_ok = w_ok && ab.wait(gdone + a, (ua & 1) ^ 1);
            if (!__all_sync(kFull, w_ok)) {
                ok = false;
                break;
            }
            // Packed row lrow of the group: 64 bytes in four 16-byte chunks, chunk c at
            // (c ^ sw) * 16.  A stage holds [kSG groups][128 rows][64 B]; for SWIGLU two
            // such boxes of 64 rows (gate rows, then up rows).
            const unsigned char* stage_w = smem + kOffW + s * kSG * kWGroupBytes;
            const unsigned char* wrow =
                SWI ? stage_w + (lrow >= 64 ? kSG * kWGroupBytes / 2 : 0) + (ge % kSG) * (kWGroupBytes / 2) + (lrow & 63) * 64
                    : stage_w + (ge % kSG) * kWGroupBytes + lrow * 64;
            uint32_t v[32];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint4 ch = *reinterpret_cast<const uint4*>(wrow + ((c ^ sw) << 4));
                v[8 * c + 0] = expand_lo(ch.x);
                v[8 * c + 1] = expand_hi(ch.x);
                v[8 * c + 2] = expand_lo(ch.y);
                v[8 * c + 3] = expand_hi(ch.y);
                v[8 * c + 4] = expand_lo(ch.z);
                v[8 * c + 5] = expand_hi(ch.z);
                v[8 * c + 6] = expand_lo(ch.w);
                v[8 * c + 7] = expand_hi(ch.w);
            }
            if (pend >= 0) publish(pend);
            tmem_st32(tmem + lane_off + kTmemA + a * 32, v);
            pend = static_cast<int>(a);
            if (ge % kSG == kSG - 1 || ge == kg - 1) ++sde;
            if (++ge == kg) ge = 0;
        }
        if (ok && pend >= 0) publish(pend);
    } else {
        // ---- scale step per group, output per tile: this warp's 32-column slice of
        //      its lane quarter's rows ----
        const int quad = warp & 3, cs = (warp - kSclWarp0) >> 2;
        const int lrow = quad * 32 + lane;  // TMEM lane = tile row of this thread
        const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
        const uint32_t d_base = tmem + lane_off + cs * kCW;
        const uint32_t go_rank0 = peer_addr(go, 0);
        if (lane == 0)
            for (int b = 0; b < kDBufs; ++b) arrive_cluster(go_rank0 + b * 8);  // groups 0 .. kDBufs-1: buffers free

        float* xchg = reinterpret_cast<float*>(smem + kOffXchg) + cs * kCW * 64;
        // the eight scales of a block in one 16-byte load: every row's scales 16-byte aligned
        const bool vec8 = kg % 8 == 0 && (reinterpret_cast<uintptr_t>(p.s) & 15) == 0;
        uint32_t xph = 0;
        uint32_t j = 0;
        bool ok = true;
        for (int i = 0; i < my_tiles && ok; ++i) {
            const int t = cluster + i * nclusters;
            const int m0 = (t % p.tok_tiles) * kTok;
            const int mbase = m0 + cs * kCW;
            int row, out_row;
            bool row_ok;
            if (SWI) {
                const int o = row0_of(t) + (lrow & 63);
                row_ok = o < p.n_out;
                row = lrow < 64 ? o : p.n_out + o;
                out_row = o;
            } else {
                row = row0_of(t) + lrow;
                row_ok = row < p.rows;
                out_row = row;
            }
            const uint16_t* srow = p.s + static_cast<size_t>(row_ok ? row : 0) * kg;
            // dx of this slice's tokens: lane i holds token mbase + 32 h + i in dx[h].
            float dx[kCW / 32];
#pragma unroll
            for (int h = 0; h < kCW / 32; ++h)
                dx[h] = (!DOTS && mbase + 32 * h + lane < p.m) ? ld_dep(p.dx + mbase + 32 * h + lane) : 0.f;
            float2 acc[kCW / 2];
#pragma unroll
            for (int e = 0; e < kCW / 2; ++e) acc[e] = make_float2(0.f, 0.f);

            // One group: wait for its accumulator, read it, release the buffer to the
            // MMA of group j + kDBufs (whose first k-step overwrites it), then the
            // scale step from registers.  The accumulator holds 16 I exactly (|16 I| <
            // 2^22), so its conversion to f32 is exact.
            auto group = [&](int g, float sc_raw) -> bool {
                const uint32_t b = j % kDBufs;
                const bool w_ok = !*abort_flag && ab.wait(gdone + j % kABufs, (j / kABufs) & 1);
                ++j;
                if (!__all_sync(kFull, w_ok)) return false;
                tc_fence_after();
                uint32_t r[32];
                tmem_ld32(d_base + b * kTok, r);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) arrive_cluster(go_rank0 + ((j - 1 + kDBufs) % kABufs) * 8);  // group j-1+kDBufs
                if (DOTS) {
                    if (row_ok) {
#pragma unroll
                        for (int e = 0; e < 32; ++e) {
                            const int m = mbase + e;
                            if (m < p.m) p.dots[(static_cast<size_t>(m) * p.rows + row) * kg + g] = static_cast<int>(r[e]) >> 4;
                        }
                    }
                } else {
                    const float sc = sc_raw * 0.0625f;  // the expansion's factor 16
                    const float2 sc2 = make_float2(sc, sc);
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const float2 f = make_float2(__int2float_rn(static_cast<int>(r[2 * e])),
                                                     __int2float_rn(static_cast<int>(r[2 * e + 1])));
                        acc[e] = __ffma2_rn(f, sc2, acc[e]);
                    }
                }
                return true;
            };
            // Scales of a block of eight groups are loaded one block ahead of their
            // use (an L2 round trip is several groups long) and the block is
            // unrolled, so no register copy waits on a load still in flight.  One
            // 16-byte load per block when the row's scales are 16-byte aligned.
            auto load8 = [&](int g0, uint32_t (&d)[4]) {
                if (vec8) {
                    const uint4 v = (row_ok && g0 < kg) ? __ldg(reinterpret_cast<const uint4*>(srow + g0)) : make_uint4(0, 0, 0, 0);
                    d[0] = v.x;
                    d[1] = v.y;
                    d[2] = v.z;
                    d[3] = v.w;
                } else {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint32_t lo = (row_ok && g0 + 2 * q < kg) ? __ldg(srow + g0 + 2 * q) : 0u;
                        const uint32_t hi = (row_ok && g0 + 2 * q + 1 < kg) ? __ldg(srow + g0 + 2 * q + 1) : 0u;
                        d[q] = lo | (hi << 16);
                    }
                }
            };
            uint32_t sc_cur[4], sc_nxt[4];
            load8(0, sc_cur);
#pragma unroll 1
            for (int g0 = 0; g0 < kg && ok; g0 += 8) {
                load8(g0 + 8, sc_nxt);
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    if (ok && g0 + q < kg)
                        ok = group(g0 + q, __half2float(__ushort_as_half(static_cast<unsigned short>(sc_cur[q >> 1] >> (16 * (q & 1))))));
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) sc_cur[q] = sc_nxt[q];
            }
            if (!ok || DOTS) continue;

            // Output: y[m, n] = acc * dx[m]; a warp stores 32 consecutive n per token.
            if (SWI) {
                if (lrow >= 64) {
#pragma unroll
                    for (int e = 0; e < kCW; ++e) {
                        const float d = __shfl_sync(kFull, dx[e >> 5], e & 31);
                        const float av = (e & 1) ? acc[e >> 1].y : acc[e >> 1].x;
                        xchg[e * 64 + (lrow - 64)] = av * d;
                    }
                }
                if (!ab.slice_sync(xbar + cs, xph)) break;
                if (lrow < 64) {
#pragma unroll
                    for (int e = 0; e < kCW; ++e) {
                        const float d = __shfl_sync(kFull, dx[e >> 5], e & 31);
                        const int m = mbase + e;
                        if (row_ok && m < p.m) {
                            const float av = ((e & 1) ? acc[e >> 1].y : acc[e >> 1].x) * d;
                            p.y[static_cast<size_t>(m) * p.y_stride + out_row] = silu_mul(av, xchg[e * 64 + lrow]);
                        }
                    }
                }
                if (!ab.slice_sync(xbar + cs, xph)) break;
            } else {
                const int mlim = p.m - mbase;  // tokens of this slice that exist
                float* dst = p.y + static_cast<size_t>(mbase) * p.y_stride + out_row;
#pragma unroll
                for (int e = 0; e < kCW; ++e) {
                    const float d = __shfl_sync(kFull, dx[e >> 5], e & 31);
                    if (row_ok && e < mlim) {
                        const float av = ((e & 1) ? acc[e >> 1].y : acc[e >> 1].x) * d;
                        if (MODE == W4A8_ADD)
                            *dst += av;
                        else
                            *dst = av;
                    }
                    dst += p.y_stride;
                }
            }
        }
    }

    tc_fence_before();
    cluster_sync();  // no CTA leaves while its peer may still signal it
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc2(tmem, kTmemCols);
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

// 3-D view (inner bytes of one group, rows, groups) of a row-major byte matrix
// with `group_bytes` bytes per group and `row_stride` bytes per row, copied in
// boxes of group_bytes x box_rows x kSG groups: each group lands as its own block.
w4a8_status encode_grouped(CUtensorMap* map, const void* base, int rows, int groups, int group_bytes, int row_stride,
                           int box_rows, CUtensorMapSwizzle swizzle) {
    const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return set_error(W4A8_ECUDA, "w4a8_gemm: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(group_bytes), static_cast<cuuint64_t>(rows),
                                static_cast<cuuint64_t>(groups)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_stride), static_cast<cuuint64_t>(group_bytes)};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(group_bytes), static_cast<cuuint32_t>(box_rows), kSG};
    const cuuint32_t elem[3] = {1, 1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, elem,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(W4A8_ECUDA, "w4a8_gemm: tensor map encode failed (%d)", static_cast<int>(r));
    return W4A8_OK;
}

template <int MODE, bool DOTS>
w4a8_status launch_inst(const CUtensorMap& tw, const CUtensorMap& tx, const TcParams& p, cudaStream_t st) {
    // per device: the raised shared-memory limit, and how many clusters of this
    // kernel fit on the GPU at once
    static FuncAttr attr;
    static std::atomic<int> max_clusters[kMaxDevices];
    auto kernel = gemm_tc_kernel<MODE, DOTS>;
    const size_t smem = smem_bytes(MODE == W4A8_SWIGLU);
    const w4a8_status a = ensure_smem(kernel, attr, smem, -1, "w4a8_gemm");
    if (a != W4A8_OK) return a;
    const int dev = current_device("w4a8_gemm");
    if (dev < 0) return W4A8_ECUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute lattr[2];
    lattr[0].id = cudaLaunchAttributeClusterDimension;
    lattr[0].val.clusterDim.x = 2;
    lattr[0].val.clusterDim.y = 1;
    lattr[0].val.clusterDim.z = 1;
    lattr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    lattr[1].val.programmaticStreamSerializationAllowed = g_use_pdl ? 1 : 0;
    cfg.attrs = lattr;
    cfg.numAttrs = 2;
    int mc = max_clusters[dev].load(std::memory_order_acquire);
    if (mc == 0) {
        // a race between first calls computes the same figure twice
        cfg.gridDim = dim3(2 * (sm_count() / 2));
        int n = 0;
        const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
        if (e != cudaSuccess || n < 1) {
            cudaGetLastError();
            n = sm_count() / 2;
        }
        mc = n;
        max_clusters[dev].store(mc, std::memory_order_release);
    }
    const int tiles = p.row_tiles * p.tok_tiles;
    const int clusters = tiles < mc ? tiles : mc;
    cfg.gridDim = dim3(2 * clusters);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, tw, tx, p);
    if (e != cudaSuccess) return set_error(W4A8_ECUDA, "w4a8_gemm (tcgen05): launch failed: %s", cudaGetErrorString(e));
    return W4A8_OK;
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
    p.row_tiles = swi ? (p.n_out + 127) / 128 : (p.n_out + 255) / 256;
    p.tok_tiles = (m + kTok - 1) / kTok;
    // Packed weights: 64 bytes per group and row, boxes of this CTA's 128 rows (64
    // gate + 64 up rows for SWIGLU), 64-byte swizzle so that one row's chunks are
    // read without bank conflicts.  Activations: 128 bytes per group and token,
    // boxes of 64 tokens, 128-byte swizzle (the MMA's K-major layout).
    CUtensorMap tw, tx;
    w4a8_status s = encode_grouped(&tw, w->q, w->n, p.kg, 64, w->k / 2, swi ? 64 : kRows, CU_TENSOR_MAP_SWIZZLE_64B);
    if (s != W4A8_OK) return s;
    s = encode_grouped(&tx, xq, m, p.kg, 128, w->k, kHalfTok, CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != W4A8_OK) return s;
    if (dots) return launch_inst<W4A8_STORE, true>(tw, tx, p, st);
    if (mode == W4A8_ADD) return launch_inst<W4A8_ADD, false>(tw, tx, p, st);
    if (swi) return launch_inst<W4A8_SWIGLU, false>(tw, tx, p, st);
    return launch_inst<W4A8_STORE, false>(tw, tx, p, st);
}

}  // namespace w4a8
