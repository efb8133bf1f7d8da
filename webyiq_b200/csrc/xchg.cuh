// The peer-memory key exchange of the column-split lm_head: buffer layout, the
// system-scope loads and stores it is built from, and the merge one CTA runs.
//
// Each rank owns one XchgBuf in its device memory; every peer opens it through a
// CUDA IPC handle (plain device memory, no NVLink multicast object).  A merge
// stores the rank's packed key of each token into slot [parity][rank] of every
// rank's buffer and waits (bounded) until every rank's key of this call is in its
// own buffer, then takes the max.  The max of the packed keys is exactly the
// one-GPU argmax (argmax.wgsl:17-39 semantics).
//  - A key carries its call: the top 8 bits of its index half (~id, all ones for
//    ids below 2^24) hold the call's sequence number mod 256.  One relaxed 64-bit
//    store both delivers and validates a key, so no fence and no flag is needed;
//    the keys of one call share the tag, so their order is unchanged.
//  - Slots are double-buffered by the parity of the call's sequence number: a rank
//    that runs ahead writes its next keys into the other half; it cannot run two
//    calls ahead, since each call waits for every rank's keys.
//  - The sequence counter lives in the rank's own buffer and is advanced on the
//    device, so captured CUDA graphs replay correctly.
#pragma once

#include "common.cuh"
#include "tma.cuh"

namespace w4a8 {

struct XchgBuf {
    unsigned long long key[2][W4A8_XCHG_MAX_RANKS][W4A8_XCHG_MAX_TOKENS];  // [parity][source rank][token], tagged
    unsigned int seq;                                                      // calls this rank has completed
};

struct XchgPeers {
    XchgBuf* buf[W4A8_XCHG_MAX_RANKS];  // every rank's buffer as seen from this GPU (own one included)
};

// What a kernel needs to run the merge itself (world == 0: no exchange).
struct XchgArgs {
    XchgPeers peers;
    int world, rank;
};

__device__ __forceinline__ void st_relaxed_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// A key tagged with call seq, the test of a slot for call seq, and the key back.
// A zero key (no valid logit) keeps a zero high half, so it stays the smallest.
__device__ __forceinline__ unsigned long long xchg_tag(unsigned long long key, unsigned int seq) {
    return (key & ~(0xFFull << 24)) | (static_cast<unsigned long long>(seq & 0xFFu) << 24);
}
__device__ __forceinline__ bool xchg_fresh(unsigned long long v, unsigned int seq) {
    return static_cast<unsigned int>((v >> 24) & 0xFFu) == (seq & 0xFFu);
}
__device__ __forceinline__ unsigned long long xchg_untag(unsigned long long v) {
    return (v >> 32) ? (v | (0xFFull << 24)) : 0ull;
}

// This rank's next sequence number, read after the dependency wait (the previous
// call, which advanced it, has completed).
__device__ __forceinline__ unsigned int xchg_next_seq(const XchgArgs& x) {
    return ld_dep(&x.peers.buf[x.rank]->seq) + 1u;
}

// The merge, run by every thread of ONE CTA of at least max(world, m) threads.
// seq: xchg_next_seq, own[t]: this rank's key of token t (visible to the CTA's
// threads).  Writes the global key and token of each token to best_key / tok_out
// (tok_out and ids may be null).  Thread r serves peer r: its stores into rank r's
// buffer, then its wait for rank r's keys here.  A wait that gives up leaves the
// rank's own key and token in the outputs and sets DEV_ERR_XCHG_TIMEOUT.
__device__ __forceinline__ void xchg_merge(const XchgArgs& x, int m, unsigned int seq, const unsigned long long* own,
                                           unsigned long long* best_key, uint32_t* tok_out, const uint32_t* ids,
                                           unsigned int* err) {
    XchgBuf* me = x.peers.buf[x.rank];
    const int tid = threadIdx.x;
    const unsigned int par = seq & 1u;
    bool ok = true;
    if (tid < x.world) {
        const int r = tid;
        for (int t = 0; t < m; ++t) st_relaxed_sys(&x.peers.buf[r]->key[par][x.rank][t], xchg_tag(own[t], seq));
        const long long t0 = clock64();
        for (int t = 0; t < m && ok; ++t)
            while (!xchg_fresh(ld_relaxed_sys(&me->key[par][r][t]), seq))
                if (clock64() - t0 > static_cast<long long>(kWaitLimitCycles)) {
                    ok = false;
                    atomicOr(err, DEV_ERR_XCHG_TIMEOUT);
                    break;
                }
    }
    ok = __syncthreads_and(ok);  // every rank's keys seen (or a wait gave up) before they are read
    if (tid == 0) me->seq = seq;  // the calls stay counted alike on every rank
    if (tid < m) {
        unsigned long long k = own[tid];
        if (ok) {
            k = 0ull;
            for (int r = 0; r < x.world; ++r) {
                const unsigned long long o = ld_relaxed_sys(&me->key[par][r][tid]);
                k = o > k ? o : k;
            }
            k = xchg_untag(k);
        }
        best_key[tid] = k;
        if (tok_out) {
            const uint32_t idx = k ? ~static_cast<uint32_t>(k & 0xffffffffull) : 0u;
            tok_out[tid] = ids ? __ldg(ids + idx) : idx;
        }
    }
}

}  // namespace w4a8
