// Column-split lm_head with the key exchange over peer memory: each rank runs the
// fused lm_head argmax on its vocabulary shard (global ids through row_offset), then
// one small kernel stores the rank's packed keys into every peer's exchange buffer
// (NVLink stores to memory opened through CUDA IPC), raises the rank's sequence flag
// there, waits (bounded) for every rank's flag in its own buffer and takes the max
// of the keys.  The max of the packed keys is exactly the one-GPU argmax
// (argmax.wgsl:17-39 semantics), so every rank gets the global key and token.
//
// Against the NCCL all-reduce of lmhead_multi.cu this replaces a collective launch
// and a key-to-token kernel by one kernel that starts under programmatic dependent
// launch while the lm_head kernel finishes; the exchange itself is one store per
// (peer, token) and one flag per peer, each peer served by its own thread.
//  - Key slots are double-buffered by the parity of the call's sequence number: a
//    rank that runs ahead writes its next keys into the other half, and it cannot
//    run two calls ahead, since each call waits for every rank's flag.
//  - The sequence counter is in the rank's own buffer and advanced by the kernel,
//    so a captured CUDA graph replays correctly; all ranks make the same calls.
//  - The flag wait is bounded (kWaitLimitCycles); a wait that gives up leaves the
//    rank's own key and token in the outputs and sets the device error word.
// Nothing here uses NVLink multicast objects; the buffers are plain device memory.
#include <cstring>

#include "common.cuh"
#include "launch.cuh"
#include "tma.cuh"

namespace w4a8 {

unsigned int* device_error_word();  // gemv_mma.cu

namespace {

struct XchgBuf {
    unsigned long long key[2][W4A8_XCHG_MAX_RANKS][W4A8_XCHG_MAX_TOKENS];  // [parity][source rank][token]
    unsigned int flag[W4A8_XCHG_MAX_RANKS];  // last sequence number each source rank published here
    unsigned int seq;                        // calls this rank has completed (its own counter)
};

struct XchgPeers {
    XchgBuf* buf[W4A8_XCHG_MAX_RANKS];  // every rank's buffer as seen from this GPU (own one included)
};

__device__ __forceinline__ void st_relaxed_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(32) lmhead_xchg_kernel(const XchgPeers peers, int world, int rank, int m, unsigned long long* best_key,
                                   uint32_t* tok_out, const uint32_t* ids, unsigned int* err) {
    pdl_launch_dependents();
    pdl_wait();  // best_key comes from the lm_head kernel
    XchgBuf* me = peers.buf[rank];
    __shared__ unsigned int s_seq;
    __shared__ int s_ok;
    const int tid = threadIdx.x;
    if (tid == 0) {
        s_seq = *reinterpret_cast<volatile unsigned int*>(&me->seq) + 1u;
        s_ok = 1;
    }
    __syncthreads();
    const unsigned int seq = s_seq, par = seq & 1u;
    if (tid < world) {
        // Thread r serves peer r: this rank's keys into slot [par][rank] of rank r's
        // buffer, published by a release store of the flag (it orders this thread's
        // stores).  One thread per peer, so the system-scope releases run side by
        // side instead of one after another.
        const int r = tid;
        for (int t = 0; t < m; ++t) st_relaxed_sys(&peers.buf[r]->key[par][rank][t], best_key[t]);
        st_release_sys(&peers.buf[r]->flag[rank], seq);
        // then the same thread waits (bounded) for rank r's flag in this buffer
        const long long t0 = clock64();
        while (static_cast<int>(ld_acquire_sys(&me->flag[r]) - seq) < 0)
            if (clock64() - t0 > static_cast<long long>(kWaitLimitCycles)) {
                s_ok = 0;
                atomicOr(err, DEV_ERR_XCHG_TIMEOUT);
                break;
            }
    }
    __syncthreads();  // every flag acquired (or given up) before the keys are read
    if (tid == 0) me->seq = seq;  // the calls stay counted alike on every rank
    if (tid < m) {
        unsigned long long k = best_key[tid];
        if (s_ok) {
            k = 0ull;
            for (int r = 0; r < world; ++r) {
                const unsigned long long o = ld_relaxed_sys(&me->key[par][r][tid]);
                k = o > k ? o : k;
            }
            best_key[tid] = k;
        }
        if (tok_out) {
            const uint32_t idx = k ? ~static_cast<uint32_t>(k & 0xffffffffull) : 0u;
            tok_out[tid] = ids ? __ldg(ids + idx) : idx;
        }
    }
}

}  // namespace
}  // namespace w4a8

struct w4a8_xchg {
    int world = 0, rank = 0, device = -1;
    w4a8::XchgBuf* local = nullptr;
    w4a8::XchgPeers peers{};
    bool opened = false;
};

using namespace w4a8;

extern "C" {

W4A8_API w4a8_status w4a8_xchg_create(int32_t world, int32_t rank, void* handle_out, w4a8_xchg** out) {
    static_assert(sizeof(cudaIpcMemHandle_t) == W4A8_XCHG_HANDLE_BYTES, "IPC handle size");
    if (!handle_out || !out || world < 1 || world > W4A8_XCHG_MAX_RANKS || rank < 0 || rank >= world)
        return set_error(W4A8_EINVAL, "w4a8_xchg_create: world=%d rank=%d (world <= %d)", world, rank,
                         W4A8_XCHG_MAX_RANKS);
    w4a8_xchg* x = new w4a8_xchg();
    x->world = world;
    x->rank = rank;
    cudaError_t e = cudaGetDevice(&x->device);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&x->local), sizeof(XchgBuf));
    if (e == cudaSuccess) e = cudaMemset(x->local, 0, sizeof(XchgBuf));
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, x->local);
    if (e != cudaSuccess) {
        if (x->local) cudaFree(x->local);
        delete x;
        return set_error(W4A8_ECUDA, "w4a8_xchg_create: %s", cudaGetErrorString(e));
    }
    memcpy(handle_out, &h, sizeof(h));
    *out = x;
    return W4A8_OK;
}

W4A8_API w4a8_status w4a8_xchg_open(w4a8_xchg* x, const void* handles) {
    if (!x || !handles) return set_error(W4A8_EINVAL, "w4a8_xchg_open: NULL");
    if (x->opened) return set_error(W4A8_EINVAL, "w4a8_xchg_open: already open");
    const unsigned char* hb = static_cast<const unsigned char*>(handles);
    for (int r = 0; r < x->world; ++r) {
        if (r == x->rank) {
            x->peers.buf[r] = x->local;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, hb + static_cast<size_t>(r) * W4A8_XCHG_HANDLE_BYTES, sizeof(h));
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < r; ++q)
                if (q != x->rank && x->peers.buf[q]) cudaIpcCloseMemHandle(x->peers.buf[q]);
            x->peers = XchgPeers{};
            return set_error(W4A8_ECUDA, "w4a8_xchg_open: peer %d: %s", r, cudaGetErrorString(e));
        }
        x->peers.buf[r] = static_cast<XchgBuf*>(p);
    }
    x->opened = true;
    return W4A8_OK;
}

W4A8_API w4a8_status w4a8_xchg_destroy(w4a8_xchg* x) {
    if (!x) return W4A8_OK;
    cudaError_t first = cudaSuccess;
    if (x->opened)
        for (int r = 0; r < x->world; ++r)
            if (r != x->rank && x->peers.buf[r]) {
                const cudaError_t e = cudaIpcCloseMemHandle(x->peers.buf[r]);
                if (first == cudaSuccess) first = e;
            }
    if (x->local) {
        const cudaError_t e = cudaFree(x->local);
        if (first == cudaSuccess) first = e;
    }
    delete x;
    if (first != cudaSuccess) return set_error(W4A8_ECUDA, "w4a8_xchg_destroy: %s", cudaGetErrorString(first));
    return W4A8_OK;
}

W4A8_API w4a8_status w4a8_lmhead_argmax_xchg(const w4a8_weight* w, int32_t row_offset, const int8_t* xq,
                                            const float* xs, int32_t act, int32_t m, float* logits,
                                            uint64_t* best_key, uint32_t* tok_out, const uint32_t* ids,
                                            void* workspace, size_t workspace_bytes, w4a8_xchg* x,
                                            void* stream) {
    if (!x || !x->opened) return set_error(W4A8_EINVAL, "w4a8_lmhead_argmax_xchg: exchange not open");
    if (!best_key) return set_error(W4A8_EINVAL, "w4a8_lmhead_argmax_xchg: best_key is NULL");
    if (m < 1 || m > W4A8_XCHG_MAX_TOKENS)
        return set_error(W4A8_EINVAL, "w4a8_lmhead_argmax_xchg: m=%d not in [1, %d]", m, W4A8_XCHG_MAX_TOKENS);
    unsigned int* err = device_error_word();
    if (!err) return set_error(W4A8_ECUDA, "w4a8_lmhead_argmax_xchg: device error word unavailable");
    // 1. this shard's best key per token (the shard's token is not final: tok NULL)
    w4a8_status s = w4a8_lmhead_argmax(w, row_offset, xq, xs, act, m, logits, best_key, nullptr, nullptr, workspace,
                                       workspace_bytes, stream);
    if (s != W4A8_OK) return s;
    // 2. the exchange, starting while the lm_head kernel finishes
    return launch_pdl("w4a8_lmhead_argmax_xchg: exchange", lmhead_xchg_kernel, dim3(1), dim3(32), 0,
                      static_cast<cudaStream_t>(stream), x->peers, x->world, x->rank, static_cast<int>(m),
                      reinterpret_cast<unsigned long long*>(best_key), tok_out, ids, err);
}

}  // extern "C"
