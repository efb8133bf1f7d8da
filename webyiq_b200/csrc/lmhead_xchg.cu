// Column-split lm_head with the key exchange over peer memory: each rank runs the
// fused lm_head argmax on its vocabulary shard (global ids through row_offset), and
// the merge of xchg.cuh gives every rank the global key and token: the rank's packed
// keys, tagged with the call's sequence number, are stored into every peer's
// exchange buffer (NVLink stores to memory opened through CUDA IPC), and the max is
// taken once every rank's keys of the call have arrived (bounded waits).
//
// Where the streaming lm_head kernel covers the call, its last CTA (the one that
// publishes the shard's key) runs the merge itself, so a call is one kernel.  The
// other lm_head kernels leave the shard's key for a 32-thread merge kernel that
// starts under programmatic dependent launch.  Against the NCCL all-reduce of
// lmhead_multi.cu this drops a collective launch and a key-to-token kernel; the
// exchange is one store per (peer, token), each peer served by its own thread.  A
// wait that gives up leaves the rank's own key and token in the outputs and sets
// the device error word.  Nothing here uses NVLink multicast objects; the buffers
// are plain device memory.
#include <cstring>

#include "launch.cuh"
#include "xchg.cuh"

namespace w4a8 {

unsigned int* device_error_word();  // gemv_mma.cu
// The lm_head argmax of capi.cu; with x, the streaming kernel runs the merge in its
// last CTA when it covers the call (*fused), otherwise the shard's key is left in
// best_key and no token is written.
w4a8_status lmhead_argmax_impl(const w4a8_weight* w, int32_t row_offset, const int8_t* xq, const float* xs,
                               int32_t act, int32_t m, float* logits, uint64_t* best_key, uint32_t* tok_out,
                               const uint32_t* ids, void* workspace, size_t workspace_bytes, void* stream,
                               const XchgArgs* x, bool* fused);

namespace {

// The merge as a kernel of its own, for the lm_head kernels that do not run it.
__global__ void __launch_bounds__(32) lmhead_xchg_kernel(const XchgArgs x, int m, unsigned long long* best_key,
                                                         uint32_t* tok_out, const uint32_t* ids, unsigned int* err) {
    pdl_launch_dependents();
    pdl_wait();  // best_key comes from the lm_head kernel
    __shared__ unsigned long long s_own[W4A8_XCHG_MAX_TOKENS];
    __shared__ unsigned int s_seq;
    if (static_cast<int>(threadIdx.x) < m) s_own[threadIdx.x] = ld_dep(best_key + threadIdx.x);
    if (threadIdx.x == 0) s_seq = xchg_next_seq(x);
    __syncthreads();
    xchg_merge(x, m, s_seq, s_own, best_key, tok_out, ids, err);
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
    // the exchanged keys carry the call's tag in the top 8 bits of the id half
    if (!w || row_offset < 0 || static_cast<long long>(row_offset) + w->n > (1ll << 24))
        return set_error(W4A8_EINVAL, "w4a8_lmhead_argmax_xchg: ids [row_offset, row_offset + n) must lie below 2^24");
    unsigned int* err = device_error_word();
    if (!err) return set_error(W4A8_ECUDA, "w4a8_lmhead_argmax_xchg: device error word unavailable");
    // The shard's lm_head; the streaming kernel merges in its last CTA, the
    // others leave the shard's key (no token) for the merge kernel, which starts
    // under programmatic dependent launch while the lm_head kernel finishes.
    const XchgArgs xa{x->peers, x->world, x->rank};
    bool fused = false;
    w4a8_status s = lmhead_argmax_impl(w, row_offset, xq, xs, act, m, logits, best_key, tok_out, ids, workspace,
                                       workspace_bytes, stream, &xa, &fused);
    if (s != W4A8_OK || fused) return s;
    return launch_pdl("w4a8_lmhead_argmax_xchg: exchange", lmhead_xchg_kernel, dim3(1), dim3(32), 0,
                      static_cast<cudaStream_t>(stream), xa, static_cast<int>(m),
                      reinterpret_cast<unsigned long long*>(best_key), tok_out, ids, err);
}

}  // extern "C"
