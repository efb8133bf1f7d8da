// w4a8_lmhead_argmax_noalloc: the fused lm_head argmax without a caller-provided
// workspace and without any device allocation.
//
// Who needs it.  Some callers cannot allocate device memory at the point where
// they sample a token: a plugin embedded in a host engine that owns every device
// allocation and hands out only the tensors of the model, or a decode loop that
// must not call cudaMalloc because it synchronizes the whole device.  They still
// own the inputs and outputs; the lm_head argmax needs only a little scratch (a
// count of finished CTAs and one running key per token), so that scratch lives in
// this library instead: one file-scope array per GPU, loaded with the library and
// held until the process exits.
//
// Limits and rules:
//  - The array is kScratchBytes = 256 bytes: the done-counter and the running keys
//    of up to 16 tokens.  Calls with m > 16 are rejected (W4A8_EINVAL).
//  - Every call on a GPU shares its array.  A call leaves it zeroed again, which is
//    the state the next call needs; calls that overlap on the GPU (different
//    streams without ordering) race on it and give wrong results.
//  - The first call on each device does the set-up: with that device current it
//    resolves the array's device address (cudaGetSymbolAddress) and zero-fills it
//    (cudaMemset).  Make that first call outside any stream capture.
//  - No cudaMalloc, cudaFree or allocating library routine is called.
#include <cstring>
#include <mutex>

#include "gemv.cuh"

// The scratch: u32 done-counter at byte 0, u64 running keys of 16 tokens at 128.
static __device__ __align__(256) unsigned char g_lmhead_scratch[256];

namespace w4a8 {
namespace {

constexpr size_t kScratchBytes = sizeof(g_lmhead_scratch);
constexpr int kScratchTokens = 16;
constexpr int kScratchDevices = 64;

std::mutex g_setup_mutex;
void* g_scratch_addr[kScratchDevices] = {nullptr};

// Device address of this device's scratch array (set-up on first use).
w4a8_status scratch_for_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(W4A8_ECUDA, "w4a8_lmhead_argmax_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kScratchDevices) return set_error(W4A8_EINVAL, "w4a8_lmhead_argmax_noalloc: device %d", dev);
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_addr[dev]) {
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_lmhead_scratch);
        if (e != cudaSuccess || !ptr)
            return set_error(W4A8_ECUDA, "w4a8_lmhead_argmax_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        e = cudaMemset(ptr, 0, kScratchBytes);
        if (e != cudaSuccess)
            return set_error(W4A8_ECUDA, "w4a8_lmhead_argmax_noalloc: zero-fill: %s", cudaGetErrorString(e));
        g_scratch_addr[dev] = ptr;
    }
    *out = g_scratch_addr[dev];
    return W4A8_OK;
}

}  // namespace
}  // namespace w4a8

using namespace w4a8;

extern "C" W4A8_API w4a8_status w4a8_lmhead_argmax_noalloc(const w4a8_weight* w, int32_t row_offset,
                                                          const int8_t* xq, const float* xs, int32_t act,
                                                          int32_t m, float* logits, uint64_t* best_key,
                                                          uint32_t* tok_out, const uint32_t* ids, void* stream) {
    if (m > kScratchTokens)
        return set_error(W4A8_EINVAL,
                         "w4a8_lmhead_argmax_noalloc: m=%d exceeds the %d tokens its %zu-byte scratch holds", m,
                         kScratchTokens, kScratchBytes);
    w4a8_status st = check_weight(w, "w4a8_lmhead_argmax_noalloc");
    if (st != W4A8_OK) return st;
    if ((st = check_act(xq, xs, act, "w4a8_lmhead_argmax_noalloc")) != W4A8_OK) return st;
    if (!best_key) return set_error(W4A8_EINVAL, "w4a8_lmhead_argmax_noalloc: best_key is NULL");
    if (m < 1) return set_error(W4A8_EINVAL, "w4a8_lmhead_argmax_noalloc: m=%d", m);
    if (row_offset < 0) return set_error(W4A8_EINVAL, "w4a8_lmhead_argmax_noalloc: row_offset=%d", row_offset);
    void* scratch = nullptr;
    if ((st = scratch_for_current_device(&scratch)) != W4A8_OK) return st;
    GemvParams p{};
    p.q = static_cast<const uint4*>(w->q);
    p.s = w->s;
    p.xq = xq;
    p.xs = xs;
    p.y = logits;
    p.counter = static_cast<unsigned int*>(scratch);
    p.ws_best = reinterpret_cast<unsigned long long*>(static_cast<char*>(scratch) + 128);
    p.best_key = reinterpret_cast<unsigned long long*>(best_key);
    p.tok_out = tok_out;
    p.ids = ids;
    p.n_out = w->n;
    p.y_stride = w->n;
    p.k = w->k;
    p.m = m;
    p.row_offset = row_offset;
    return launch_gemv(p, w->group, w->has_min != 0, act, W4A8_STORE, OUT_ARGMAX, static_cast<cudaStream_t>(stream));
}
