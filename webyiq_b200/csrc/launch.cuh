// Kernel launch with programmatic dependent launch enabled, so a kernel's CTAs may
// be scheduled while the previous kernel in the stream drains (its griddepcontrol
// wait still orders every read of that kernel's output), and the per-device launch
// state of the kernels (raised shared-memory limits, occupancy figures).
#pragma once

#include <atomic>
#include <mutex>

#include "common.cuh"

namespace w4a8 {

// Set to 0 by w4a8_set_pdl(0) (for A/B timing); read at every launch.
extern int g_use_pdl;

constexpr int kMaxDevices = 64;

// The calling thread's current device, or -1 (with the error message set) when it
// cannot be read or is beyond kMaxDevices.
int current_device(const char* what);

// A kernel's attributes (its dynamic shared-memory limit, its carveout) belong to
// the device that is current when they are set, so each kernel instantiation keeps
// one record per device.  The first call on a device sets them under the record's
// lock; later calls read the atomic and skip the lock.  Records live in function-
// local statics (zero-initialised before first use, constructed thread-safely).
struct FuncAttr {
    std::atomic<size_t> smem[kMaxDevices];
    std::mutex mu;
};

// Raise `kernel`'s dynamic shared-memory limit to at least `smem` bytes on the
// current device (and, with carveout >= 0, set its preferred carveout).
template <typename Kernel>
w4a8_status ensure_smem(Kernel kernel, FuncAttr& rec, size_t smem, int carveout, const char* what) {
    const int dev = current_device(what);
    if (dev < 0) return W4A8_ECUDA;
    // 1 marks "attributes set" for kernels that need no more than the default
    if (rec.smem[dev].load(std::memory_order_acquire) >= (smem ? smem : 1)) return W4A8_OK;
    std::lock_guard<std::mutex> lock(rec.mu);
    if (rec.smem[dev].load(std::memory_order_relaxed) >= (smem ? smem : 1)) return W4A8_OK;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return set_error(W4A8_ECUDA, "%s: smem attribute: %s", what, cudaGetErrorString(e));
    if (carveout >= 0) {
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, carveout);
        if (e != cudaSuccess) return set_error(W4A8_ECUDA, "%s: carveout: %s", what, cudaGetErrorString(e));
    }
    rec.smem[dev].store(smem ? smem : 1, std::memory_order_release);
    return W4A8_OK;
}

template <typename Kernel, typename... Args>
w4a8_status launch_pdl(const char* what, Kernel kernel, dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = g_use_pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
    if (e != cudaSuccess) return set_error(W4A8_ECUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
    return W4A8_OK;
}

}  // namespace w4a8
