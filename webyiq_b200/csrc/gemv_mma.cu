// Instantiation and launch of the tensor-core GEMV (group 128, per-token int8).
#include "gemv_mma.cuh"
#include "launch.cuh"

namespace w4a8 {

int sm_count();  // capi.cu

namespace {

// One CTA per SM (fewer when rows are scarce) on balanced row ranges; a round is
// RT tiles of 16 rows (8 output rows for SWIGLU); RT x KS warps, KS = ceil(KG/4),
// at most max_warps.  Fills p.ks, p.rt, p.stages and the shared-memory plan; false
// when no plan fits in smem_cap bytes.
bool configure(MmaParams& p, bool swi, bool has_min, int max_warps, size_t smem_cap, int& ctas, MmaSmem& plan) {
    const int kg = p.k / 128;
    p.ks = (kg + kMmaGPS - 1) / kMmaGPS;
    if (p.ks > max_warps) return false;
    const int tr = swi ? 8 : 16;
    const int sms = sm_count();
    ctas = (p.n_out + 7) / 8;
    if (ctas > sms) ctas = sms;
    if (ctas < 1) ctas = 1;
    const int rows = (p.n_out + ctas - 1) / ctas;
    int rt = (rows + tr - 1) / tr;
    const int rt_max = max_warps / p.ks;
    if (rt > rt_max) rt = rt_max;
    p.rt = rt < 1 ? 1 : rt;
    const int rounds = (rows + p.rt * tr - 1) / (p.rt * tr);
    p.stages = rounds < kMmaMaxStages ? rounds : kMmaMaxStages;
    const int sb = has_min ? 4 : 2;
    plan = mma_smem_plan(p.m, p.k, p.rt, p.ks, p.stages, sb);
    while (plan.total > smem_cap && p.stages > 1) plan = mma_smem_plan(p.m, p.k, p.rt, p.ks, --p.stages, sb);
    while (plan.total > smem_cap && p.rt > 1) plan = mma_smem_plan(p.m, p.k, --p.rt, p.ks, p.stages, sb);
    return plan.total <= smem_cap;
}

template <bool HAS_MIN, int MODE, int OUT, int MT, bool FQ>
w4a8_status launch_mt(MmaParams p, cudaStream_t st) {
    constexpr bool SWI = MODE == W4A8_SWIGLU;
    int ctas = 0;
    MmaSmem plan{};
    // Several tokens into y: the two-CTAs-an-SM kernel when a plan of at most 12
    // warps fits twice in an SM
    if constexpr (MT > 1 && !HAS_MIN && OUT == OUT_Y && !FQ) {
        MmaParams q = p;
        if (configure(q, SWI, HAS_MIN, kMmaPairWarps, kMmaPairSmem, ctas, plan)) {
            static FuncAttr attr;
            auto kernel = gemv_mma_kernel<HAS_MIN, MODE, OUT, MT, FQ, true>;
            const w4a8_status a = ensure_smem(kernel, attr, plan.total, 100, "w4a8 gemv (mma)");
            if (a != W4A8_OK) return a;
            return launch_pdl("w4a8 gemv (mma)", kernel, dim3(ctas), dim3(q.rt * q.ks * 32), plan.total, st, q);
        }
    }
    static FuncAttr attr;  // set on first use per device: static shared memory counts against the default 48 KB too
    auto kernel = gemv_mma_kernel<HAS_MIN, MODE, OUT, MT, FQ>;
    if (!configure(p, SWI, HAS_MIN, kMmaMaxWarps, 227 * 1024, ctas, plan)) {
        if (p.ks > kMmaMaxWarps) return set_error(W4A8_EINVAL, "w4a8 gemv: k=%d too large", p.k);
        return set_error(W4A8_EINVAL, "w4a8 gemv: shared memory plan too large");
    }
    const w4a8_status a = ensure_smem(kernel, attr, plan.total, -1, "w4a8 gemv (mma)");
    if (a != W4A8_OK) return a;
    return launch_pdl("w4a8 gemv (mma)", kernel, dim3(ctas), dim3(p.rt * p.ks * 32), plan.total, st, p);
}

template <bool HAS_MIN, int MODE, int OUT, bool FQ = false>
w4a8_status launch_one(const MmaParams& p, cudaStream_t st) {
    if (p.m <= 1) return launch_mt<HAS_MIN, MODE, OUT, 1, FQ>(p, st);
    if (p.m <= 2) return launch_mt<HAS_MIN, MODE, OUT, 2, FQ>(p, st);
    if (p.m <= 4) return launch_mt<HAS_MIN, MODE, OUT, 4, FQ>(p, st);
    return launch_mt<HAS_MIN, MODE, OUT, 8, FQ>(p, st);
}

template <bool HAS_MIN>
w4a8_status launch_mode(const MmaParams& p, int mode, int out, cudaStream_t st) {
    if (p.xf32) {  // f32 activations, quantized inside (OUT_Y only)
        if (mode == W4A8_STORE) return launch_one<HAS_MIN, W4A8_STORE, OUT_Y, true>(p, st);
        if (mode == W4A8_ADD) return launch_one<HAS_MIN, W4A8_ADD, OUT_Y, true>(p, st);
        return launch_one<HAS_MIN, W4A8_SWIGLU, OUT_Y, true>(p, st);
    }
    if (out == OUT_DOTS) return launch_one<HAS_MIN, W4A8_STORE, OUT_DOTS>(p, st);
    if (out == OUT_ARGMAX) return launch_one<HAS_MIN, W4A8_STORE, OUT_ARGMAX>(p, st);
    if (mode == W4A8_STORE) return launch_one<HAS_MIN, W4A8_STORE, OUT_Y>(p, st);
    if (mode == W4A8_ADD) return launch_one<HAS_MIN, W4A8_ADD, OUT_Y>(p, st);
    return launch_one<HAS_MIN, W4A8_SWIGLU, OUT_Y>(p, st);
}

}  // namespace

// GemvParams -> tensor-core launches: outputs into y take up to 16 tokens a launch
// (two mma blocks of 8 over one pass of the weights); the argmax and the group-dot
// hook take 8.
w4a8_status launch_gemv_mma(const GemvParams& g, bool has_min, int mode, int out, cudaStream_t st) {
    const int kg = g.k / 128;
    const int step = out == OUT_Y ? kMmaMaxTokens : kMmaTokens;
    for (int t0 = 0; t0 < g.m; t0 += step) {
        MmaParams p{};
        p.q = g.q;
        p.s = g.s;
        p.m = g.m - t0 < step ? g.m - t0 : step;
        p.xq = g.xq ? g.xq + static_cast<size_t>(t0) * g.k : nullptr;
        p.xf32 = g.xf32 ? g.xf32 + static_cast<size_t>(t0) * g.k : nullptr;
        p.xs = g.xs ? g.xs + t0 : nullptr;
        p.y = g.y ? g.y + static_cast<size_t>(t0) * g.y_stride : nullptr;
        p.dots = g.dots ? g.dots + static_cast<size_t>(t0) * g.n_out * kg : nullptr;
        p.counter = g.counter;
        p.ws_best = g.ws_best ? g.ws_best + t0 : nullptr;
        p.best_key = g.best_key ? g.best_key + t0 : nullptr;
        p.tok_out = g.tok_out ? g.tok_out + t0 : nullptr;
        p.ids = g.ids;
        p.n_out = g.n_out;
        p.k = g.k;
        p.y_stride = g.y_stride;
        p.row_offset = g.row_offset;
        const w4a8_status s = has_min ? launch_mode<true>(p, mode, out, st) : launch_mode<false>(p, mode, out, st);
        if (s != W4A8_OK) return s;
    }
    return W4A8_OK;
}

namespace {

// Failure detection without a fault: one thread waits on an mbarrier that nothing
// ever arrives on, gives up after `limit` cycles like every wait of the library,
// records DEV_ERR_SELFTEST and returns; the context stays usable.
__global__ void selftest_wait_kernel(long long limit) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_init_fence();
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    const uint32_t a = smem_u32(&bar);
    const long long t0 = clock64();
    while (true) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(a)
            : "memory");
        if (done) return;  // cannot happen: nothing arrives
        if (clock64() - t0 > limit) {
            atomicOr(&g_w4a8_dev_error, DEV_ERR_SELFTEST);
            return;
        }
    }
}

}  // namespace

w4a8_status selftest_wait_timeout(cudaStream_t st) {
    selftest_wait_kernel<<<1, 32, 0, st>>>(1ll << 24);  // ~10 ms
    return check_launch("w4a8_selftest_wait_timeout");
}

// Device address of the error word, for kernels compiled in other files (each
// file has its own __device__ variables, so they take it as a parameter).
unsigned int* device_error_word() {
    static std::atomic<unsigned int*> addr[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    unsigned int* a = addr[dev].load(std::memory_order_acquire);
    if (!a) {  // every thread that resolves it first stores the same address
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_w4a8_dev_error) != cudaSuccess) return nullptr;
        a = static_cast<unsigned int*>(p);
        addr[dev].store(a, std::memory_order_release);
    }
    return a;
}

w4a8_status device_error(unsigned int* code, cudaStream_t st) {
    unsigned int v = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_w4a8_dev_error, sizeof(v), 0, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return set_error(W4A8_ECUDA, "w4a8_device_error: %s", cudaGetErrorString(e));
    if (v) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbolAsync(g_w4a8_dev_error, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) return set_error(W4A8_ECUDA, "w4a8_device_error: %s", cudaGetErrorString(e));
    }
    if (code) *code = v;
    return v ? set_error(W4A8_ETIMEOUT, "a bounded device-side wait gave up (code 0x%x)", v) : W4A8_OK;
}

}  // namespace w4a8
