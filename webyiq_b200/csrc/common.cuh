// Device helpers shared by the W4A8 kernels: f16 scale decoding into exact fixed
// point, nibble unpack + dp4a group dots, the packed argmax key, status plumbing.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "w4a8.h"

namespace w4a8 {

// ---------------------------------------------------------------------------
// Host-side status helpers (defined in capi.cu)
w4a8_status set_error(w4a8_status st, const char* fmt, ...);
w4a8_status check_launch(const char* what);
// Argument checks of the entry points (EINVAL with a message naming `what`): a
// weight view's group, shape and pointer alignment; activation pointers, layout
// and alignment (xq 16 bytes, xs 8 bytes for W4A8_ACT_GROUP32, else 4).
w4a8_status check_weight(const w4a8_weight* w, const char* what);
w4a8_status check_act(const int8_t* xq, const float* xs, int act, const char* what);
bool aligned(const void* p, size_t a);

constexpr int kWarp = 32;
constexpr unsigned kFull = 0xffffffffu;

// ---------------------------------------------------------------------------
// Packed weights (tools/convert.py:7-11): in each u32 of a row, byte b holds
// w[8i+b] in its low nibble and w[8i+4+b] in its high nibble, so the low nibbles
// are 4 consecutive weights and the high nibbles the next 4.
__device__ __forceinline__ uint32_t lo_nibbles(uint32_t u) { return u & 0x0F0F0F0Fu; }
__device__ __forceinline__ uint32_t hi_nibbles(uint32_t u) { return (u >> 4) & 0x0F0F0F0Fu; }

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) {
    // signed x signed byte dot; nibble bytes are 0..15 so they read the same signed
    return __dp4a(static_cast<int>(a), static_cast<int>(b), c);
}

// Dot product of the 32 weights of one 16-byte chunk (4 words) with 32 int8
// activations (8 words xa, xb), added to d: the same term order as gdot
// (gemv_q4q8.wgsl:29-34), although any order gives the same int32.
__device__ __forceinline__ int chunk_dot(const uint32_t lo[4], const uint32_t hi[4], const uint4& xa,
                                         const uint4& xb, int d) {
    d = dp4a(lo[0], xa.x, d);
    d = dp4a(hi[0], xa.y, d);
    d = dp4a(lo[1], xa.z, d);
    d = dp4a(hi[1], xa.w, d);
    d = dp4a(lo[2], xb.x, d);
    d = dp4a(hi[2], xb.y, d);
    d = dp4a(lo[3], xb.z, d);
    d = dp4a(hi[3], xb.w, d);
    return d;
}

// Sum of the 32 int8 activations of a chunk.
__device__ __forceinline__ int chunk_sum(const uint4& xa, const uint4& xb) {
    const uint32_t ones = 0x01010101u;
    int s = 0;
    s = dp4a(ones, xa.x, s);
    s = dp4a(ones, xa.y, s);
    s = dp4a(ones, xa.z, s);
    s = dp4a(ones, xa.w, s);
    s = dp4a(ones, xb.x, s);
    s = dp4a(ones, xb.y, s);
    s = dp4a(ones, xb.z, s);
    s = dp4a(ones, xb.w, s);
    return s;
}

// ---------------------------------------------------------------------------
// An f16 value h is exactly mant * 2^sh * 2^-24 with a signed integer mantissa
// |mant| <= 2047 and 0 <= sh <= 29 (normal: (1024|f) << (e-1); subnormal: f).
// A group term mant * I fits int32 for |I| < 2^20, and shifting it by sh in int64
// keeps the whole row sum exact.  Non-finite scales (e = 31) are outside the
// format; they decode deterministically (sh = 30) and give meaningless output.
struct Fix16 {
    int mant;
    int sh;
};

__device__ __host__ __forceinline__ Fix16 fix16(uint32_t h) {
    const int e = (h >> 10) & 31;
    const int f = h & 1023;
    int mant = e ? (f | 1024) : f;
    if (h & 0x8000u) mant = -mant;
    return Fix16{mant, e ? e - 1 : 0};
}

__device__ __forceinline__ long long shl64(int p, int sh) {
    return static_cast<long long>(static_cast<unsigned long long>(static_cast<long long>(p)) << sh);
}

// Output of the exact path: ((float)acc * 2^-24) * dx, two round-to-nearest steps.
__device__ __forceinline__ float fix_to_float(long long acc, float dx) {
    float t = __ll2float_rn(acc);
    t = __fmul_rn(t, 5.9604644775390625e-08f);  // 2^-24, exact
    return __fmul_rn(t, dx);
}

__device__ __forceinline__ float silu_mul(float a, float u) {
    // gemv_q4q8.wgsl:128: a / (1 + exp(-a)) * u
    return __fdiv_rn(a, __fadd_rn(1.0f, expf(-a))) * u;
}

// ---------------------------------------------------------------------------
// Packed argmax key (argmax.wgsl:17-39 semantics).  Valid values are v > -3e38
// (NaN and anything <= -3e38 never win).  The float is mapped to an unsigned
// integer with the same order (-0 taken as +0, since the reference compares with
// `>` and `==`), placed in the high word; the low word is ~index so that, among
// equal values, the lowest index has the largest key.  Key 0 means "no valid
// value" and decodes to index 0, as the reference returns for such a row.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    if (!(v > -3.0e38f)) return 0ull;
    uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(b) << 32) | static_cast<unsigned long long>(~idx);
}

__device__ __forceinline__ unsigned long long shfl_xor_u64(unsigned long long v, int m) {
    return __shfl_xor_sync(kFull, v, m);
}

__device__ __forceinline__ long long shfl_xor_i64(long long v, int m) {
    return __shfl_xor_sync(kFull, v, m);
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch: a kernel may start while the previous kernel in
// the stream is finishing; it must wait before touching that kernel's outputs.
__device__ __forceinline__ void pdl_wait() {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
    asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}
// A load of data that an earlier kernel of the chain writes (activations, their
// scales, logits), after pdl_wait.  A plain global load (.ca): L1 lines are
// invalidated between dependent grids, so it sees the writes, and the warps of an
// SM share the L1 copy of the few lines of an activation vector.  Not __ldg
// (ld.global.nc): a kernel launched early is resident while that data is still
// being written, which breaks the read-only contract of the non-coherent path (a
// chain whose inputs change between steps read stale lines).  Not ld.global.cg:
// bypassing L1, every warp of every SM requests the same L2 lines at once.
template <typename T>
__device__ __forceinline__ T ld_dep(const T* p) {
    return *p;
}

__device__ __forceinline__ void pdl_launch_dependents() {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
}

// Read-only, no-L1-allocate 16-byte load for streamed weights.
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

}  // namespace w4a8
