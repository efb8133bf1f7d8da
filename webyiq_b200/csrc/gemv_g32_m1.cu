// GEMV instantiations for group 32, has_min 1.
#include "gemv_launch.cuh"

namespace w4a8 {
w4a8_status launch_gemv_g32_m1(const GemvParams& p, int act, int mode, int out, cudaStream_t st) {
    return launch_gemv_gh<32, true>(p, act, mode, out, st);
}
}  // namespace w4a8
