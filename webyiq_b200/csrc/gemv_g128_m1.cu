// GEMV instantiations for group 128, has_min 1.
#include "gemv_launch.cuh"

namespace w4a8 {
w4a8_status launch_gemv_g128_m1(const GemvParams& p, int act, int mode, int out, cudaStream_t st) {
    return launch_gemv_gh<128, true>(p, act, mode, out, st);
}
}  // namespace w4a8
