// GEMV instantiations for group 128, has_min 0.
#include "gemv_launch.cuh"

namespace w4a8 {
w4a8_status launch_gemv_g128_m0(const GemvParams& p, int act, int mode, int out, cudaStream_t st) {
    return launch_gemv_gh<128, false>(p, act, mode, out, st);
}
}  // namespace w4a8
