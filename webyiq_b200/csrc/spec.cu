// The two small kernels of the MTP speculative step around the W4A8 path:
//  - gather_rows (gather_rows.wgsl:1-24): the one-time gather of the draft lm_head,
//    destination row r = source row ids[r], packed weights and scales alike
//    (graph.rs:471-516 builds it from the tied embedding and mtp.head_ids); the
//    draft argmax then runs w4a8_lmhead_argmax on it with ids mapping the index
//    back to the vocabulary (argmax.wgsl:41).
//  - spec_accept (spec_accept.wgsl:1-38): the end of a step that ran the model on
//    tok = [x, d]: the draft d is accepted when it equals the greedy token after x;
//    the step emits y[0] (and y[1] if accepted), the next step runs on [y[a], e[a]]
//    at pos + 1 + a and the DeltaNet state slot advances to (slot + 1 + a) % 3.  The
//    params are read from device memory (they may be the previous step's ctl), so a
//    captured step replays without a host copy.
#include "common.cuh"
#include "launch.cuh"

namespace w4a8 {
namespace {

// One CTA row per output row; 16-byte pieces of the packed row, 4-byte pieces of the
// scale row.  Rows whose id is out of range are left untouched.
__global__ void gather_rows_kernel(const uint4* __restrict__ sq, const uint32_t* __restrict__ ss,
                                   const uint32_t* __restrict__ ids, int n, int qw16, int sw4, uint4* __restrict__ dq,
                                   uint32_t* __restrict__ ds) {
    pdl_launch_dependents();
    pdl_wait();
    const int r = blockIdx.y;
    const uint32_t src = __ldg(ids + r);
    if (src >= static_cast<uint32_t>(n)) return;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < qw16 + sw4; i += gridDim.x * blockDim.x) {
        if (i < qw16)
            dq[static_cast<size_t>(r) * qw16 + i] = __ldg(sq + static_cast<size_t>(src) * qw16 + i);
        else
            ds[static_cast<size_t>(r) * sw4 + (i - qw16)] = __ldg(ss + static_cast<size_t>(src) * sw4 + (i - qw16));
    }
}

__global__ void spec_accept_kernel(uint32_t* tok, const uint32_t* y, const uint32_t* e, const uint32_t* params,
                                   uint32_t* ctl, uint32_t* out) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t pos = params[0], slot = params[3];  // read before ctl (which may alias params) is written
    const uint32_t y0 = y[0], y1 = y[1];
    const uint32_t a = tok[1] == y0 ? 1u : 0u;
    const uint32_t npos = pos + 1u + a, nslot = (slot + 1u + a) % 3u;
    tok[0] = a ? y1 : y0;
    tok[1] = e[a];
    ctl[0] = npos;
    ctl[1] = npos + 2u;
    ctl[2] = 2u;
    ctl[3] = nslot;
    if (out) {
        out[0] = 1u + a;
        out[1] = y0;
        out[2] = y1;
        out[3] = npos;
        out[4] = nslot;
    }
}

}  // namespace
}  // namespace w4a8

using namespace w4a8;

extern "C" {

W4A8_API w4a8_status w4a8_gather_rows(const w4a8_weight* src, const uint32_t* ids, int32_t rows, void* dst_q,
                                     void* dst_s, void* stream) {
    if (!src || !src->q || !src->s || !ids || !dst_q || !dst_s || rows < 1)
        return set_error(W4A8_EINVAL, "w4a8_gather_rows: NULL pointer or rows=%d", rows);
    if (src->group != 32 && src->group != 128) return set_error(W4A8_EINVAL, "w4a8_gather_rows: group %d", src->group);
    if (src->k % src->group) return set_error(W4A8_EINVAL, "w4a8_gather_rows: k=%d", src->k);
    const size_t srow = static_cast<size_t>(src->k / src->group) * (src->has_min ? 4 : 2);  // scale bytes a row
    if ((reinterpret_cast<uintptr_t>(src->q) | reinterpret_cast<uintptr_t>(dst_q)) & 15)
        return set_error(W4A8_EINVAL, "w4a8_gather_rows: packed rows not 16-byte aligned");
    if (srow % 4 || ((reinterpret_cast<uintptr_t>(src->s) | reinterpret_cast<uintptr_t>(dst_s)) & 3))
        return set_error(W4A8_EINVAL, "w4a8_gather_rows: scale rows not in 4-byte units");
    const int qw16 = src->k / 32, sw4 = static_cast<int>(srow / 4);
    const int threads = 128, blocks_x = (qw16 + sw4 + threads - 1) / threads;
    return launch_pdl("w4a8_gather_rows", gather_rows_kernel, dim3(blocks_x, rows), dim3(threads), 0,
                      static_cast<cudaStream_t>(stream), static_cast<const uint4*>(src->q),
                      static_cast<const uint32_t*>(src->s), ids, static_cast<int>(src->n), qw16, sw4,
                      static_cast<uint4*>(dst_q), static_cast<uint32_t*>(dst_s));
}

W4A8_API w4a8_status w4a8_spec_accept(uint32_t* tok, const uint32_t* y, const uint32_t* e, const uint32_t* params,
                                     uint32_t* ctl, uint32_t* out, void* stream) {
    if (!tok || !y || !e || !params || !ctl) return set_error(W4A8_EINVAL, "w4a8_spec_accept: NULL pointer");
    return launch_pdl("w4a8_spec_accept", spec_accept_kernel, dim3(1), dim3(1), 0, static_cast<cudaStream_t>(stream),
                      tok, y, e, params, ctl, out);
}

}  // extern "C"
