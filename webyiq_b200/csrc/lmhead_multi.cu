// Column-split lm_head across GPUs: every rank holds a contiguous block of
// vocabulary rows, runs the fused lm_head argmax on it (rows carry their global
// ids through row_offset) and the ranks then all-reduce the packed argmax keys with
// NCCL (max over u64).  A key orders first by the logit and then by the lowest
// index, so the reduced key is exactly the one-GPU argmax (argmax.wgsl:17-39
// semantics: strict '>' scan, lowest index on ties, NaN never wins).
//
// Reference: head_ops (graph.rs:476-486) computes the whole vocabulary on one
// device; here the exchange step of the sharded head replaces the all-gather of
// (max, index) pairs.  NCCL is opened at run time (dlopen of libnccl.so.2), so the
// library has no link-time NCCL dependency; inside a PyTorch process that resolves
// to the NCCL PyTorch already loaded.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace w4a8 {
namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
    char why[256] = "";
};

NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            snprintf(api.why, sizeof(api.why), "libnccl.so.2 not found: %s", dlerror());
            return;
        }
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce && api.error_string;
        if (!api.ok) snprintf(api.why, sizeof(api.why), "libnccl.so.2 lacks an expected symbol");
    });
    return api;
}

w4a8_status nccl_error(const char* what, ncclResult_t r) {
    return set_error(W4A8_ENCCL, "%s: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
}

// tok[t] = ids[index] (or index) of the reduced key of token t.
__global__ void key_to_token_kernel(const unsigned long long* key, const uint32_t* ids, uint32_t* tok, int m) {
    const int t = threadIdx.x;
    if (t < m) {
        const unsigned long long k = key[t];
        const uint32_t idx = k ? ~static_cast<uint32_t>(k & 0xffffffffull) : 0u;
        tok[t] = ids ? ids[idx] : idx;
    }
}

}  // namespace
}  // namespace w4a8

using namespace w4a8;

extern "C" {

W4A8_API w4a8_status w4a8_nccl_get_unique_id(void* id_out) {
    if (!id_out) return set_error(W4A8_EINVAL, "w4a8_nccl_get_unique_id: NULL");
    if (!nccl().ok) return set_error(W4A8_ENCCL, "w4a8_nccl_get_unique_id: %s", nccl().why);
    ncclUniqueId id;
    const ncclResult_t r = nccl().get_unique_id(&id);
    if (r != ncclSuccess) return nccl_error("ncclGetUniqueId", r);
    memcpy(id_out, &id, sizeof(id));
    return W4A8_OK;
}

W4A8_API w4a8_status w4a8_nccl_comm_init(int32_t nranks, const void* id, int32_t rank, void** comm_out) {
    if (!id || !comm_out || nranks < 1 || rank < 0 || rank >= nranks)
        return set_error(W4A8_EINVAL, "w4a8_nccl_comm_init: nranks=%d rank=%d", nranks, rank);
    if (!nccl().ok) return set_error(W4A8_ENCCL, "w4a8_nccl_comm_init: %s", nccl().why);
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclComm_t comm = nullptr;
    const ncclResult_t r = nccl().comm_init_rank(&comm, nranks, uid, rank);
    if (r != ncclSuccess) return nccl_error("ncclCommInitRank", r);
    *comm_out = comm;
    return W4A8_OK;
}

W4A8_API w4a8_status w4a8_nccl_comm_destroy(void* comm) {
    if (!comm) return W4A8_OK;
    if (!nccl().ok) return set_error(W4A8_ENCCL, "w4a8_nccl_comm_destroy: %s", nccl().why);
    const ncclResult_t r = nccl().comm_destroy(static_cast<ncclComm_t>(comm));
    if (r != ncclSuccess) return nccl_error("ncclCommDestroy", r);
    return W4A8_OK;
}

W4A8_API w4a8_status w4a8_lmhead_argmax_allreduce(const w4a8_weight* w, int32_t row_offset, const int8_t* xq,
                                                  const float* xs, int32_t act, int32_t m, float* logits,
                                                  uint64_t* best_key, uint32_t* tok_out, const uint32_t* ids,
                                                  void* workspace, size_t workspace_bytes, void* nccl_comm,
                                                  void* stream) {
    if (!nccl_comm) return set_error(W4A8_EINVAL, "w4a8_lmhead_argmax_allreduce: nccl_comm is NULL");
    if (!best_key) return set_error(W4A8_EINVAL, "w4a8_lmhead_argmax_allreduce: best_key is NULL");
    if (!nccl().ok) return set_error(W4A8_ENCCL, "w4a8_lmhead_argmax_allreduce: %s", nccl().why);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    // 1. this shard's best key per token (the shard's token is not final: tok NULL)
    w4a8_status s = w4a8_lmhead_argmax(w, row_offset, xq, xs, act, m, logits, best_key, nullptr, nullptr, workspace,
                                       workspace_bytes, stream);
    if (s != W4A8_OK) return s;
    // 2. max over the ranks (in place, u64 compare = key order)
    const ncclResult_t r = nccl().all_reduce(best_key, best_key, static_cast<size_t>(m), ncclUint64, ncclMax,
                                             static_cast<ncclComm_t>(nccl_comm), st);
    if (r != ncclSuccess) return nccl_error("w4a8_lmhead_argmax_allreduce: ncclAllReduce", r);
    // 3. the winning token on every rank
    if (tok_out) {
        key_to_token_kernel<<<1, 32, 0, st>>>(reinterpret_cast<const unsigned long long*>(best_key), ids, tok_out, m);
        return check_launch("w4a8_lmhead_argmax_allreduce: key_to_token");
    }
    return W4A8_OK;
}

}  // extern "C"
