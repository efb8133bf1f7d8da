// Host side of the W4A8 path in C++, mirroring the reference engine's operator
// surface over the C ABI of include/w4a8.h:
//   Manifest          manifest.rs:6-95 (parse + validation, shard sizes)
//   Engine            lib.rs:41-48 (owns one device buffer per tensor),
//                     lib.rs:177-187 (upload_shard)
//   Builder           graph.rs:190-222 (gemv, gemm, matmul, quant) and the argmax /
//                     lm_head ops of head_ops (graph.rs:476-486)
// Errors are returned as Status (the reference's Result<_, String>); nothing
// throws across the C ABI.  The reference records wgpu compute passes and submits
// them in queue order; here the Builder records C-ABI calls into a Plan that runs
// them in order on one CUDA stream, or captures them once into a CUDA graph and
// replays it (one launch per decode step).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <map>
#include <string>
#include <vector>

#include "json.h"
#include "w4a8.h"

namespace webyiq {

struct Status {
    std::string err;  // empty: success
    bool ok() const { return err.empty(); }
    static Status Ok() { return Status{}; }
    static Status Error(std::string e) { return Status{std::move(e)}; }
};

struct TensorInfo {
    size_t shard = 0;
    uint64_t offset = 0, bytes = 0;
    std::string dtype;
    std::vector<uint64_t> shape;
};

struct Manifest {
    std::string format, arch;
    Json config;
    uint32_t bits = 0, group = 0;
    std::string scheme;
    std::vector<std::string> shards;
    std::map<std::string, TensorInfo> tensors;

    // Manifest::parse (manifest.rs:77-86): format "webyiq-v2", arch llama | qwen3_5,
    // 4-bit quantization with group 32 (the engine's) or 128.
    static Status parse(const std::string& json, Manifest& out);
    // Reads <dir>/manifest.json and parses it.
    static Status load(const std::string& dir, Manifest& out);
    // Bytes each shard file must hold (manifest.rs:88-95).
    std::vector<uint64_t> shard_bytes() const;
};

struct DeviceBuffer {
    void* ptr = nullptr;
    size_t bytes = 0;
};

class Engine {
public:
    Engine(Manifest m, std::string dir);
    ~Engine();
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;

    // One device buffer per tensor (sized from the manifest).
    Status alloc();
    // Copies every tensor stored in shard `idx` from `data` (the whole shard file)
    // into its own buffer (lib.rs:177-187).
    Status upload_shard(size_t idx, const std::vector<uint8_t>& data);
    // alloc(), then each shard file read and uploaded in turn.
    Status load_all();

    const Manifest& manifest() const { return m_; }
    const DeviceBuffer* buffer(const std::string& name) const;
    // The q4 weight `name` ({name}.q packed nibbles, {name}.s scales) as a C-ABI
    // view; has_min follows the scale size (4 bytes: f16 scale | f16 min; 2 bytes:
    // f16 scale, symmetric).
    Status weight(const std::string& name, w4a8_weight& out) const;

private:
    Manifest m_;
    std::string dir_;
    std::map<std::string, DeviceBuffer> bufs_;
};

// One recorded call of the C ABI.
struct Op {
    std::string name;
    std::function<w4a8_status(cudaStream_t)> run;
};

// graph.rs Path: decode (1 token), speculative verify (T tokens), prefill.
enum class Path { Decode, Verify, Prefill };

class Builder {
public:
    explicit Builder(const Engine& e) : e_(e) {}

    // y (+)= W x for t tokens (graph.rs:190-198); W = {w}.q / {w}.s, N % 8 == 0.
    Status gemv(const std::string& name, const std::string& w, uint32_t k, uint32_t n, uint32_t mode, uint32_t t,
                const int8_t* xq, const float* xs, int act, float* y);
    // Prefill GEMM over m tokens (graph.rs:200-205); N % 32 == 0, K % 128 == 0.
    Status gemm(const std::string& name, const std::string& w, uint32_t k, uint32_t n, uint32_t mode, uint32_t m,
                const int8_t* xq, const float* xs, int act, float* y);
    // GEMM for prefill, GEMV otherwise (graph.rs:207-214).
    Status matmul(Path path, uint32_t tokens, const std::string& name, const std::string& w, uint32_t k, uint32_t n,
                  uint32_t mode, const int8_t* xq, const float* xs, int act, float* y);
    // int8 quantization of `rows` rows of x (k wide), RMSNorm'ed with `norm` if not
    // null (graph.rs:216-222, quant.wgsl).
    Status quant(const std::string& name, uint32_t k, double eps, const float* x, const float* norm, uint32_t rows,
                 int act, int8_t* xq, float* xs);
    // The norm_quant prologue and the projection in one launch (graph.rs:266,323 then
    // 190-198): x f32 [t, k] RMSNorm'ed with `norm` (f32 [k], or none if null),
    // quantized per token and y (+)= W x, bit-identical to quant + gemv
    // (w4a8_gemv_x / w4a8_gemv_xn); group-128 weights, t <= 2 with a norm.
    Status quant_gemv(const std::string& name, const std::string& w, uint32_t k, uint32_t n, uint32_t mode,
                      uint32_t t, const float* x, const float* norm, double eps, float* y);
    // Greedy token per row of logits [rows, v] (argmax.wgsl, graph.rs:484).
    Status argmax(const std::string& name, const float* logits, uint32_t rows, uint32_t v, const uint32_t* ids,
                  uint32_t* tok);
    // lm_head GEMV with the argmax fused (head_ops, graph.rs:476-486).
    Status lm_head(const std::string& name, const std::string& w, uint32_t k, uint32_t rows, const int8_t* xq,
                   const float* xs, int act, float* logits, uint64_t* key, uint32_t* tok, const uint32_t* ids,
                   void* workspace, size_t workspace_bytes);

    const std::vector<Op>& ops() const { return ops_; }
    std::vector<Op> take() { return std::move(ops_); }

private:
    Status w(const std::string& name, uint32_t k, uint32_t n, w4a8_weight& out) const;
    const Engine& e_;
    std::vector<Op> ops_;
};

// Runs recorded ops in order on a stream, or as one captured CUDA graph.
class Plan {
public:
    explicit Plan(std::vector<Op> ops) : ops_(std::move(ops)) {}
    ~Plan();
    Plan(const Plan&) = delete;
    Plan& operator=(const Plan&) = delete;

    Status run(cudaStream_t st) const;
    Status capture(cudaStream_t st);
    Status replay(cudaStream_t st) const;
    size_t size() const { return ops_.size(); }

private:
    std::vector<Op> ops_;
    cudaGraph_t graph_ = nullptr;
    cudaGraphExec_t exec_ = nullptr;
};

// Reads a whole file; false on failure.
bool read_file(const std::string& path, std::vector<uint8_t>& out);

}  // namespace webyiq
