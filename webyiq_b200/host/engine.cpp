#include "engine.h"

#include <cstdarg>
#include <cstdio>
#include <fstream>
#include <sstream>

namespace webyiq {

namespace {

std::string str(const char* fmt, ...) __attribute__((format(printf, 1, 2)));
std::string str(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    return buf;
}

Status cuda_status(const char* what, cudaError_t e) {
    return e == cudaSuccess ? Status::Ok() : Status::Error(str("%s: %s", what, cudaGetErrorString(e)));
}

Status abi_status(const std::string& what, w4a8_status s) {
    return s == W4A8_OK ? Status::Ok() : Status::Error(what + ": " + w4a8_last_error());
}

}  // namespace

bool read_file(const std::string& path, std::vector<uint8_t>& out) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    f.seekg(0, std::ios::end);
    const std::streamoff n = f.tellg();
    if (n < 0) return false;
    f.seekg(0, std::ios::beg);
    out.resize(static_cast<size_t>(n));
    if (n > 0 && !f.read(reinterpret_cast<char*>(out.data()), n)) return false;
    return true;
}

// --- Manifest --------------------------------------------------------------------

Status Manifest::parse(const std::string& json, Manifest& out) {
    Json j;
    std::string err;
    if (!parse_json(json, j, err)) return Status::Error("manifest.json: " + err);
    out = Manifest();
    out.format = j["format"].str;
    out.arch = j["arch"].str;
    if (out.format != "webyiq-v2" || (out.arch != "llama" && out.arch != "qwen3_5"))
        return Status::Error("unsupported model: " + out.format + " / " + out.arch);
    const Json& q = j["quant"];
    out.bits = static_cast<uint32_t>(q["bits"].num);
    out.group = static_cast<uint32_t>(q["group"].num);
    out.scheme = q["scheme"].str;
    if (out.bits != 4 || (out.group != 32 && out.group != 128))
        return Status::Error(str("unsupported quant: bits %u group %u scheme %s", out.bits, out.group,
                                 out.scheme.c_str()));
    out.config = j["config"];
    for (const Json& s : j["shards"].arr) out.shards.push_back(s.str);
    for (const auto& kv : j["tensors"].obj) {
        const Json& t = kv.second;
        TensorInfo ti;
        if (t["shard"].kind != Json::Number || t["offset"].kind != Json::Number || t["bytes"].kind != Json::Number)
            return Status::Error("tensor " + kv.first + ": shard/offset/bytes missing");
        ti.shard = static_cast<size_t>(t["shard"].num);
        ti.offset = static_cast<uint64_t>(t["offset"].num);
        ti.bytes = static_cast<uint64_t>(t["bytes"].num);
        ti.dtype = t["dtype"].str;
        for (const Json& d : t["shape"].arr) ti.shape.push_back(static_cast<uint64_t>(d.num));
        if (ti.shard >= out.shards.size()) return Status::Error("tensor " + kv.first + ": shard index out of range");
        out.tensors[kv.first] = ti;
    }
    return Status::Ok();
}

Status Manifest::load(const std::string& dir, Manifest& out) {
    std::vector<uint8_t> raw;
    if (!read_file(dir + "/manifest.json", raw)) return Status::Error("cannot read " + dir + "/manifest.json");
    return parse(std::string(raw.begin(), raw.end()), out);
}

std::vector<uint64_t> Manifest::shard_bytes() const {
    std::vector<uint64_t> sizes(shards.size(), 0);
    for (const auto& kv : tensors) {
        const TensorInfo& t = kv.second;
        if (t.offset + t.bytes > sizes[t.shard]) sizes[t.shard] = t.offset + t.bytes;
    }
    return sizes;
}

// --- Engine ----------------------------------------------------------------------

Engine::Engine(Manifest m, std::string dir) : m_(std::move(m)), dir_(std::move(dir)) {}

Engine::~Engine() {
    for (auto& kv : bufs_)
        if (kv.second.ptr) cudaFree(kv.second.ptr);
}

Status Engine::alloc() {
    for (const auto& kv : m_.tensors) {
        if (bufs_.count(kv.first)) continue;
        DeviceBuffer b;
        b.bytes = static_cast<size_t>(kv.second.bytes);
        const Status s = cuda_status(("alloc " + kv.first).c_str(), cudaMalloc(&b.ptr, b.bytes ? b.bytes : 16));
        if (!s.ok()) return s;
        bufs_[kv.first] = b;
    }
    return Status::Ok();
}

Status Engine::upload_shard(size_t idx, const std::vector<uint8_t>& data) {
    for (const auto& kv : m_.tensors) {
        const TensorInfo& t = kv.second;
        if (t.shard != idx) continue;
        if (t.offset + t.bytes > data.size())
            return Status::Error(str("tensor %s past the end of shard %zu (%llu+%llu > %zu)", kv.first.c_str(), idx,
                                     static_cast<unsigned long long>(t.offset),
                                     static_cast<unsigned long long>(t.bytes), data.size()));
        auto it = bufs_.find(kv.first);
        if (it == bufs_.end()) return Status::Error("upload before alloc: " + kv.first);
        const Status s = cuda_status(("upload " + kv.first).c_str(),
                                     cudaMemcpy(it->second.ptr, data.data() + t.offset, t.bytes, cudaMemcpyHostToDevice));
        if (!s.ok()) return s;
    }
    return Status::Ok();
}

Status Engine::load_all() {
    Status s = alloc();
    if (!s.ok()) return s;
    for (size_t i = 0; i < m_.shards.size(); ++i) {
        std::vector<uint8_t> data;
        if (!read_file(dir_ + "/" + m_.shards[i], data)) return Status::Error("cannot read shard " + m_.shards[i]);
        s = upload_shard(i, data);
        if (!s.ok()) return s;
    }
    return Status::Ok();
}

const DeviceBuffer* Engine::buffer(const std::string& name) const {
    auto it = bufs_.find(name);
    return it == bufs_.end() ? nullptr : &it->second;
}

Status Engine::weight(const std::string& name, w4a8_weight& out) const {
    auto tq = m_.tensors.find(name + ".q");
    auto ts = m_.tensors.find(name + ".s");
    if (tq == m_.tensors.end()) return Status::Error("missing tensor " + name + ".q");
    if (ts == m_.tensors.end()) return Status::Error("missing tensor " + name + ".s");
    const std::vector<uint64_t>& shape = tq->second.shape;
    if (shape.size() != 2) return Status::Error("tensor " + name + ".q: expected a 2-D shape [n, k]");
    const uint64_t n = shape[0], k = shape[1], g = m_.group;
    if (k % g || tq->second.bytes != n * k / 2)
        return Status::Error(str("tensor %s: %llu bytes do not match shape %llux%llu", name.c_str(),
                                 static_cast<unsigned long long>(tq->second.bytes), static_cast<unsigned long long>(n),
                                 static_cast<unsigned long long>(k)));
    int has_min;
    if (ts->second.bytes == n * (k / g) * 4)
        has_min = 1;
    else if (ts->second.bytes == n * (k / g) * 2)
        has_min = 0;
    else
        return Status::Error("tensor " + name + ".s: size matches neither (scale, min) u32 nor f16 scales");
    const DeviceBuffer* bq = buffer(name + ".q");
    const DeviceBuffer* bs = buffer(name + ".s");
    if (!bq || !bs) return Status::Error("tensor " + name + " not on the device (alloc / upload first)");
    return abi_status("weight " + name, w4a8_weight_view(bq->ptr, bs->ptr, static_cast<int32_t>(n),
                                                         static_cast<int32_t>(k), static_cast<int32_t>(g), has_min, &out));
}

// --- Builder ---------------------------------------------------------------------

Status Builder::w(const std::string& name, uint32_t k, uint32_t n, w4a8_weight& out) const {
    const Status s = e_.weight(name, out);
    if (!s.ok()) return s;
    if (static_cast<uint32_t>(out.k) != k || static_cast<uint32_t>(out.n) != n)
        return Status::Error(str("tensor %s is %dx%d, op wants %ux%u", name.c_str(), out.n, out.k, n, k));
    return Status::Ok();
}

Status Builder::gemv(const std::string& name, const std::string& wn, uint32_t k, uint32_t n, uint32_t mode, uint32_t t,
                     const int8_t* xq, const float* xs, int act, float* y) {
    w4a8_weight wt;
    Status s = w(wn, k, n, wt);
    if (!s.ok()) return s;
    if (n % 8) return Status::Error(str("%s: gemv rows %u not a multiple of 8", name.c_str(), n));
    if (t < 1 || t > W4A8_GEMV_MAX_M) return Status::Error(str("%s: gemv tokens %u", name.c_str(), t));
    ops_.push_back({name, [=](cudaStream_t st) {
                        return w4a8_gemv(&wt, xq, xs, act, static_cast<int32_t>(t), static_cast<int32_t>(mode), y, st);
                    }});
    return Status::Ok();
}

Status Builder::gemm(const std::string& name, const std::string& wn, uint32_t k, uint32_t n, uint32_t mode, uint32_t m,
                     const int8_t* xq, const float* xs, int act, float* y) {
    w4a8_weight wt;
    Status s = w(wn, k, n, wt);
    if (!s.ok()) return s;
    if (n % 32 || k % 128) return Status::Error(str("%s: gemm needs n %% 32 == 0 and k %% 128 == 0 (%ux%u)", name.c_str(), n, k));
    if (m < 1) return Status::Error(str("%s: gemm tokens %u", name.c_str(), m));
    ops_.push_back({name, [=](cudaStream_t st) {
                        return w4a8_gemm(&wt, xq, xs, act, static_cast<int32_t>(m), static_cast<int32_t>(mode), y, st);
                    }});
    return Status::Ok();
}

Status Builder::matmul(Path path, uint32_t tokens, const std::string& name, const std::string& wn, uint32_t k,
                       uint32_t n, uint32_t mode, const int8_t* xq, const float* xs, int act, float* y) {
    if (path == Path::Prefill) return gemm(name, wn, k, n, mode, tokens, xq, xs, act, y);
    return gemv(name, wn, k, n, mode, path == Path::Decode ? 1 : tokens, xq, xs, act, y);
}

Status Builder::quant(const std::string& name, uint32_t k, double eps, const float* x, const float* norm, uint32_t rows,
                      int act, int8_t* xq, float* xs) {
    if (k % 32) return Status::Error(str("%s: quant width %u not a multiple of 32", name.c_str(), k));
    ops_.push_back({name, [=](cudaStream_t st) {
                        return w4a8_quant(x, norm, static_cast<float>(eps), static_cast<int32_t>(rows),
                                          static_cast<int32_t>(k), act, xq, xs, st);
                    }});
    return Status::Ok();
}

Status Builder::quant_gemv(const std::string& name, const std::string& wn, uint32_t k, uint32_t n, uint32_t mode,
                          uint32_t t, const float* x, const float* norm, double eps, float* y) {
    w4a8_weight wt;
    Status s = w(wn, k, n, wt);
    if (!s.ok()) return s;
    if (wt.group != 128) return Status::Error(str("%s: quant_gemv needs group-128 weights (group %d)", name.c_str(), wt.group));
    if (t < 1 || t > (norm ? 2u : static_cast<uint32_t>(W4A8_GEMV_MAX_M)))
        return Status::Error(str("%s: quant_gemv tokens %u", name.c_str(), t));
    ops_.push_back({name, [=](cudaStream_t st) {
                        if (norm)
                            return w4a8_gemv_xn(&wt, x, norm, static_cast<float>(eps), static_cast<int32_t>(t),
                                                static_cast<int32_t>(mode), y, st);
                        return w4a8_gemv_x(&wt, x, static_cast<int32_t>(t), static_cast<int32_t>(mode), y, st);
                    }});
    return Status::Ok();
}

Status Builder::argmax(const std::string& name, const float* logits, uint32_t rows, uint32_t v, const uint32_t* ids,
                       uint32_t* tok) {
    ops_.push_back({name, [=](cudaStream_t st) {
                        return w4a8_argmax(logits, static_cast<int32_t>(rows), static_cast<int32_t>(v), ids, tok, st);
                    }});
    return Status::Ok();
}

Status Builder::lm_head(const std::string& name, const std::string& wn, uint32_t k, uint32_t rows, const int8_t* xq,
                        const float* xs, int act, float* logits, uint64_t* key, uint32_t* tok, const uint32_t* ids,
                        void* workspace, size_t workspace_bytes) {
    w4a8_weight wt;
    Status s = e_.weight(wn, wt);
    if (!s.ok()) return s;
    if (static_cast<uint32_t>(wt.k) != k) return Status::Error(str("%s: lm_head k %u vs weight %d", name.c_str(), k, wt.k));
    ops_.push_back({name, [=](cudaStream_t st) {
                        return w4a8_lmhead_argmax(&wt, 0, xq, xs, act, static_cast<int32_t>(rows), logits, key, tok, ids,
                                                  workspace, workspace_bytes, st);
                    }});
    return Status::Ok();
}

// --- Plan ------------------------------------------------------------------------

Plan::~Plan() {
    if (exec_) cudaGraphExecDestroy(exec_);
    if (graph_) cudaGraphDestroy(graph_);
}

Status Plan::run(cudaStream_t st) const {
    for (const Op& op : ops_) {
        const w4a8_status s = op.run(st);
        if (s != W4A8_OK) return Status::Error(op.name + ": " + w4a8_last_error());
    }
    return Status::Ok();
}

Status Plan::capture(cudaStream_t st) {
    Status s = cuda_status("graph capture", cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    if (!s.ok()) return s;
    const Status r = run(st);
    cudaGraph_t g = nullptr;
    s = cuda_status("graph capture end", cudaStreamEndCapture(st, &g));
    if (!r.ok()) {
        if (g) cudaGraphDestroy(g);
        return r;
    }
    if (!s.ok()) return s;
    cudaGraphExec_t e = nullptr;
    s = cuda_status("graph instantiate", cudaGraphInstantiate(&e, g, 0));
    if (!s.ok()) {
        cudaGraphDestroy(g);
        return s;
    }
    if (exec_) cudaGraphExecDestroy(exec_);
    if (graph_) cudaGraphDestroy(graph_);
    graph_ = g;
    exec_ = e;
    return Status::Ok();
}

Status Plan::replay(cudaStream_t st) const {
    if (!exec_) return Status::Error("replay before capture");
    return cuda_status("graph launch", cudaGraphLaunch(exec_, st));
}

}  // namespace webyiq
