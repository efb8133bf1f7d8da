// webyiq_cli: native runner of the W4A8 path over a converted model directory
// (manifest.json + shards), the counterpart of the reference CLI's --ref / --bench
// modes (crates/cli/src/main.rs:270-350) for this path:
//
//   webyiq_cli <model_dir> --list
//       tensors of the manifest (no GPU needed)
//   webyiq_cli <model_dir> --ref <prefix>
//       <prefix>.json {"op": "model", "steps": T}: the decode step's W4A8 path over every
//       layer of the model (see reference_model below), logits and greedy tokens
//       checked as crates/cli/src/main.rs:274-318 checks a model; or
//       <prefix>.json {"op": "matmul" | "quant_gemv" | "lm_head", "weight": name, "m": M,
//                      "act": "token" | "group32", "mode": 0 | 1 | 2, "eps": e}
//       <prefix>.x.f32  activations f32 [M, K] (quantized on the GPU)
//       <prefix>.nw.f32 (quant_gemv, optional) RMSNorm weights f32 [K]
//       <prefix>.y0.f32 (mode 1 only) y before the call
//       <prefix>.y.f32  expected y f32 [M, N] (matmul, quant_gemv) or <prefix>.tok.u32 (lm_head)
//       runs quant + matmul, the fused (norm +) quant + GEMV, or the fused lm_head
//       argmax through the Builder and checks |y - ref| <= 1e-3 |ref| + 1e-3 rms(ref)
//       (tokens: exact); exit 0 / 1
//   webyiq_cli <model_dir> --bench <iters>
//       every q4 weight: GEMV (M = 1) and GEMM (M = 1024) timed with CUDA events,
//       and all GEMVs as one captured decode-step graph
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "engine.h"

using namespace webyiq;

namespace {

int fail(const Status& s) {
    fprintf(stderr, "error: %s\n", s.err.c_str());
    return 2;
}

#define CK(expr)                                                                  \
    do {                                                                          \
        cudaError_t e_ = (expr);                                                  \
        if (e_ != cudaSuccess) {                                                  \
            fprintf(stderr, "error: %s: %s\n", #expr, cudaGetErrorString(e_));    \
            return 2;                                                             \
        }                                                                         \
    } while (0)

int list(const Manifest& m) {
    printf("format %s arch %s quant %u-bit group %u (%s), %zu shards\n", m.format.c_str(), m.arch.c_str(), m.bits,
           m.group, m.scheme.c_str(), m.shards.size());
    for (const auto& kv : m.tensors) {
        std::string shape;
        for (size_t i = 0; i < kv.second.shape.size(); ++i)
            shape += (i ? "x" : "") + std::to_string(kv.second.shape[i]);
        printf("%-40s %-5s %-12s %12llu bytes (shard %zu @ %llu)\n", kv.first.c_str(), kv.second.dtype.c_str(),
               shape.c_str(), static_cast<unsigned long long>(kv.second.bytes), kv.second.shard,
               static_cast<unsigned long long>(kv.second.offset));
    }
    return 0;
}

template <typename T>
bool read_array(const std::string& path, std::vector<T>& out, size_t count) {
    std::vector<uint8_t> raw;
    if (!read_file(path, raw) || raw.size() != count * sizeof(T)) return false;
    out.resize(count);
    memcpy(out.data(), raw.data(), raw.size());
    return true;
}

// --ref op "model": the W4A8 part of a decode step over every layer of a converted
// Llama-style model, run through the Builder and one captured graph per token, and
// compared as the reference CLI compares a model (crates/cli/src/main.rs:274-318):
// last-position logits (cosine, max |diff|, top 10) and the greedy tokens.
// Per layer l (graph.rs:300-311, mlp): x += down(quant(silu(g) * u)), (g, u) =
// gate_up(norm_quant(x, l{l}.ffn_norm)), as two fused launches (norm + quant +
// SWIGLU GEMV, quant + residual GEMV); then head_ops (graph.rs:476-486): norm_quant(x,
// norm), the lm_head GEMV (lm_head, or the tied embed) with the argmax fused.  The
// attention / DeltaNet blocks are not part of this path and are not run.
//   <prefix>.x.f32       hidden states f32 [steps, hidden] (one decode step each)
//   <prefix>.logits.f32  expected logits of the last step f32 [vocab]
//   <prefix>.tok.u32     expected greedy token of every step u32 [steps]
int reference_model(Engine& e, const std::string& prefix, const Json& j) {
    const Json& c = e.manifest().config;
    const uint32_t layers = static_cast<uint32_t>(c["num_layers"].num);
    const uint32_t hd = static_cast<uint32_t>(c["hidden_size"].num);
    const uint32_t ffn = static_cast<uint32_t>(c["intermediate_size"].num);
    const uint32_t vocab = static_cast<uint32_t>(c["vocab_size"].num);
    const double eps = c.has("rms_norm_eps") ? c["rms_norm_eps"].num : 1e-6;
    const uint32_t steps = j.has("steps") ? static_cast<uint32_t>(j["steps"].num) : 1;
    if (!layers || !hd || !ffn || !vocab || !steps) return fail(Status::Error("model: config needs num_layers, hidden_size, intermediate_size, vocab_size"));
    const std::string head = e.manifest().tensors.count("lm_head.q") ? "lm_head" : "embed";
    const DeviceBuffer* norm = e.buffer("norm");
    if (!norm) return fail(Status::Error("missing tensor norm"));
    std::vector<float> x, want;
    std::vector<uint32_t> want_tok;
    if (!read_array(prefix + ".x.f32", x, static_cast<size_t>(steps) * hd))
        return fail(Status::Error("bad " + prefix + ".x.f32 (want f32 [steps, hidden])"));
    if (!read_array(prefix + ".logits.f32", want, vocab)) return fail(Status::Error("bad " + prefix + ".logits.f32"));
    if (!read_array(prefix + ".tok.u32", want_tok, steps)) return fail(Status::Error("bad " + prefix + ".tok.u32"));

    float *dx = nullptr, *dh = nullptr, *dlog = nullptr, *dxs = nullptr;
    int8_t* dxq = nullptr;
    uint64_t* dkey = nullptr;
    uint32_t* dtok = nullptr;
    void* ws = nullptr;
    const size_t wsb = w4a8_lmhead_workspace_bytes(static_cast<int32_t>(vocab), 1);
    CK(cudaMalloc(&dx, static_cast<size_t>(hd) * 4));
    CK(cudaMalloc(&dh, static_cast<size_t>(ffn) * 4));
    CK(cudaMalloc(&dlog, static_cast<size_t>(vocab) * 4));
    CK(cudaMalloc(&dxq, hd));
    CK(cudaMalloc(&dxs, static_cast<size_t>(hd / 32) * 8));
    CK(cudaMalloc(&dkey, 8));
    CK(cudaMalloc(&dtok, 4));
    CK(cudaMalloc(&ws, wsb));
    CK(cudaMemset(ws, 0, wsb));
    Builder b(e);
    Status s;
    for (uint32_t l = 0; l < layers && s.ok(); ++l) {
        const std::string p = "l" + std::to_string(l) + ".";
        const DeviceBuffer* fn = e.buffer(p + "ffn_norm");
        if (!fn) return fail(Status::Error("missing tensor " + p + "ffn_norm"));
        s = b.quant_gemv("gate_up", p + "gate_up", hd, 2 * ffn, W4A8_SWIGLU, 1, dx, static_cast<const float*>(fn->ptr), eps, dh);
        if (s.ok()) s = b.quant_gemv("down", p + "down", ffn, hd, W4A8_ADD, 1, dh, nullptr, eps, dx);
    }
    if (s.ok()) s = b.quant("norm_quant", hd, eps, dx, static_cast<const float*>(norm->ptr), 1, W4A8_ACT_TOKEN, dxq, dxs);
    if (s.ok()) s = b.lm_head("lm_head", head, hd, 1, dxq, dxs, W4A8_ACT_TOKEN, dlog, dkey, dtok, nullptr, ws, wsb);
    if (!s.ok()) return fail(s);
    cudaStream_t st;
    CK(cudaStreamCreate(&st));
    Plan plan(b.take());
    // one eager step sets the kernels' per-device attributes; the steps then replay the graph
    CK(cudaMemcpyAsync(dx, x.data(), static_cast<size_t>(hd) * 4, cudaMemcpyHostToDevice, st));
    s = plan.run(st);
    if (s.ok()) s = plan.capture(st);
    if (!s.ok()) return fail(s);
    std::vector<uint32_t> got_tok(steps);
    std::vector<float> got(vocab);
    for (uint32_t t = 0; t < steps; ++t) {
        CK(cudaMemcpyAsync(dx, x.data() + static_cast<size_t>(t) * hd, static_cast<size_t>(hd) * 4, cudaMemcpyHostToDevice, st));
        s = plan.replay(st);
        if (!s.ok()) return fail(s);
        CK(cudaMemcpyAsync(&got_tok[t], dtok, 4, cudaMemcpyDeviceToHost, st));
    }
    CK(cudaMemcpyAsync(got.data(), dlog, static_cast<size_t>(vocab) * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    uint32_t code = 0;
    if (w4a8_device_error(&code, st) != W4A8_OK) return fail(Status::Error("device error word set: a bounded wait gave up"));
    double dot = 0, na = 0, nb = 0, maxd = 0;
    for (uint32_t i = 0; i < vocab; ++i) {
        dot += static_cast<double>(got[i]) * want[i];
        na += static_cast<double>(got[i]) * got[i];
        nb += static_cast<double>(want[i]) * want[i];
        maxd = std::fmax(maxd, std::fabs(static_cast<double>(got[i]) - want[i]));
    }
    auto top = [&](const std::vector<float>& l) {
        std::vector<uint32_t> idx(l.size());
        for (uint32_t i = 0; i < l.size(); ++i) idx[i] = i;
        std::partial_sort(idx.begin(), idx.begin() + std::min<size_t>(10, idx.size()), idx.end(),
                          [&](uint32_t a, uint32_t bb) { return l[a] > l[bb] || (l[a] == l[bb] && a < bb); });
        idx.resize(std::min<size_t>(10, idx.size()));
        return idx;
    };
    const auto te = top(got), tr = top(want);
    int shared = 0;
    for (uint32_t a : te) shared += std::count(tr.begin(), tr.end(), a) ? 1 : 0;
    const double cosine = dot / (std::sqrt(na) * std::sqrt(nb) + 1e-30);
    printf("last-position logits: cosine %.6f, max |diff| %.3e, top-10 overlap %d/10\n", cosine, maxd, shared);
    printf("  top10 engine:");
    for (uint32_t a : te) printf(" %u", a);
    printf("\n  top10 ref   :");
    for (uint32_t a : tr) printf(" %u", a);
    printf("\n");
    uint32_t matched = 0;
    while (matched < steps && got_tok[matched] == want_tok[matched]) ++matched;
    printf("greedy: %u/%u tokens match reference (%u layers, hidden %u, ffn %u, vocab %u, %zu launches a step)\n",
           matched, steps, layers, hd, ffn, vocab, plan.size());
    printf("  engine:");
    for (uint32_t t = 0; t < steps; ++t) printf(" %u", got_tok[t]);
    printf("\n  ref   :");
    for (uint32_t t = 0; t < steps; ++t) printf(" %u", want_tok[t]);
    printf("\n");
    cudaFree(dx);
    cudaFree(dh);
    cudaFree(dlog);
    cudaFree(dxq);
    cudaFree(dxs);
    cudaFree(dkey);
    cudaFree(dtok);
    cudaFree(ws);
    cudaStreamDestroy(st);
    return (matched == steps && cosine >= 0.9999 && shared >= 9) ? 0 : 1;
}

int reference(Engine& e, const std::string& prefix) {
    std::vector<uint8_t> raw;
    if (!read_file(prefix + ".json", raw)) return fail(Status::Error("cannot read " + prefix + ".json"));
    Json j;
    std::string err;
    if (!parse_json(std::string(raw.begin(), raw.end()), j, err)) return fail(Status::Error(prefix + ".json: " + err));
    const std::string op = j.has("op") ? j["op"].str : "matmul";
    if (op == "model") return reference_model(e, prefix, j);
    const std::string wname = j["weight"].str;
    const uint32_t m = static_cast<uint32_t>(j["m"].num);
    const int act = j["act"].str == "group32" ? W4A8_ACT_GROUP32 : W4A8_ACT_TOKEN;
    const uint32_t mode = static_cast<uint32_t>(j["mode"].num);
    const double eps = j.has("eps") ? j["eps"].num : 1e-6;
    w4a8_weight w;
    Status s = e.weight(wname, w);
    if (!s.ok()) return fail(s);
    const uint32_t k = static_cast<uint32_t>(w.k), rows = static_cast<uint32_t>(w.n);
    const uint32_t n = mode == W4A8_SWIGLU ? rows / 2 : rows;
    std::vector<float> x;
    if (!read_array(prefix + ".x.f32", x, static_cast<size_t>(m) * k))
        return fail(Status::Error("bad " + prefix + ".x.f32 (want f32 [m, k])"));

    float *dx = nullptr, *dxs = nullptr, *dy = nullptr;
    int8_t* dxq = nullptr;
    CK(cudaMalloc(&dx, x.size() * 4));
    CK(cudaMalloc(&dxq, x.size()));
    CK(cudaMalloc(&dxs, static_cast<size_t>(m) * (k / 32) * 8));
    CK(cudaMalloc(&dy, static_cast<size_t>(m) * rows * 4));
    CK(cudaMemcpy(dx, x.data(), x.size() * 4, cudaMemcpyHostToDevice));
    cudaStream_t st;
    CK(cudaStreamCreate(&st));
    Builder b(e);
    float* dnw = nullptr;
    if (op == "quant_gemv") {
        // optional RMSNorm weights <prefix>.nw.f32 (f32 [k])
        std::vector<float> nw;
        if (read_array(prefix + ".nw.f32", nw, k)) {
            CK(cudaMalloc(&dnw, static_cast<size_t>(k) * 4));
            CK(cudaMemcpy(dnw, nw.data(), static_cast<size_t>(k) * 4, cudaMemcpyHostToDevice));
        }
    } else {
        s = b.quant("quant", k, eps, dx, nullptr, m, act, dxq, dxs);
        if (!s.ok()) return fail(s);
    }
    int rc = 0;
    if (op == "lm_head") {
        uint64_t* dkey = nullptr;
        uint32_t* dtok = nullptr;
        void* ws = nullptr;
        const size_t wsb = w4a8_lmhead_workspace_bytes(w.n, static_cast<int32_t>(m));
        CK(cudaMalloc(&dkey, m * 8));
        CK(cudaMalloc(&dtok, m * 4));
        CK(cudaMalloc(&ws, wsb));
        CK(cudaMemset(ws, 0, wsb));
        s = b.lm_head("lm_head", wname, k, m, dxq, dxs, act, dy, dkey, dtok, nullptr, ws, wsb);
        if (!s.ok()) return fail(s);
        Plan p(b.take());
        s = p.run(st);
        if (!s.ok()) return fail(s);
        CK(cudaStreamSynchronize(st));
        std::vector<uint32_t> tok(m), want;
        CK(cudaMemcpy(tok.data(), dtok, m * 4, cudaMemcpyDeviceToHost));
        if (!read_array(prefix + ".tok.u32", want, m)) return fail(Status::Error("bad " + prefix + ".tok.u32"));
        int match = 0;
        for (uint32_t t = 0; t < m; ++t) match += tok[t] == want[t];
        printf("lm_head %s: %d/%u greedy tokens match the reference\n", wname.c_str(), match, m);
        rc = match == static_cast<int>(m) ? 0 : 1;
        cudaFree(dkey);
        cudaFree(dtok);
        cudaFree(ws);
    } else {
        std::vector<float> want, y0;
        if (!read_array(prefix + ".y.f32", want, static_cast<size_t>(m) * n))
            return fail(Status::Error("bad " + prefix + ".y.f32 (want f32 [m, n])"));
        if (mode == W4A8_ADD) {
            if (!read_array(prefix + ".y0.f32", y0, static_cast<size_t>(m) * n))
                return fail(Status::Error("bad " + prefix + ".y0.f32"));
            CK(cudaMemcpy(dy, y0.data(), y0.size() * 4, cudaMemcpyHostToDevice));
        }
        const Path path = m == 1 ? Path::Decode : m <= W4A8_GEMV_MAX_M ? Path::Verify : Path::Prefill;
        if (op == "quant_gemv")
            s = b.quant_gemv("quant_gemv", wname, k, rows, mode, m, dx, dnw, eps, dy);
        else
            s = b.matmul(path, m, "matmul", wname, k, rows, mode, dxq, dxs, act, dy);
        if (!s.ok()) return fail(s);
        Plan p(b.take());
        s = p.run(st);
        if (!s.ok()) return fail(s);
        CK(cudaStreamSynchronize(st));
        std::vector<float> y(static_cast<size_t>(m) * n);
        CK(cudaMemcpy(y.data(), dy, y.size() * 4, cudaMemcpyDeviceToHost));
        double maxd = 0, maxr = 0, ss = 0, dot = 0, na = 0, nb = 0;
        for (size_t i = 0; i < y.size(); ++i) {
            maxd = std::fmax(maxd, std::fabs(static_cast<double>(y[i]) - want[i]));
            maxr = std::fmax(maxr, std::fabs(static_cast<double>(want[i])));
            ss += static_cast<double>(want[i]) * want[i];
            dot += static_cast<double>(y[i]) * want[i];
            na += static_cast<double>(y[i]) * y[i];
            nb += static_cast<double>(want[i]) * want[i];
        }
        const double rms = std::sqrt(ss / static_cast<double>(y.size() ? y.size() : 1));
        size_t bad = 0;
        for (size_t i = 0; i < y.size(); ++i)
            bad += std::fabs(static_cast<double>(y[i]) - want[i]) > 1e-3 * std::fabs(static_cast<double>(want[i])) + 1e-3 * rms;
        const double rel = maxr > 0 ? maxd / maxr : maxd;
        printf("%s %s m=%u (%s): max |diff| / max |ref| = %.3e, cosine %.8f, %zu of %zu outside 1e-3\n",
               op.c_str(), wname.c_str(), m,
               op == "quant_gemv" ? (dnw ? "norm + quant + gemv, one launch" : "quant + gemv, one launch")
                                  : path == Path::Prefill ? "gemm" : "gemv",
               rel, dot / (std::sqrt(na * nb) + 1e-30), bad, y.size());
        rc = (rel <= 1e-3 && bad == 0) ? 0 : 1;
    }
    cudaFree(dx);
    cudaFree(dxq);
    cudaFree(dxs);
    cudaFree(dy);
    if (dnw) cudaFree(dnw);
    cudaStreamDestroy(st);
    return rc;
}

int bench(Engine& e, int iters) {
    std::vector<std::string> names;
    for (const auto& kv : e.manifest().tensors) {
        const std::string& nm = kv.first;
        if (nm.size() > 2 && nm.compare(nm.size() - 2, 2, ".q") == 0) names.push_back(nm.substr(0, nm.size() - 2));
    }
    if (names.empty()) return fail(Status::Error("no q4 weights in the manifest"));
    uint32_t kmax = 0;
    for (const auto& nm : names) {
        w4a8_weight w;
        Status s = e.weight(nm, w);
        if (!s.ok()) return fail(s);
        kmax = std::max<uint32_t>(kmax, static_cast<uint32_t>(w.k));
    }
    const uint32_t mmax = 1024;
    float *dx = nullptr, *dxs = nullptr, *dy = nullptr;
    int8_t* dxq = nullptr;
    size_t ymax = 0;
    for (const auto& nm : names) {
        w4a8_weight w;
        e.weight(nm, w);
        ymax = std::max(ymax, static_cast<size_t>(w.n) * mmax);
    }
    CK(cudaMalloc(&dx, static_cast<size_t>(mmax) * kmax * 4));
    CK(cudaMalloc(&dxq, static_cast<size_t>(mmax) * kmax));
    CK(cudaMalloc(&dxs, static_cast<size_t>(mmax) * (kmax / 32) * 8));
    CK(cudaMalloc(&dy, ymax * 4));
    std::vector<float> hx(static_cast<size_t>(mmax) * kmax);
    uint32_t r = 12345;
    for (float& v : hx) {
        r = r * 1664525u + 1013904223u;
        v = (static_cast<float>(r >> 8) / 16777216.0f - 0.5f) * 3.4f;
    }
    CK(cudaMemcpy(dx, hx.data(), hx.size() * 4, cudaMemcpyHostToDevice));
    cudaStream_t st;
    CK(cudaStreamCreate(&st));
    cudaEvent_t a, b2;
    CK(cudaEventCreate(&a));
    CK(cudaEventCreate(&b2));
    const int act = e.manifest().group == 32 ? W4A8_ACT_GROUP32 : W4A8_ACT_TOKEN;
    double step_bytes = 0;
    Builder step(e);
    for (const auto& nm : names) {
        w4a8_weight w;
        e.weight(nm, w);
        const uint32_t k = w.k, n = w.n;
        const double wbytes = static_cast<double>(n) * k / 2 + static_cast<double>(n) * (k / w.group) * (w.has_min ? 4 : 2);
        for (uint32_t m : {1u, mmax}) {
            if (m > 1 && (n % 32 || k % 128)) continue;
            Builder bq(e);
            Status s = bq.quant("quant", k, 1e-6, dx, nullptr, m, act, dxq, dxs);
            if (!s.ok()) return fail(s);
            Plan pq(bq.take());
            s = pq.run(st);
            if (!s.ok()) return fail(s);
            Builder bm(e);
            s = bm.matmul(m == 1 ? Path::Decode : Path::Prefill, m, nm, nm, k, n, W4A8_STORE, dxq, dxs, act, dy);
            if (!s.ok()) return fail(s);
            Plan p(bm.take());
            s = p.capture(st);
            if (!s.ok()) return fail(s);
            for (int i = 0; i < 3; ++i) p.replay(st);
            CK(cudaEventRecord(a, st));
            for (int i = 0; i < iters; ++i) p.replay(st);
            CK(cudaEventRecord(b2, st));
            CK(cudaEventSynchronize(b2));
            float ms = 0;
            CK(cudaEventElapsedTime(&ms, a, b2));
            const double us = ms * 1e3 / iters;
            if (m == 1)
                printf("%-36s gemv  %6ux%-6u %9.2f us  %8.1f GB/s\n", nm.c_str(), n, k, us,
                       (wbytes + k + 4.0 * n) / (us * 1e-6) / 1e9);
            else
                printf("%-36s gemm  %6ux%-6u m=%u %9.2f us  %8.1f TOPS\n", nm.c_str(), n, k, m, us,
                       2.0 * m * n * k / (us * 1e-6) / 1e12);
        }
        step_bytes += wbytes;
        Status s = step.gemv(nm, nm, k, n, W4A8_STORE, 1, dxq, dxs, act, dy);
        if (!s.ok()) return fail(s);
    }
    Plan ps(step.take());
    Status s = ps.capture(st);
    if (!s.ok()) return fail(s);
    for (int i = 0; i < 3; ++i) ps.replay(st);
    CK(cudaEventRecord(a, st));
    for (int i = 0; i < iters; ++i) ps.replay(st);
    CK(cudaEventRecord(b2, st));
    CK(cudaEventSynchronize(b2));
    float ms = 0;
    CK(cudaEventElapsedTime(&ms, a, b2));
    printf("decode step (%zu GEMVs, one graph): %.2f us, %.1f GB/s of weights\n", ps.size(), ms * 1e3 / iters,
           step_bytes / (ms * 1e-3 / iters) / 1e9);
    uint32_t code = 0;
    if (w4a8_device_error(&code, st) != W4A8_OK) return fail(Status::Error(w4a8_last_error()));
    cudaFree(dx);
    cudaFree(dxq);
    cudaFree(dxs);
    cudaFree(dy);
    cudaStreamDestroy(st);
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    std::string dir, ref;
    int bench_iters = 0, device = 0;
    bool do_list = false;
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        if (a == "--list") do_list = true;
        else if (a == "--ref" && i + 1 < argc) ref = argv[++i];
        else if (a == "--bench" && i + 1 < argc) bench_iters = atoi(argv[++i]);
        else if (a == "--device" && i + 1 < argc) device = atoi(argv[++i]);
        else if (!a.empty() && a[0] != '-') dir = a;
        else {
            fprintf(stderr, "usage: webyiq_cli <model_dir> [--list] [--ref <prefix>] [--bench <iters>] [--device N]\n");
            return 2;
        }
    }
    if (dir.empty()) {
        fprintf(stderr, "usage: webyiq_cli <model_dir> [--list] [--ref <prefix>] [--bench <iters>] [--device N]\n");
        return 2;
    }
    Manifest m;
    Status s = Manifest::load(dir, m);
    if (!s.ok()) return fail(s);
    if (do_list) return list(m);
    if (ref.empty() && bench_iters <= 0) return list(m);
    CK(cudaSetDevice(device));
    Engine e(m, dir);
    s = e.load_all();
    if (!s.ok()) return fail(s);
    int rc = 0;
    if (!ref.empty()) rc = reference(e, ref);
    if (rc == 0 && bench_iters > 0) rc = bench(e, bench_iters);
    return rc;
}
