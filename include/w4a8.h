/*
 * webyIQ W4A8 quantized-matmul hot path for NVIDIA B200 (sm_100a): the C ABI.
 *
 * This is the drop-in boundary for the operator surface of the webyIQ engine
 * (crates/engine/src/graph.rs:190-222, 476-486): the int4-weight x int8-activation
 * GEMV (decode and MTP verify), the prefill GEMM, the activation quantizer
 * (optionally fused with RMSNorm) and the greedy argmax over lm_head logits.
 *
 * Conventions
 *  - Every pointer argument except `w4a8_weight_view`'s output struct and the
 *    workspace-size queries is a DEVICE pointer owned by the caller.  Nothing is
 *    allocated, freed or copied between host and device inside these calls, and
 *    no call synchronizes the host: every launch is ordered on `stream`
 *    (a cudaStream_t passed as void*; NULL = the legacy default stream).
 *  - Errors are returned as a w4a8_status; w4a8_last_error() gives a message for
 *    the calling thread.  Shapes, modes and pointer alignment are validated on the
 *    host before any launch, so an EINVAL call launches nothing.
 *  - Calls on distinct streams are thread-safe, and one process may drive several
 *    GPUs: a call runs on the calling thread's current device, and each kernel's
 *    launch state (its raised shared-memory limit, its occupancy figure) is kept
 *    per device and set under a lock by the first call on that device.
 *
 * Weight layout (tools/convert.py:7-12, 68-75 of the reference): a quantized linear
 * weight with n output rows and k inputs is
 *   q : u32[n, k/8]   word i of a row holds weights 8i..8i+7 with
 *                      byte b = w[8i+b] | w[8i+4+b] << 4   (nibbles are unsigned 0..15)
 *   s : has_min = 1 -> u32[n, k/group]  = f16 scale | f16 min << 16,  w = q*scale + min
 *       has_min = 0 -> f16[n, k/group]  = scale,                       w = (q-8)*scale
 * has_min = 1 with group 32 is exactly what convert.py / gptq.py write.  has_min = 0
 * is the symmetric signed-int4 format (values -8..7 stored as q-8 nibbles).
 *
 * Activation layout (crates/engine/src/shaders/quant.wgsl:1-4, 41-61): xq is int8[m, k]
 * (row = token).  Its scales `xs` come in two layouts:
 *   W4A8_ACT_GROUP32 : f32[m, k/32, 2] = (dx, dx * sum(xq)) per 32 inputs (the engine's)
 *   W4A8_ACT_TOKEN   : f32[m]          = dx per token (per-row absmax)
 *
 * Numerics.  The int32 dot product of every (token, row, group) is exact.  With
 * W4A8_ACT_TOKEN the whole row sum is exact as well: every group term
 * scale*I + min*sum(xq) is an integer multiple of 2^-24 (f16 scales are), it is
 * accumulated in int64, and the output is ((float)acc * 2^-24) * dx, rounded twice
 * and independent of how the work was split.  So results are bit-identical across
 * the GEMV kernels, any grid size and any number of GPUs, and the argmax ids are
 * exact.  The tensor-core GEMM (group 128, symmetric, W4A8_ACT_TOKEN, used by
 * w4a8_gemm) keeps the int32 group dots exact but does the scale step in f32:
 * y = (sum_g f32(s) * f32(I)) * dx, within 1e-6 relative of the exact path.  The accumulator cannot overflow while k * 1905 * (|scale| + |min|) < 2^39
 * for every group (for k = 8192: |scale| + |min| < 35000).  With W4A8_ACT_GROUP32 the
 * group terms s*dx*I + m*dxsum are accumulated in f32 (as gemv_q4q8.wgsl:68 does),
 * so results agree with any other order to f32 rounding.
 */
#ifndef WEBYIQ_W4A8_H
#define WEBYIQ_W4A8_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define W4A8_API __attribute__((visibility("default")))
#else
#define W4A8_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum w4a8_status {
    W4A8_OK = 0,
    W4A8_EINVAL = 1,   /* shape, mode, alignment or pointer rejected; nothing launched */
    W4A8_ECUDA = 2,    /* a CUDA runtime call or launch failed */
    W4A8_ENCCL = 3,    /* an NCCL call failed */
    W4A8_ETIMEOUT = 4, /* a bounded device-side wait gave up */
    W4A8_ENOTSUP = 5   /* a valid request this build does not implement */
} w4a8_status;

/* activation scale layouts */
enum { W4A8_ACT_GROUP32 = 0, W4A8_ACT_TOKEN = 1 };

/* output modes: MODE of gemv_q4q8.wgsl:4 / gemm_q4q8.wgsl:3 */
enum {
    W4A8_STORE = 0,  /* y = W x */
    W4A8_ADD = 1,    /* y += W x (residual) */
    W4A8_SWIGLU = 2  /* y[j] = silu(W[j] x) * W[j + n/2] x, output width n/2 */
};

/* largest token count the GEMV takes; larger batches go to the GEMM */
#define W4A8_GEMV_MAX_M 16

typedef struct w4a8_weight {
    const void* q;   /* device u32[n, k/8] */
    const void* s;   /* device, see the header comment */
    int32_t n;       /* rows (output channels) of the stored tensor */
    int32_t k;       /* inputs */
    int32_t group;   /* 32 or 128 */
    int32_t has_min; /* 1: (scale, min) pairs; 0: symmetric, scale only */
} w4a8_weight;

/* Describe a quantized weight already in device memory (no copy, no allocation).
 * Replaces the binding of `{w}.q` / `{w}.s` in Builder::gemv / Builder::gemm
 * (graph.rs:192-204) and the q4 checks of Manifest::parse (manifest.rs:82).
 * Checks: group in {32, 128}; k % group == 0; n >= 1; q 16-byte aligned; s 4-byte
 * aligned (every tensor of a converted model is 256-byte aligned, convert.py:24). */
W4A8_API w4a8_status w4a8_weight_view(const void* q, const void* s, int32_t n, int32_t k, int32_t group,
                             int32_t has_min, w4a8_weight* out);

/* Activation quantization, optionally fused with RMSNorm (quant.wgsl:19-62,
 * Builder::quant graph.rs:216-222):
 *   v = norm_w ? x * (1/sqrt(mean(x^2) + eps)) * norm_w : x
 *   GROUP32: per 32 inputs  dx = amax/127, xq = rint(v * (1/dx)), xs = (dx, dx*sum xq)
 *   TOKEN  : per row        dx = amax/127, xq = rint(v * (1/dx)), xs = dx
 * (amax == 0 gives dx = 0 and xq = 0.)  x f32[m, k], norm_w f32[k] or NULL.
 * Needs k % 32 == 0, x and norm_w 16-byte aligned, xq 16-byte aligned. */
W4A8_API w4a8_status w4a8_quant(const float* x, const float* norm_w, float eps, int32_t m, int32_t k,
                       int32_t act, int8_t* xq, float* xs, void* stream);

/* Decode / verify GEMV, m in [1, W4A8_GEMV_MAX_M] tokens (gemv_q4q8.wgsl:36-131,
 * Builder::gemv graph.rs:190-198).  y f32[m, n] (n/2 for SWIGLU), token stride n
 * (n/2).  xq 16-byte aligned. */
W4A8_API w4a8_status w4a8_gemv(const w4a8_weight* w, const int8_t* xq, const float* xs, int32_t act,
                      int32_t m, int32_t mode, float* y, void* stream);

/* Per-token quantization and GEMV in one launch, for group-128 weights: the
 * quant of a projection's input followed by the projection (Builder::quant then
 * Builder::gemv, graph.rs:216-222 and 190-198; quant.wgsl with one scale per token,
 * no norm, then gemv_q4q8.wgsl).  x f32[m, k] (16-byte aligned), m in
 * [1, W4A8_GEMV_MAX_M]; y as w4a8_gemv.  The result is bit-identical to
 * w4a8_quant(act = W4A8_ACT_TOKEN, norm_w = NULL) followed by w4a8_gemv.
 * W4A8_ENOTSUP for other groups. */
W4A8_API w4a8_status w4a8_gemv_x(const w4a8_weight* w, const float* x, int32_t m, int32_t mode, float* y,
                                 void* stream);

/* The norm_quant prologue of a decode block fused as well: RMSNorm with weights
 * norm_w f32[k] and eps, per-token quantization and the GEMV in one launch
 * (graph.rs:266,323 norm_quant then Builder::gemv; quant.wgsl:19-62 with NORM).
 * Bit-identical to w4a8_quant(x, norm_w, eps, m, k, W4A8_ACT_TOKEN) followed by
 * w4a8_gemv.  Group-128 weights, m in [1, 2] tokens (the decode and MTP-verify
 * widths); W4A8_ENOTSUP for other calls. */
W4A8_API w4a8_status w4a8_gemv_xn(const w4a8_weight* w, const float* x, const float* norm_w, float eps, int32_t m,
                                 int32_t mode, float* y, void* stream);

/* Prefill GEMM Y[m, n] = X W^T for any m >= 1 (gemm_q4q8.wgsl:46-121,
 * Builder::gemm graph.rs:200-205).  Group-128 symmetric weights with
 * W4A8_ACT_TOKEN run on the tcgen05 tensor cores (int4 expanded to int8 in shared
 * memory, int32 accumulators in tensor memory); other formats run the GEMV kernels
 * over blocks of W4A8_GEMV_MAX_M tokens. */
W4A8_API w4a8_status w4a8_gemm(const w4a8_weight* w, const int8_t* xq, const float* xs, int32_t act,
                      int32_t m, int32_t mode, float* y, void* stream);

/* Builder::matmul (graph.rs:207-214): the GEMV for m <= W4A8_GEMV_MAX_M, the GEMM
 * above that. */
W4A8_API w4a8_status w4a8_matmul(const w4a8_weight* w, const int8_t* xq, const float* xs, int32_t act,
                        int32_t m, int32_t mode, float* y, void* stream);

/* Greedy sampling over f32 logits[m, v] (argmax.wgsl:14-43): tok_out[r] is the lowest
 * index among the maxima of row r, over values > -3e38 (NaN never wins; a row with
 * no such value gives 0).  ids (u32[v]) or NULL: with ids, tok_out[r] = ids[index]. */
W4A8_API w4a8_status w4a8_argmax(const float* logits, int32_t m, int32_t v, const uint32_t* ids,
                        uint32_t* tok_out, void* stream);

/* lm_head GEMV with fused argmax (head_ops, graph.rs:476-486, fused): for each token
 * r, best_key[r] = the packed key of the argmax over this weight's rows, with global
 * row ids row_offset + j (row_offset = this shard's first vocabulary row when the
 * vocabulary is split across GPUs).  Keys compare as unsigned integers, so the max
 * of the shard keys is the key of the global argmax: see w4a8_key_index.
 * logits (f32[m, n]) may be NULL to skip writing them; tok_out (u32[m]) may be NULL;
 * ids as in w4a8_argmax (indexed by the global row id).  mode is always STORE.
 * workspace: w4a8_lmhead_workspace_bytes(n, m) bytes of device memory, zero-filled
 * before its first use; every call leaves it zero-filled again.  Calls that share a
 * workspace must not overlap on the GPU. */
W4A8_API w4a8_status w4a8_lmhead_argmax(const w4a8_weight* w, int32_t row_offset, const int8_t* xq,
                               const float* xs, int32_t act, int32_t m, float* logits,
                               uint64_t* best_key, uint32_t* tok_out, const uint32_t* ids,
                               void* workspace, size_t workspace_bytes, void* stream);
W4A8_API size_t w4a8_lmhead_workspace_bytes(int32_t n, int32_t m);

/* w4a8_lmhead_argmax without a workspace and without any device allocation, for
 * callers that cannot allocate device memory where they sample (a plugin inside an
 * engine that owns all device memory; a decode loop that must not call cudaMalloc,
 * which synchronizes the device).  The scratch (CTA-done counter and the running
 * keys of up to 16 tokens) is a 256-byte array inside this library, one per GPU,
 * held until the process exits.  m > 16 is rejected with W4A8_EINVAL.  Every call
 * on a GPU shares that array and leaves it zeroed; calls that overlap on the GPU
 * race on it.  The first call on a device looks up the array's address and
 * zero-fills it (cudaGetSymbolAddress, cudaMemset): make that first call outside
 * any stream capture.  Other arguments as w4a8_lmhead_argmax.
 * No counterpart in the reference (an addition of this library). */
W4A8_API w4a8_status w4a8_lmhead_argmax_noalloc(const w4a8_weight* w, int32_t row_offset,
                                               const int8_t* xq, const float* xs, int32_t act,
                                               int32_t m, float* logits, uint64_t* best_key,
                                               uint32_t* tok_out, const uint32_t* ids, void* stream);

/* Column-split lm_head over GPUs (head_ops, graph.rs:476-486, with the vocabulary
 * sharded): this rank's weight holds vocabulary rows [row_offset, row_offset + n);
 * the call runs w4a8_lmhead_argmax on the shard and then an in-place NCCL
 * all-reduce (max, u64) of best_key[m] over nccl_comm (an ncclComm_t of all the
 * ranks that hold shards), so every rank gets the key and token of the global
 * argmax, bit-identical to one GPU.  tok_out may be NULL; ids (u32[vocab], indexed
 * by the global row id) or NULL.  Every rank must make the same call with the same
 * m, on streams the NCCL communicator may use.  W4A8_ENCCL if NCCL cannot be
 * loaded (libnccl.so.2 is opened at run time) or fails. */
W4A8_API w4a8_status w4a8_lmhead_argmax_allreduce(const w4a8_weight* w, int32_t row_offset,
                                                 const int8_t* xq, const float* xs, int32_t act,
                                                 int32_t m, float* logits, uint64_t* best_key,
                                                 uint32_t* tok_out, const uint32_t* ids,
                                                 void* workspace, size_t workspace_bytes,
                                                 void* nccl_comm, void* stream);

/* NCCL communicator helpers for hosts that do not create one themselves: a
 * 128-byte unique id made on one rank and given to all, then one communicator per
 * rank (the calling thread's current CUDA device).  Thin wrappers over
 * ncclGetUniqueId / ncclCommInitRank / ncclCommDestroy. */
W4A8_API w4a8_status w4a8_nccl_get_unique_id(void* id_out);
W4A8_API w4a8_status w4a8_nccl_comm_init(int32_t nranks, const void* id, int32_t rank, void** comm_out);
W4A8_API w4a8_status w4a8_nccl_comm_destroy(void* comm);

/* Peer-memory key exchange for the column-split lm_head, the alternative to the
 * NCCL all-reduce above for ranks of one node (one process per GPU, GPUs that can
 * reach each other's memory over NVLink).  Each rank owns a small exchange buffer
 * in its GPU memory; every rank opens every other rank's buffer through a CUDA IPC
 * handle (W4A8_XCHG_HANDLE_BYTES bytes, passed between the processes by the host,
 * e.g. an all-gather over torch.distributed).  A call then runs the shard's
 * lm_head argmax and the exchange: the rank's keys, tagged with the call's
 * sequence number, are stored into every peer's buffer, and once every rank's keys
 * of the call are in (bounded waits) their max gives every rank the key and token
 * of the global argmax, bit-identical to one GPU, without NCCL.  Where the
 * streaming lm_head covers the shard (group 128, per-token, one or two tokens,
 * whole 8-row blocks) its last CTA runs the exchange, so a call is one kernel;
 * otherwise a small exchange kernel follows.  The vocabulary ids of the shard
 * (row_offset + row) must lie below 2^24: the tag lives in the top 8 bits of the
 * key's id half.  The key slots are double-buffered by the sequence's parity and
 * the sequence counter lives on the device, so the calls can be captured in a CUDA
 * graph; every rank must make the same number of calls with the same m
 * (<= W4A8_XCHG_MAX_TOKENS).  A wait that
 * gives up (a peer ~0.3 s late, e.g. stalled on its host) leaves this rank's own
 * keys in best_key and sets the device error word, and the call itself still
 * returns W4A8_OK: callers must check w4a8_device_error (W4A8_ETIMEOUT) after their
 * exchange calls, at the latest before they trust a token (a synchronizing check,
 * so once per step or per batch of steps).  No counterpart in the reference: this
 * is the exchange step of a column-split head, done over peer memory. */
#define W4A8_XCHG_HANDLE_BYTES 64
#define W4A8_XCHG_MAX_RANKS 8
#define W4A8_XCHG_MAX_TOKENS 16
typedef struct w4a8_xchg w4a8_xchg;
/* Allocates this rank's exchange buffer on the current device (rank in
 * [0, world), world <= W4A8_XCHG_MAX_RANKS) and writes its IPC handle. */
W4A8_API w4a8_status w4a8_xchg_create(int32_t world, int32_t rank, void* handle_out, w4a8_xchg** out);
/* Opens the peers' buffers: handles holds world handles of W4A8_XCHG_HANDLE_BYTES
 * bytes in rank order (this rank's own entry is not used). */
W4A8_API w4a8_status w4a8_xchg_open(w4a8_xchg* x, const void* handles);
W4A8_API w4a8_status w4a8_xchg_destroy(w4a8_xchg* x);
/* As w4a8_lmhead_argmax_allreduce, with the exchange over x instead of NCCL. */
W4A8_API w4a8_status w4a8_lmhead_argmax_xchg(const w4a8_weight* w, int32_t row_offset, const int8_t* xq,
                                            const float* xs, int32_t act, int32_t m, float* logits,
                                            uint64_t* best_key, uint32_t* tok_out, const uint32_t* ids,
                                            void* workspace, size_t workspace_bytes, w4a8_xchg* x,
                                            void* stream);

/* MTP speculative step, around the W4A8 path (the verify integration).
 * w4a8_gather_rows (gather_rows.wgsl:1-24, graph.rs:471-516): the one-time gather of
 * the draft lm_head, row r of (dst_q, dst_s) = row ids[r] of src's packed weights
 * and scales (dst_q u32[rows, k/8] 16-byte aligned, dst_s in src's scale format);
 * rows whose id is >= src->n are left untouched.  The draft argmax is then
 * w4a8_lmhead_argmax on w4a8_weight_view(dst_q, dst_s, rows, ...) with ids mapping
 * the index back to the vocabulary (argmax.wgsl:41). */
W4A8_API w4a8_status w4a8_gather_rows(const w4a8_weight* src, const uint32_t* ids, int32_t rows, void* dst_q,
                                     void* dst_s, void* stream);
/* w4a8_spec_accept (spec_accept.wgsl:1-38): the end of a step that ran the model on
 * tok = [x, d] (u32[2], rewritten), with greedy tokens y[2] and MTP drafts e[2]:
 * a = (d == y[0]); tok = [y[a], e[a]]; ctl = (pos + 1 + a, pos + 3 + a, 2,
 * (slot + 1 + a) % 3) from params = (pos, seq_len, m, slot) (u32[4]; may be the
 * previous step's ctl); out (u32[5] or NULL) = (1 + a, y[0], y[1], pos', slot').
 * All device pointers; one thread. */
W4A8_API w4a8_status w4a8_spec_accept(uint32_t* tok, const uint32_t* y, const uint32_t* e, const uint32_t* params,
                                     uint32_t* ctl, uint32_t* out, void* stream);

/* Decode attention over an f16 KV cache, flash-decoding (attn.wgsl:41-115, the
 * "attn" op of graph.rs:282-285): for token t of a step (at position pos + t, pos =
 * params[0] read on the device, so a captured graph replays for every position) and
 * each query head, softmax(q k^T / sqrt(D)) v over positions 0 ..= pos + t, in chunks
 * of 32 positions.  qkv f32 [m, (H + 2 KVH) D] (the q heads are its first H rows of
 * D); kc, vc f16 [KVH, maxctx, D]; query heads grouped H / KVH (<= 16) per kv head.
 * part (f32 [m, H, maxctx / 32, D + 2]) receives each chunk's (P V, max, sum).
 * chunks (1 .. maxctx / 32) chunks are dispatched; those past pos + t exit at once, so
 * dispatch enough for the largest position.  D a multiple of 32 up to 1024, maxctx a
 * multiple of 32, m in [1, W4A8_GEMV_MAX_M]; qkv, kc, vc 16-byte aligned. */
W4A8_API w4a8_status w4a8_attn_decode(const float* qkv, const void* kc, const void* vc, int32_t H, int32_t KVH,
                                      int32_t D, int32_t maxctx, const uint32_t* params, int32_t m, int32_t chunks,
                                      float* part, void* stream);
/* The merge of those chunks per query head and token (attn_combine.wgsl:31-83): the
 * head output, times sigmoid(gate) when gsrc (f32 [m, 2 (H + KVH) D], head h's gate
 * at h * 2D + D) is given, quantized per 32 into the W4A8_ACT_GROUP32 format of
 * w4a8_quant: xq int8 [m, H D], xs f32 [m, H D / 32, 2] (the o projection's input).
 * o_out (f32 [m, H, D]) or NULL receives the head outputs before quantization. */
W4A8_API w4a8_status w4a8_attn_combine(const float* part, int32_t H, int32_t KVH, int32_t D, int32_t maxctx,
                                       const uint32_t* params, int32_t m, const float* gsrc, int8_t* xq, float* xs,
                                       float* o_out, void* stream);

/* Gated DeltaNet token mixer of a hybrid decoder's linear-attention layers
 * (deltanet.wgsl:80-160, the "deltanet" op of graph.rs:301-310): per head of 128
 * key and 128 value dims, the causal depthwise conv + SiLU of q/k/v, L2-normalized q
 * and k, the gated delta rule on the head's state and the gated RMSNorm, for the m
 * tokens of a step in order.  proj f32 [m, C + nh 128 + 2 nh] (C = 384 nh: rows
 * q | k | v | z | b | a), conv_w f32 [C, 4] (16-byte aligned), conv_state f32
 * [3, C, 3] and state f32 [3, nh, 128, 128] (three slots; params[3] on the device
 * names the current one), neg_a = -exp(A_log) and dt_bias f32 [nh], gate_norm f32
 * [128]; out f32 [m, nh 128].  spec = 0 updates the current slot in place; spec = 1
 * (draft verification) writes the state after token t to slot (slot + 1 + t) % 3. */
W4A8_API w4a8_status w4a8_deltanet(const float* proj, const float* conv_w, float* conv_state, float* state, float* out,
                                   const float* neg_a, const float* dt_bias, const float* gate_norm,
                                   const uint32_t* params, int32_t nh, int32_t m, float eps, int32_t spec,
                                   void* stream);

/* Index carried by a packed argmax key (0 for the "no value > -3e38" key 0). */
static inline uint32_t w4a8_key_index(uint64_t key) {
    return key ? ~(uint32_t)(key & 0xffffffffu) : 0u;
}

/* Test hook: the exact int32 dot product of every (token, row, group),
 * dots[t, j, g] = sum over the group of q'[j, i] * xq[t, i], with q' = q (has_min)
 * or q - 8 (symmetric), computed by the GEMV's own load / unpack / dp4a path.
 * dots int32[m, n, k/group], m in [1, W4A8_GEMV_MAX_M]. */
W4A8_API w4a8_status w4a8_group_dots(const w4a8_weight* w, const int8_t* xq, int32_t m, int32_t* dots,
                            void* stream);

/* Test hook: the int32 group dots of the tensor-core GEMM (same layout and values
 * as w4a8_group_dots, any m >= 1), read back from its tensor-memory accumulators.
 * Group-128 symmetric weights only (W4A8_ENOTSUP otherwise). */
W4A8_API w4a8_status w4a8_gemm_group_dots(const w4a8_weight* w, const int8_t* xq, int32_t m,
                                          int32_t* dots, void* stream);

/* Tuning: enable (default) or disable programmatic dependent launch, which lets a
 * kernel's CTAs start (and prefetch weights) while the previous kernel in the
 * stream drains.  Process-wide. */
W4A8_API void w4a8_set_pdl(int enable);

/* Tuning / testing: route group-128 per-token GEMVs to the tensor-core kernel
 * (1, default) or to the dp4a kernel (0).  Both give bit-identical results.
 * Process-wide. */
W4A8_API void w4a8_set_gemv_kernel(int tensor_core);

/* Tuning / testing: route the GEMM formats the tcgen05 kernel covers to it (1,
 * default) or to the GEMV kernels over token blocks (0).  Process-wide. */
W4A8_API void w4a8_set_gemm_kernel(int tensor_core);

/* Device-side error word: every wait inside a kernel (for a TMA copy to land, for
 * a tensor-core step to finish) is bounded; a wait that gives up records a code here and the kernel returns
 * without touching its outputs.  This call synchronizes `stream`, returns
 * W4A8_ETIMEOUT and the code if any was recorded (and clears it), else W4A8_OK.
 * code may be NULL. */
W4A8_API w4a8_status w4a8_device_error(uint32_t* code, void* stream);

/* Test hook for the failure path above, without a GPU fault: launches one kernel
 * whose bounded wait can never complete (nothing arrives on its barrier); it gives
 * up after ~10 ms and records code 4, so the next w4a8_device_error returns
 * W4A8_ETIMEOUT with that code and the context stays usable. */
W4A8_API w4a8_status w4a8_selftest_wait_timeout(void* stream);

/* Message for the last failed call on this thread ("" if none). */
W4A8_API const char* w4a8_last_error(void);

/* Build identification string. */
W4A8_API const char* w4a8_version(void);

#ifdef __cplusplus
}
#endif

#endif /* WEBYIQ_W4A8_H */
