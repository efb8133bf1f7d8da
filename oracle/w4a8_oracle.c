/*
 * TEST INFRASTRUCTURE ONLY - the CPU checker for the W4A8 hot path.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load
 * this library, and only to check or to time the reference's algorithm; the
 * product (webyiq_b200/) never calls it and has no CPU fallback.
 *
 * A plain-C restatement of the reference's arithmetic (rtx527896828/webyIQ):
 *   weights      tools/convert.py:7-12, 68-75    nibble packing, (scale, min) pairs
 *   quant        crates/engine/src/shaders/quant.wgsl:19-62
 *   group dot    crates/engine/src/shaders/gemv_q4q8.wgsl:29-34 (gdot)
 *   GEMV / GEMM  gemv_q4q8.wgsl:50-80, 117-130; gemm_q4q8.wgsl:96, 104-119
 *   argmax       crates/engine/src/shaders/argmax.wgsl:14-43
 * Where the reference leaves an order of float operations open (a reduction
 * tree, an f32 accumulation over groups), this file follows the order the CUDA
 * kernels document, so that the quantizer and the per-token GEMV are compared
 * bit for bit:
 *   - RMSNorm sum of squares: 256 partial sums, partial t = fma(x_i, x_i, .) over
 *     i = 4t + 1024j (+0..3) in order; butterfly within each 32-lane warp
 *     (xor 16, 8, 4, 2, 1); warp totals added in warp order.
 *   - per-token GEMV (W4A8_ACT_TOKEN): exact int64 sum of f16-fixed-point terms,
 *     then ((float)acc * 2^-24) * dx.
 * The per-group-32 GEMV accumulates in f32 over groups in order, like one thread
 * of gemv_q4q8.wgsl; the GPU sums the same terms in another order, so that path is
 * compared with a tolerance.
 *
 * Build: cc -O2 -ffp-contract=off -shared -fPIC -pthread (see oracle/Makefile).
 * Rows are spread over threads (orc_set_threads); each output is computed by one
 * thread start to finish, so the thread count never changes a result.
 * No FMA contraction: every fused multiply-add here is an explicit fmaf().
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* parallel for over [0, n) with up to g_threads pthreads */
static int g_threads = 1;
void orc_set_threads(int n) { g_threads = n < 1 ? 1 : (n > 256 ? 256 : n); }

typedef void (*range_fn)(void* ctx, int lo, int hi);
typedef struct {
    range_fn fn;
    void* ctx;
    int lo, hi;
} range_job;

static void* run_range(void* p) {
    range_job* j = (range_job*)p;
    j->fn(j->ctx, j->lo, j->hi);
    return NULL;
}

static void parallel_for(int n, range_fn fn, void* ctx) {
    int nt = g_threads < n ? g_threads : n;
    if (nt <= 1) {
        fn(ctx, 0, n);
        return;
    }
    pthread_t th[256];
    range_job jobs[256];
    for (int i = 0; i < nt; ++i) {
        jobs[i].fn = fn;
        jobs[i].ctx = ctx;
        jobs[i].lo = (int)((long long)n * i / nt);
        jobs[i].hi = (int)((long long)n * (i + 1) / nt);
    }
    int joined[256] = {0};
    for (int i = 1; i < nt; ++i) {
        if (pthread_create(&th[i], NULL, run_range, &jobs[i]) == 0)
            joined[i] = 1;
        else
            run_range(&jobs[i]); /* no thread: run it here */
    }
    run_range(&jobs[0]);
    for (int i = 1; i < nt; ++i)
        if (joined[i]) pthread_join(th[i], NULL);
}

#define ACT_GROUP32 0
#define ACT_TOKEN 1

/* weight j (0..k-1) of a packed row: word j/8, byte (j%8)%4, high nibble if j%8 >= 4 */
static inline int nibble(const uint32_t* row, int j) {
    const uint32_t word = row[j >> 3];
    const int b = j & 7;
    const int shift = 8 * (b & 3) + ((b >= 4) ? 4 : 0);
    return (int)((word >> shift) & 15u);
}

static inline uint32_t scale_bits(const void* s, int has_min, size_t idx) {
    return has_min ? ((const uint32_t*)s)[idx] : (uint32_t)((const uint16_t*)s)[idx];
}

static float f16_to_f32(uint32_t h) {
    const int e = (h >> 10) & 31, f = h & 1023;
    float v;
    if (e == 0)
        v = ldexpf((float)f, -24);
    else if (e == 31)
        v = f ? NAN : INFINITY;
    else
        v = ldexpf((float)(f | 1024), e - 25);
    return (h & 0x8000u) ? -v : v;
}

/* exact fixed point: h == mant * 2^sh * 2^-24 */
static inline void fix16(uint32_t h, int* mant, int* sh) {
    const int e = (h >> 10) & 31, f = h & 1023;
    int m = e ? (f | 1024) : f;
    if (h & 0x8000u) m = -m;
    *mant = m;
    *sh = e ? e - 1 : 0;
}

static inline int64_t shl64(int64_t p, int sh) { return (int64_t)((uint64_t)p << sh); }

/* ------------------------------------------------------------------------ */
void orc_unpack(const uint32_t* q, int n, int k, uint8_t* out) {
    for (int r = 0; r < n; ++r)
        for (int j = 0; j < k; ++j) out[(size_t)r * k + j] = (uint8_t)nibble(q + (size_t)r * (k / 8), j);
}

/* quant.wgsl:19-62 with the documented reduction order */
void orc_quant(const float* x, const float* nw, float eps, int m, int k, int act, int8_t* xq, float* xs) {
    for (int row = 0; row < m; ++row) {
        const float* xr = x + (size_t)row * k;
        float scale = 1.0f;
        if (nw) {
            float part[256];
            for (int t = 0; t < 256; ++t) {
                float ss = 0.0f;
                for (int i = 4 * t; i < k; i += 1024)
                    for (int c = 0; c < 4; ++c) ss = fmaf(xr[i + c], xr[i + c], ss);
                part[t] = ss;
            }
            float tot = 0.0f;
            for (int w = 0; w < 8; ++w) {
                float v[32];
                memcpy(v, part + 32 * w, sizeof(v));
                for (int off = 16; off > 0; off >>= 1) {
                    float nv[32];
                    for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ off];
                    memcpy(v, nv, sizeof(v));
                }
                tot = tot + v[0];
            }
            scale = 1.0f / sqrtf(tot / (float)k + eps);
        }
        float dx_tok = 0.0f, inv_tok = 0.0f;
        if (act == ACT_TOKEN) {
            float amax = 0.0f;
            for (int i = 0; i < k; ++i) {
                float e = xr[i];
                if (nw) e = (e * scale) * nw[i];
                amax = fmaxf(amax, fabsf(e));
            }
            dx_tok = amax / 127.0f;
            inv_tok = amax > 0.0f ? 1.0f / dx_tok : 0.0f;
            xs[row] = dx_tok;
        }
        for (int g = 0; g < k / 32; ++g) {
            float e[32];
            float amax = 0.0f;
            for (int i = 0; i < 32; ++i) {
                e[i] = xr[32 * g + i];
                if (nw) e[i] = (e[i] * scale) * nw[32 * g + i];
                amax = fmaxf(amax, fabsf(e[i]));
            }
            float dx = dx_tok, inv = inv_tok;
            if (act == ACT_GROUP32) {
                dx = amax / 127.0f;
                inv = amax > 0.0f ? 1.0f / dx : 0.0f;
            }
            int sum = 0;
            for (int i = 0; i < 32; ++i) {
                const int q = (int)rintf(e[i] * inv);
                sum += q;
                xq[(size_t)row * k + 32 * g + i] = (int8_t)q;
            }
            if (act == ACT_GROUP32) {
                xs[((size_t)row * (k / 32) + g) * 2] = dx;
                xs[((size_t)row * (k / 32) + g) * 2 + 1] = dx * (float)sum;
            }
        }
    }
}

/* exact int32 dot of every (token, row, group); q' = q (has_min) or q - 8 */
typedef struct {
    const uint32_t* q;
    int n, k, group, has_min, m;
    const int8_t* xq;
    int32_t* dots;
} dots_ctx;

static void dots_rows(void* p, int lo, int hi) {
    const dots_ctx* c = (const dots_ctx*)p;
    const uint32_t* q = c->q;
    const int n = c->n, k = c->k, group = c->group, has_min = c->has_min, m = c->m;
    const int8_t* xq = c->xq;
    int32_t* dots = c->dots;
    const int kg = k / group;
    for (int r = lo; r < hi; ++r) {
        const uint32_t* row = q + (size_t)r * (k / 8);
        for (int t = 0; t < m; ++t)
            for (int g = 0; g < kg; ++g) {
                int32_t d = 0;
                for (int i = g * group; i < (g + 1) * group; ++i)
                    d += (nibble(row, i) - (has_min ? 0 : 8)) * (int32_t)xq[(size_t)t * k + i];
                dots[((size_t)t * n + r) * kg + g] = d;
            }
    }
}

void orc_group_dots(const uint32_t* q, int n, int k, int group, int has_min, const int8_t* xq, int m,
                    int32_t* dots) {
    dots_ctx c = {q, n, k, group, has_min, m, xq, dots};
    parallel_for(n, dots_rows, &c);
}

/* One output value (before the mode epilogue) of weight row r for token t. */
static float row_value(const uint32_t* q, const void* s, int k, int group, int has_min, const int8_t* xq,
                       const float* xs, int act, int r, int t) {
    const uint32_t* row = q + (size_t)r * (k / 8);
    const int8_t* xt = xq + (size_t)t * k;
    const int kg = k / group;
    if (act == ACT_TOKEN) {
        int64_t acc = 0;
        for (int g = 0; g < kg; ++g) {
            int32_t I = 0, X = 0;
            for (int i = g * group; i < (g + 1) * group; ++i) {
                I += nibble(row, i) * (int32_t)xt[i];
                X += xt[i];
            }
            const uint32_t sb = scale_bits(s, has_min, (size_t)r * kg + g);
            int ms, ss, mm, sm;
            fix16(sb & 0xffffu, &ms, &ss);
            if (has_min) {
                fix16(sb >> 16, &mm, &sm);
                acc += shl64((int64_t)ms * I, ss) + shl64((int64_t)mm * X, sm);
            } else {
                acc += shl64((int64_t)ms * (I - 8 * X), ss);
            }
        }
        float v = (float)acc;
        v = v * 5.9604644775390625e-08f;
        return v * xs[t];
    }
    /* per group of 32 activations, f32, groups in order (gemv_q4q8.wgsl:68) */
    float acc = 0.0f;
    for (int c = 0; c < k / 32; ++c) {
        int32_t I = 0, X = 0;
        for (int i = 32 * c; i < 32 * c + 32; ++i) {
            I += nibble(row, i) * (int32_t)xt[i];
            X += xt[i];
        }
        const uint32_t sb = scale_bits(s, has_min, (size_t)r * kg + (32 * c) / group);
        const float dx = xs[((size_t)t * (k / 32) + c) * 2], dxs = xs[((size_t)t * (k / 32) + c) * 2 + 1];
        const float sc = f16_to_f32(sb & 0xffffu);
        if (has_min)
            acc += sc * dx * (float)I + f16_to_f32(sb >> 16) * dxs;
        else
            acc += sc * dx * (float)(I - 8 * X);
    }
    return acc;
}

typedef struct {
    const uint32_t* q;
    const void* s;
    int n, k, group, has_min;
    const int8_t* xq;
    const float* xs;
    int act, m, mode;
    float* y;
} gemv_ctx;

static void gemv_rows(void* p, int lo, int hi) {
    const gemv_ctx* c = (const gemv_ctx*)p;
    const uint32_t* q = c->q;
    const void* s = c->s;
    const int n = c->n, k = c->k, group = c->group, has_min = c->has_min, act = c->act, m = c->m, mode = c->mode;
    const int8_t* xq = c->xq;
    const float* xs = c->xs;
    float* y = c->y;
    const int n_out = mode == 2 ? n / 2 : n;
    for (int j = lo; j < hi; ++j)
        for (int t = 0; t < m; ++t) {
            const float a = row_value(q, s, k, group, has_min, xq, xs, act, j, t);
            float* yp = y + (size_t)t * n_out + j;
            if (mode == 0) {
                *yp = a;
            } else if (mode == 1) {
                *yp = *yp + a;
            } else {
                const float u = row_value(q, s, k, group, has_min, xq, xs, act, j + n_out, t);
                *yp = a / (1.0f + expf(-a)) * u;
            }
        }
}

/* y[t, j] for j < n_out (n_out = n, or n/2 for SWIGLU) */
void orc_gemv(const uint32_t* q, const void* s, int n, int k, int group, int has_min, const int8_t* xq,
              const float* xs, int act, int m, int mode, float* y) {
    gemv_ctx c = {q, s, n, k, group, has_min, xq, xs, act, m, mode, y};
    parallel_for(mode == 2 ? n / 2 : n, gemv_rows, &c);
}

/* argmax.wgsl:14-43: 256 strided strict-greater scans from -3e38, then a tree that
 * keeps the larger value and, on equal values, the lower index. */
void orc_argmax(const float* logits, int m, int v, const uint32_t* ids, uint32_t* out) {
    for (int row = 0; row < m; ++row) {
        const float* lr = logits + (size_t)row * v;
        float bv[256];
        uint32_t bi[256];
        for (int lid = 0; lid < 256; ++lid) {
            float best = -3.0e38f;
            uint32_t idx = 0;
            for (int i = lid; i < v; i += 256)
                if (lr[i] > best) {
                    best = lr[i];
                    idx = (uint32_t)i;
                }
            bv[lid] = best;
            bi[lid] = idx;
        }
        for (int s = 128; s > 0; s >>= 1)
            for (int lid = 0; lid < s; ++lid) {
                const float ov = bv[lid + s];
                const uint32_t oi = bi[lid + s];
                if (ov > bv[lid] || (ov == bv[lid] && oi < bi[lid])) {
                    bv[lid] = ov;
                    bi[lid] = oi;
                }
            }
        out[row] = ids ? ids[bi[0]] : bi[0];
    }
}
