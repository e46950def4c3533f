/* CPU restatement of NNop's memory-bound ops, fp32, multi-threaded.
 *
 * TEST INFRASTRUCTURE ONLY: the CPU baseline of bench.py's memory suite and a
 * second checker for the tests.  The product (libnnop_b200.so) never links or
 * calls it.
 *
 * What it restates (reference package NNop v0.2.0, Julia), rows contiguous:
 *   rms_norm    src/rms_norm.jl:3-38 (y = (w + offset) x rstd,
 *               rstd = 1/sqrt(mean(x^2) + eps)) and its backward
 *               src/rms_norm.jl:43-115 (dx = rstd m - rstd^3/N (sum m x) x with
 *               m = dy (w + offset); dw = sum over rows of dy x rstd);
 *   layer_norm  src/layer_norm.jl:8-63 (biased variance) and its backward
 *               src/layer_norm.jl:65-148 (c1 = mean(w dy xn), c2 = mean(w dy),
 *               dx = (w dy - (xn c1 + c2)) rstd, dw = sum dy xn, db = sum dy);
 *   online_softmax src/softmax.jl:1-58 (over each row) and its backward
 *               src/softmax.jl:70-80 (dx = dy y - y sum(dy y));
 *   llama_rope  src/rope/llama_rope.jl:24-98: pairs (i, i + E/2) rotated by
 *               cos/sin of index i, the backward with the sine negated.
 * Rows are split evenly over the threads; the weight gradients are summed
 * from per-thread partials. */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* Row kernels are built for x86-64-v4 (AVX-512), v3 (AVX2 + FMA) and the
   baseline, the best chosen when the library loads. */
#define ROWS_ISA __attribute__((target_clones("arch=x86-64-v4", "arch=x86-64-v3", "default")))

typedef float v8 __attribute__((vector_size(32)));
typedef int v8i __attribute__((vector_size(32)));

static inline v8 ld8(const float *p)
{
    v8 v;
    __builtin_memcpy(&v, p, sizeof v);
    return v;
}

static inline void st8(float *p, v8 v) { __builtin_memcpy(p, &v, sizeof v); }

static inline v8 bc8(float x) { return (v8){0} + x; }

static inline v8 sel8(v8i m, v8 a, v8 b) { return (v8)(((v8i)a & m) | ((v8i)b & ~m)); }

static inline float hsum8(v8 v)
{
    float s = 0.0f;
    for (int i = 0; i < 8; ++i)
        s += v[i];
    return s;
}

/* exp by Cody-Waite reduction and a degree-6 Taylor polynomial of e^r,
 * |r| <= ln2/2 (the same method as the attention restatement); 0 below -87. */
static inline v8 vexp8(v8 x)
{
    const v8i tiny = x < bc8(-87.0f);
    x = sel8(x > bc8(88.0f), bc8(88.0f), x);
    x = sel8(tiny, bc8(-87.0f), x);
    const v8 n = (x * 1.44269504088896341f + 12582912.0f) - 12582912.0f;
    v8 r = x - n * 0.693359375f;
    r = r - n * -2.12194440054690583e-4f;
    v8 p = bc8(1.0f / 720.0f);
    p = p * r + 1.0f / 120.0f;
    p = p * r + 1.0f / 24.0f;
    p = p * r + 1.0f / 6.0f;
    p = p * r + 0.5f;
    p = p * r + 1.0f;
    p = p * r + 1.0f;
    const v8i e = (__builtin_convertvector(n, v8i) + 127) << 23;
    return (v8)((v8i)(p * (v8)e) & ~tiny);
}

static inline float sexp(float x)
{
    v8 v = bc8(x);
    return vexp8(v)[0];
}

/* ---------------------------------------------------------------- rows pool */
typedef void (*rows_fn)(void *ctx, long lo, long hi, int tid);

typedef struct {
    rows_fn fn;
    void *ctx;
    long lo, hi;
    int tid;
} part_t;

static void *part_run(void *a)
{
    part_t *p = (part_t *)a;
    p->fn(p->ctx, p->lo, p->hi, p->tid);
    return 0;
}

/* fn over rows [0, n) in nthreads even, contiguous parts (the caller runs part
 * 0 and any part whose thread could not start). */
static int parallel_rows(rows_fn fn, void *ctx, long n, int nthreads)
{
    if (nthreads < 1)
        nthreads = 1;
    if (n < nthreads)
        nthreads = n > 0 ? (int)n : 1;
    part_t *parts = calloc((size_t)nthreads, sizeof(part_t));
    pthread_t *tid = calloc((size_t)nthreads, sizeof(pthread_t));
    char *started = calloc((size_t)nthreads, 1);
    if (!parts || !tid || !started) {
        free(parts), free(tid), free(started);
        return -3;
    }
    for (int t = 0; t < nthreads; ++t)
        parts[t] = (part_t){fn, ctx, n * t / nthreads, n * (t + 1) / nthreads, t};
    for (int t = 1; t < nthreads; ++t)
        started[t] = pthread_create(&tid[t], 0, part_run, &parts[t]) == 0;
    part_run(&parts[0]);
    for (int t = 1; t < nthreads; ++t) {
        if (started[t])
            pthread_join(tid[t], 0);
        else
            part_run(&parts[t]);
    }
    free(parts), free(tid), free(started);
    return 0;
}

/* Column sums of per-thread partials: out[e] = sum_t part[t][e]. */
static void sum_parts(const float *part, int nparts, int emb, float *out)
{
    for (int e = 0; e < emb; ++e) {
        float s = 0.0f;
        for (int t = 0; t < nparts; ++t)
            s += part[(size_t)t * emb + e];
        out[e] = s;
    }
}

static int threads_for(long n, int nthreads)
{
    if (nthreads < 1)
        nthreads = 1;
    return n < nthreads ? (n > 0 ? (int)n : 1) : nthreads;
}

/* Row sum of a*b over emb floats (8-wide partial sums, then the tail). */
static inline float dot(const float *a, const float *b, int emb)
{
    v8 s = (v8){0};
    int e = 0;
    for (; e + 8 <= emb; e += 8)
        s += ld8(a + e) * ld8(b + e);
    float t = hsum8(s);
    for (; e < emb; ++e)
        t += a[e] * b[e];
    return t;
}

static inline float rowsum(const float *a, int emb)
{
    v8 s = (v8){0};
    int e = 0;
    for (; e + 8 <= emb; e += 8)
        s += ld8(a + e);
    float t = hsum8(s);
    for (; e < emb; ++e)
        t += a[e];
    return t;
}

/* ---------------------------------------------------------------- RMSNorm */
typedef struct {
    const float *x, *w, *dy, *rstd_in;
    float *y, *rstd, *dx, *part;
    int emb;
    float eps, offset;
} norm_ctx;

ROWS_ISA static void rms_fwd_rows(void *c_, long lo, long hi, int tid)
{
    (void)tid;
    const norm_ctx *c = c_;
    const int emb = c->emb;
    for (long r = lo; r < hi; ++r) {
        const float *x = c->x + (size_t)r * emb;
        float *y = c->y + (size_t)r * emb;
        const float rs = 1.0f / sqrtf(dot(x, x, emb) / (float)emb + c->eps);
        c->rstd[r] = rs;
        for (int e = 0; e < emb; ++e)
            y[e] = (c->w[e] + c->offset) * x[e] * rs;
    }
}

int nnop_cpu_rms_norm_fwd(const float *x, const float *w, float *y, float *rstd, int emb, long n, float eps,
                          float offset, int nthreads)
{
    if (emb <= 0 || n < 0)
        return -1;
    norm_ctx c = {.x = x, .w = w, .y = y, .rstd = rstd, .emb = emb, .eps = eps, .offset = offset};
    return parallel_rows(rms_fwd_rows, &c, n, nthreads);
}

ROWS_ISA static void rms_bwd_rows(void *c_, long lo, long hi, int tid)
{
    const norm_ctx *c = c_;
    const int emb = c->emb;
    float *dw = c->part + (size_t)tid * emb;
    memset(dw, 0, (size_t)emb * sizeof(float));
    for (long r = lo; r < hi; ++r) {
        const float *x = c->x + (size_t)r * emb, *dy = c->dy + (size_t)r * emb;
        float *dx = c->dx + (size_t)r * emb;
        const float rs = c->rstd_in[r];
        v8 d8 = (v8){0};
        int e = 0;
        for (; e + 8 <= emb; e += 8)
            d8 += ld8(dy + e) * (ld8(c->w + e) + c->offset) * ld8(x + e);
        float dd = hsum8(d8);
        for (; e < emb; ++e)
            dd += dy[e] * (c->w[e] + c->offset) * x[e];
        const float k = rs * rs * rs * dd / (float)emb;
        for (e = 0; e < emb; ++e) {
            dx[e] = rs * dy[e] * (c->w[e] + c->offset) - k * x[e];
            dw[e] += dy[e] * x[e] * rs;
        }
    }
}

int nnop_cpu_rms_norm_bwd(const float *dy, const float *x, const float *w, const float *rstd, float *dx, float *dw,
                          int emb, long n, float offset, int nthreads)
{
    if (emb <= 0 || n < 0)
        return -1;
    const int nt = threads_for(n, nthreads);
    norm_ctx c = {.x = x, .w = w, .dy = dy, .rstd_in = rstd, .dx = dx, .emb = emb, .offset = offset};
    c.part = calloc((size_t)nt * emb, sizeof(float));
    if (!c.part)
        return -3;
    const int rc = parallel_rows(rms_bwd_rows, &c, n, nt);
    sum_parts(c.part, nt, emb, dw);
    free(c.part);
    return rc;
}

/* -------------------------------------------------------------- LayerNorm */
typedef struct {
    const float *x, *w, *b, *dy, *mean_in, *rstd_in;
    float *y, *mean, *rstd, *dx, *part;
    int emb;
    float eps;
} ln_ctx;

ROWS_ISA static void ln_fwd_rows(void *c_, long lo, long hi, int tid)
{
    (void)tid;
    const ln_ctx *c = c_;
    const int emb = c->emb;
    for (long r = lo; r < hi; ++r) {
        const float *x = c->x + (size_t)r * emb;
        float *y = c->y + (size_t)r * emb;
        const float mu = rowsum(x, emb) / (float)emb;
        v8 v8s = (v8){0};
        int e = 0;
        for (; e + 8 <= emb; e += 8) {
            const v8 d = ld8(x + e) - mu;
            v8s += d * d;
        }
        float var = hsum8(v8s);
        for (; e < emb; ++e)
            var += (x[e] - mu) * (x[e] - mu);
        const float rs = 1.0f / sqrtf(var / (float)emb + c->eps);
        c->mean[r] = mu;
        c->rstd[r] = rs;
        for (e = 0; e < emb; ++e)
            y[e] = (x[e] - mu) * rs * c->w[e] + c->b[e];
    }
}

int nnop_cpu_layer_norm_fwd(const float *x, const float *w, const float *b, float *y, float *mean, float *rstd,
                            int emb, long n, float eps, int nthreads)
{
    if (emb <= 0 || n < 0)
        return -1;
    ln_ctx c = {.x = x, .w = w, .b = b, .y = y, .mean = mean, .rstd = rstd, .emb = emb, .eps = eps};
    return parallel_rows(ln_fwd_rows, &c, n, nthreads);
}

ROWS_ISA static void ln_bwd_rows(void *c_, long lo, long hi, int tid)
{
    const ln_ctx *c = c_;
    const int emb = c->emb;
    float *dw = c->part + (size_t)tid * 2 * emb, *db = dw + emb;
    memset(dw, 0, (size_t)2 * emb * sizeof(float));
    for (long r = lo; r < hi; ++r) {
        const float *x = c->x + (size_t)r * emb, *dy = c->dy + (size_t)r * emb;
        float *dx = c->dx + (size_t)r * emb;
        const float mu = c->mean_in[r], rs = c->rstd_in[r];
        v8 a1 = (v8){0}, a2 = (v8){0};
        int e = 0;
        for (; e + 8 <= emb; e += 8) {
            const v8 wdy = ld8(c->w + e) * ld8(dy + e);
            a1 += wdy * ((ld8(x + e) - mu) * rs);
            a2 += wdy;
        }
        float c1 = hsum8(a1), c2 = hsum8(a2);
        for (; e < emb; ++e) {
            const float wdy = c->w[e] * dy[e];
            c1 += wdy * (x[e] - mu) * rs;
            c2 += wdy;
        }
        c1 /= (float)emb;
        c2 /= (float)emb;
        for (e = 0; e < emb; ++e) {
            const float xn = (x[e] - mu) * rs;
            dx[e] = (c->w[e] * dy[e] - (xn * c1 + c2)) * rs;
            dw[e] += dy[e] * xn;
            db[e] += dy[e];
        }
    }
}

int nnop_cpu_layer_norm_bwd(const float *dy, const float *x, const float *w, const float *mean, const float *rstd,
                            float *dx, float *dw, float *db, int emb, long n, int nthreads)
{
    if (emb <= 0 || n < 0)
        return -1;
    const int nt = threads_for(n, nthreads);
    ln_ctx c = {.x = x, .w = w, .dy = dy, .mean_in = mean, .rstd_in = rstd, .dx = dx, .emb = emb};
    c.part = calloc((size_t)nt * 2 * emb, sizeof(float));
    if (!c.part)
        return -3;
    const int rc = parallel_rows(ln_bwd_rows, &c, n, nt);
    for (int e = 0; e < emb; ++e) {
        float sw = 0.0f, sb = 0.0f;
        for (int t = 0; t < nt; ++t) {
            sw += c.part[(size_t)t * 2 * emb + e];
            sb += c.part[(size_t)t * 2 * emb + emb + e];
        }
        dw[e] = sw;
        db[e] = sb;
    }
    free(c.part);
    return rc;
}

/* ---------------------------------------------------------------- softmax */
typedef struct {
    const float *x, *y, *dy;
    float *out;
    int N;
} sm_ctx;

ROWS_ISA static void sm_fwd_rows(void *c_, long lo, long hi, int tid)
{
    (void)tid;
    const sm_ctx *c = c_;
    const int N = c->N;
    for (long r = lo; r < hi; ++r) {
        const float *x = c->x + (size_t)r * N;
        float *y = c->out + (size_t)r * N;
        v8 m8 = bc8(-INFINITY);
        int i = 0;
        for (; i + 8 <= N; i += 8) {
            const v8 v = ld8(x + i);
            m8 = sel8(v > m8, v, m8);
        }
        float m = m8[0];
        for (int l = 1; l < 8; ++l)
            m = m8[l] > m ? m8[l] : m;
        for (; i < N; ++i)
            m = x[i] > m ? x[i] : m;
        v8 s8 = (v8){0};
        i = 0;
        for (; i + 8 <= N; i += 8) {
            const v8 t = vexp8(ld8(x + i) - m);
            st8(y + i, t);
            s8 += t;
        }
        float s = hsum8(s8);
        for (; i < N; ++i) {
            y[i] = sexp(x[i] - m);
            s += y[i];
        }
        const float inv = 1.0f / s;    /* an all -Inf row: m = -Inf, NaN like the naive softmax */
        if (m == -INFINITY)
            for (i = 0; i < N; ++i)
                y[i] = NAN;
        else
            for (i = 0; i < N; ++i)
                y[i] *= inv;
    }
}

int nnop_cpu_softmax_fwd(const float *x, float *y, int N, long rows, int nthreads)
{
    if (N <= 0 || rows < 0)
        return -1;
    sm_ctx c = {.x = x, .out = y, .N = N};
    return parallel_rows(sm_fwd_rows, &c, rows, nthreads);
}

ROWS_ISA static void sm_bwd_rows(void *c_, long lo, long hi, int tid)
{
    (void)tid;
    const sm_ctx *c = c_;
    const int N = c->N;
    for (long r = lo; r < hi; ++r) {
        const float *y = c->y + (size_t)r * N, *dy = c->dy + (size_t)r * N;
        float *dx = c->out + (size_t)r * N;
        const float s = dot(dy, y, N);
        for (int i = 0; i < N; ++i)
            dx[i] = dy[i] * y[i] - y[i] * s;
    }
}

int nnop_cpu_softmax_bwd(const float *dy, const float *y, float *dx, int N, long rows, int nthreads)
{
    if (N <= 0 || rows < 0)
        return -1;
    sm_ctx c = {.y = y, .dy = dy, .out = dx, .N = N};
    return parallel_rows(sm_bwd_rows, &c, rows, nthreads);
}

/* ------------------------------------------------------------------ RoPE */
typedef struct {
    const float *x, *cos, *sin;
    float *out;
    int E, L, H;
    float sign;
} rope_ctx;

ROWS_ISA static void rope_rows(void *c_, long lo, long hi, int tid)
{
    (void)tid;
    const rope_ctx *c = c_;
    const int E = c->E, half = E / 2;
    for (long r = lo; r < hi; ++r) {           /* r = (b * H + h) * L + l */
        const long l = r % c->L, b = r / ((long)c->L * c->H);
        const float *x = c->x + (size_t)r * E;
        const float *cs = c->cos + ((size_t)b * c->L + l) * E, *sn = c->sin + ((size_t)b * c->L + l) * E;
        float *o = c->out + (size_t)r * E;
        for (int i = 0; i < half; ++i) {
            const float s = sn[i] * c->sign, x1 = x[i], x2 = x[i + half];
            o[i] = x1 * cs[i] - x2 * s;
            o[i + half] = x2 * cs[i] + x1 * s;
        }
    }
}

/* q (B,QH,L,E), k (B,KH,L,E), cos/sin (B,L,E); sign +1 forward, -1 backward. */
int nnop_cpu_llama_rope(const float *q, const float *k, const float *cos, const float *sin, float *qo, float *ko,
                        int E, int L, int QH, int KH, int B, float sign, int nthreads)
{
    if (E <= 0 || E % 2 || L < 0 || QH <= 0 || KH <= 0 || B < 0)
        return -1;
    rope_ctx c = {.x = q, .cos = cos, .sin = sin, .out = qo, .E = E, .L = L, .H = QH, .sign = sign};
    int rc = parallel_rows(rope_rows, &c, (long)B * QH * L, nthreads);
    if (rc)
        return rc;
    c.x = k, c.out = ko, c.H = KH;
    return parallel_rows(rope_rows, &c, (long)B * KH * L, nthreads);
}
