/* Blocked fp32 attention forward/backward -- one instruction-set instance.
 *
 * TEST INFRASTRUCTURE ONLY (the CPU baseline and a second checker); see
 * attention_cpu.c, which includes this file once per instruction set with
 *   ISA   the name suffix (generic, avx2, avx512)
 *   VW    floats per vector register
 *   ROWS  rows of the register tile of the block products
 *   CW    vectors per row of that tile
 * defined, inside "#pragma GCC target" for that set.
 *
 * Block products use GCC vector extensions: a ROWS x (CW*VW) tile of C lives
 * in registers while the shared dimension streams through.  The algorithm is
 * the reference's (src/attention.jl:8-143 forward with an online softmax;
 * src/attention_bwd.jl:1-175 backward with P recomputed from the saved
 * log-sum-exp), on 64 x 64 blocks. */

#define CAT2_(a, b) a##_##b
#define CAT_(a, b) CAT2_(a, b)
#define SFX(n) CAT_(n, ISA)
#define VF SFX(vf)
#define VI SFX(vi)

typedef float VF __attribute__((vector_size(VW * 4)));
typedef int VI __attribute__((vector_size(VW * 4)));

static inline VF SFX(ld)(const float *p)
{
    VF v;
    __builtin_memcpy(&v, p, sizeof v);
    return v;
}

static inline void SFX(st)(float *p, VF v) { __builtin_memcpy(p, &v, sizeof v); }

static inline VF SFX(bc)(float x) { return (VF){0} + x; }

static inline VF SFX(sel)(VI m, VF a, VF b) { return (VF)(((VI)a & m) | ((VI)b & ~m)); }

/* exp(x) by Cody-Waite range reduction and a Taylor polynomial (Cody & Waite,
 * "Software Manual for the Elementary Functions", 1980): x = n*ln2 + r with
 * n = round(x/ln2), |r| <= ln2/2, ln2 split into a short high part (exact
 * products n*hi) and a low correction; e^r by its degree-6 Taylor polynomial
 * (truncation below 1.2e-7 relative); the result is e^r * 2^n with 2^n built
 * in the exponent field.  Inputs below -87 (including -Inf) give 0. */
static inline VF SFX(vexp)(VF x)
{
    const VI tiny = x < SFX(bc)(-87.0f);
    x = SFX(sel)(x > SFX(bc)(88.0f), SFX(bc)(88.0f), x);
    x = SFX(sel)(tiny, SFX(bc)(-87.0f), x);
    const VF shifter = SFX(bc)(12582912.0f);            /* 1.5 * 2^23: round to nearest */
    const VF n = (x * 1.44269504088896341f + shifter) - shifter;
    VF r = x - n * 0.693359375f;
    r = r - n * -2.12194440054690583e-4f;
    VF p = SFX(bc)(1.0f / 720.0f);
    p = p * r + 1.0f / 120.0f;
    p = p * r + 1.0f / 24.0f;
    p = p * r + 1.0f / 6.0f;
    p = p * r + 0.5f;
    p = p * r + 1.0f;
    p = p * r + 1.0f;
    const VI e = (__builtin_convertvector(n, VI) + 127) << 23;
    const VF y = p * (VF)e;
    return (VF)((VI)y & ~tiny);
}

static inline float SFX(hmax)(VF v)
{
    float m = v[0];
    for (int l = 1; l < VW; ++l)
        m = v[l] > m ? v[l] : m;
    return m;
}

static inline float SFX(hsum)(VF v)
{
    float s = 0.0f;
    for (int l = 0; l < VW; ++l)
        s += v[l];
    return s;
}

/* C[M][N] = A[M][K] * B[K][N] (acc = 0) or C += A*B (acc = 1); all row-major
 * with leading dimensions; M % ROWS == 0 and N % VW == 0. */
static void SFX(gemm)(int M, int N, int K, const float *restrict A, int lda, const float *restrict B, int ldb,
                      float *restrict C, int ldc, int acc)
{
    for (int i = 0; i < M; i += ROWS) {
        int n = 0;
        for (; n + CW * VW <= N; n += CW * VW) {
            VF c[ROWS][CW];
#pragma GCC unroll 16
            for (int r = 0; r < ROWS; ++r)
#pragma GCC unroll 16
                for (int w = 0; w < CW; ++w)
                    c[r][w] = acc ? SFX(ld)(C + (size_t)(i + r) * ldc + n + w * VW) : (VF){0};
            for (int kk = 0; kk < K; ++kk) {
                VF b[CW];
#pragma GCC unroll 16
                for (int w = 0; w < CW; ++w)
                    b[w] = SFX(ld)(B + (size_t)kk * ldb + n + w * VW);
#pragma GCC unroll 16
                for (int r = 0; r < ROWS; ++r) {
                    const VF a = SFX(bc)(A[(size_t)(i + r) * lda + kk]);
#pragma GCC unroll 16
                    for (int w = 0; w < CW; ++w)
                        c[r][w] += a * b[w];
                }
            }
#pragma GCC unroll 16
            for (int r = 0; r < ROWS; ++r)
#pragma GCC unroll 16
                for (int w = 0; w < CW; ++w)
                    SFX(st)(C + (size_t)(i + r) * ldc + n + w * VW, c[r][w]);
        }
        for (; n < N; n += VW) {
            VF c[ROWS];
#pragma GCC unroll 16
            for (int r = 0; r < ROWS; ++r)
                c[r] = acc ? SFX(ld)(C + (size_t)(i + r) * ldc + n) : (VF){0};
            for (int kk = 0; kk < K; ++kk) {
                const VF b = SFX(ld)(B + (size_t)kk * ldb + n);
#pragma GCC unroll 16
                for (int r = 0; r < ROWS; ++r)
                    c[r] += SFX(bc)(A[(size_t)(i + r) * lda + kk]) * b;
            }
#pragma GCC unroll 16
            for (int r = 0; r < ROWS; ++r)
                SFX(st)(C + (size_t)(i + r) * ldc + n, c[r]);
        }
    }
}

/* Logits of one 64 x 64 block in place: s <- s*scale + pair, -Inf where the
 * key is invalid (past KL, after the query under the causal mask, or dropped by
 * the key-padding mask).  Rows i >= nq are left as they are. */
static void SFX(logits)(const job_t *jb, float *restrict s, const float *restrict pb, int b, int q0, int nq, int k0,
                        int nk, int masked)
{
    const float scale = jb->scale;
    if (!masked) {
        for (int i = 0; i < nq; ++i)
            for (int j = 0; j < BK; j += VW) {
                VF x = SFX(ld)(s + i * BK + j) * scale;
                if (pb)
                    x += SFX(ld)(pb + i * BK + j);
                SFX(st)(s + i * BK + j, x);
            }
        return;
    }
    const uint8_t *mk = jb->mask ? jb->mask + (size_t)b * jb->KL : 0;
    for (int i = 0; i < nq; ++i) {
        const int qi = q0 + i;
        for (int j = 0; j < BK; ++j) {
            const int kj = k0 + j;
            const int ok = j < nk && !(jb->causal && kj > qi) && !(mk && !mk[kj]);
            s[i * BK + j] = ok ? s[i * BK + j] * scale + (pb ? pb[i * BK + j] : 0.0f) : -INFINITY;
        }
    }
}

/* Does block (queries q0.., keys k0..) need per-element masking?  It does when
 * it is ragged (nk < BK), when the key-padding mask drops one of its keys, or
 * when a key lies after the first query under the causal mask. */
static int SFX(block_masked)(const job_t *jb, int b, int q0, int k0, int nk)
{
    if (nk < BK)
        return 1;
    if (jb->kblock_full && !jb->kblock_full[(size_t)b * jb->nkb + k0 / BK])
        return 1;
    return jb->causal && k0 + BK - 1 > q0;
}

/* pb[hh][i][j] = pair[b][k0 + j][q0 + i][h0 + hh] for i < nq, j < nk; a head's
 * block is PBS floats long.  Keys go in chunks of 8, so each (query, chunk)
 * reads 8 runs of G heads and fills 8 consecutive floats of G staging lines. */
static void SFX(gather_pair)(const job_t *jb, float *restrict pb, int b, int h0, int G, int q0, int nq, int k0, int nk)
{
    const int QL = jb->QL, QH = jb->QH;
    for (int j0 = 0; j0 < nk; j0 += 8) {
        const int jn = nk - j0 < 8 ? nk - j0 : 8;
        for (int i = 0; i < nq; ++i)
            for (int jj = 0; jj < jn; ++jj) {
                const float *src = jb->pair + (((size_t)b * jb->KL + k0 + j0 + jj) * QL + q0 + i) * QH + h0;
                float *dst = pb + (size_t)i * BK + j0 + jj;
                for (int hh = 0; hh < G; ++hh)
                    dst[(size_t)hh * PBS] = src[hh];
            }
    }
}

/* dpair[b][k0 + j][q0 + i][h0 + hh] = dsb[hh][i][j], the inverse of gather_pair. */
static void SFX(scatter_dpair)(const job_t *jb, const float *restrict dsb, int b, int h0, int G, int q0, int nq,
                               int k0, int nk)
{
    const int QL = jb->QL, QH = jb->QH;
    for (int j0 = 0; j0 < nk; j0 += 8) {
        const int jn = nk - j0 < 8 ? nk - j0 : 8;
        for (int i = 0; i < nq; ++i)
            for (int jj = 0; jj < jn; ++jj) {
                float *dst = jb->dpair + (((size_t)b * jb->KL + k0 + j0 + jj) * QL + q0 + i) * QH + h0;
                const float *src = dsb + (size_t)i * BK + j0 + jj;
                for (int hh = 0; hh < G; ++hh)
                    dst[hh] = src[(size_t)hh * PBS];
            }
    }
}

/* kt[e][j] = K[k0 + j][e] (zero for j >= nk); optionally kr[j][e] = K rows. */
static void SFX(load_keys)(const float *src, int E, int nk, float *restrict kt, float *restrict kr)
{
    for (int e = 0; e < E; ++e)
        for (int j = 0; j < BK; ++j)
            kt[e * BK + j] = j < nk ? src[(size_t)j * E + e] : 0.0f;
    if (kr) {
        memcpy(kr, src, (size_t)nk * E * sizeof(float));
        memset(kr + (size_t)nk * E, 0, (size_t)(BK - nk) * E * sizeof(float));
    }
}

static void SFX(load_rows)(const float *src, int E, int n, float *restrict dst)
{
    memcpy(dst, src, (size_t)n * E * sizeof(float));
    memset(dst + (size_t)n * E, 0, (size_t)(BQ - n) * E * sizeof(float));
}

/* ------------------------------------------------------------------ forward
 * Task = (batch b, head group g, query block qb).  Key blocks outer, heads of
 * the group inner, so a pair block is gathered once for all heads. */
static void SFX(fwd_task)(job_t *jb, float *ws, int task)
{
    const int E = jb->E, QL = jb->QL, KL = jb->KL, QH = jb->QH, KH = jb->KH, G = jb->G;
    const int rep = QH / KH;
    const int qb = task % jb->nqb, g = (task / jb->nqb) % jb->ngroups, b = task / (jb->nqb * jb->ngroups);
    const int h0 = g * G, q0 = qb * BQ, nq = QL - q0 < BQ ? QL - q0 : BQ;
    float *qs = ws;                                   /* [G][BQ][E] */
    float *acc = qs + (size_t)G * BQ * E;             /* [G][BQ][E] */
    float *m = acc + (size_t)G * BQ * E;              /* [G][BQ] */
    float *l = m + (size_t)G * BQ;                    /* [G][BQ] */
    float *kt = l + (size_t)G * BQ;                   /* [E][BK] */
    float *vs = kt + (size_t)E * BK;                  /* [BK][E] */
    float *s = vs + (size_t)BK * E;                   /* [BQ][BK] */
    float *pb = s + (size_t)BQ * BK;                  /* [G][PBS] */
    for (int hh = 0; hh < G; ++hh) {
        SFX(load_rows)(jb->q + (((size_t)b * QH + h0 + hh) * QL + q0) * E, E, nq, qs + (size_t)hh * BQ * E);
        for (int i = 0; i < BQ; ++i) {
            m[hh * BQ + i] = -INFINITY;
            l[hh * BQ + i] = 0.0f;
        }
    }
    memset(acc, 0, (size_t)G * BQ * E * sizeof(float));
    const int kend = jb->causal ? (q0 + nq < KL ? q0 + nq : KL) : KL;
    for (int k0 = 0; k0 < kend; k0 += BK) {
        const int nk = KL - k0 < BK ? KL - k0 : BK;
        const int masked = SFX(block_masked)(jb, b, q0, k0, nk);
        if (jb->pair)
            SFX(gather_pair)(jb, pb, b, h0, G, q0, nq, k0, nk);
        int cur = -1;
        for (int hh = 0; hh < G; ++hh) {
            const int h = h0 + hh, kvh = h / rep;
            if (kvh != cur) {
                const size_t off = (((size_t)b * KH + kvh) * KL + k0) * E;
                SFX(load_keys)(jb->k + off, E, nk, kt, 0);
                memcpy(vs, jb->v + off, (size_t)nk * E * sizeof(float));
                memset(vs + (size_t)nk * E, 0, (size_t)(BK - nk) * E * sizeof(float));
                cur = kvh;
            }
            SFX(gemm)(BQ, BK, E, qs + (size_t)hh * BQ * E, E, kt, BK, s, BK, 0);
            SFX(logits)(jb, s, jb->pair ? pb + (size_t)hh * PBS : 0, b, q0, nq, k0, nk, masked);
            float *mh = m + hh * BQ, *lh = l + hh * BQ, *ah = acc + (size_t)hh * BQ * E;
            for (int i = 0; i < nq; ++i) {
                float *row = s + i * BK;
                VF mv = SFX(ld)(row);
                for (int j = VW; j < BK; j += VW) {
                    const VF x = SFX(ld)(row + j);
                    mv = SFX(sel)(x > mv, x, mv);
                }
                const float mx = SFX(hmax)(mv);
                const float mnew = mx > mh[i] ? mx : mh[i];
                if (mnew == -INFINITY) {                 /* nothing visible yet in this row */
                    memset(row, 0, BK * sizeof(float));
                    continue;
                }
                VF sv = (VF){0};
                for (int j = 0; j < BK; j += VW) {
                    const VF p = SFX(vexp)(SFX(ld)(row + j) - mnew);
                    sv += p;
                    SFX(st)(row + j, p);
                }
                const float alpha = mh[i] == -INFINITY ? 0.0f : expf(mh[i] - mnew);
                lh[i] = lh[i] * alpha + SFX(hsum)(sv);
                mh[i] = mnew;
                if (alpha != 1.0f)
                    for (int e = 0; e < E; e += VW)
                        SFX(st)(ah + (size_t)i * E + e, SFX(ld)(ah + (size_t)i * E + e) * alpha);
            }
            if (nq < BQ)
                memset(s + (size_t)nq * BK, 0, (size_t)(BQ - nq) * BK * sizeof(float));
            SFX(gemm)(BQ, E, BK, s, BK, vs, E, ah, E, 1);
        }
    }
    for (int hh = 0; hh < G; ++hh) {
        const size_t row0 = ((size_t)b * QH + h0 + hh) * QL + q0;
        for (int i = 0; i < nq; ++i) {
            const float li = l[hh * BQ + i];
            float *dst = jb->o_out + (row0 + i) * E;
            const float *src = acc + ((size_t)hh * BQ + i) * E;
            if (li == 0.0f) {                            /* every key masked: NaN like softmax of all -Inf */
                for (int e = 0; e < E; ++e)
                    dst[e] = NAN;
                jb->lse_out[row0 + i] = NAN;
                continue;
            }
            const float inv = 1.0f / li;
            for (int e = 0; e < E; ++e)
                dst[e] = src[e] * inv;
            jb->lse_out[row0 + i] = m[hh * BQ + i] + logf(li);
        }
    }
}

/* ------------------------------------------------------------------ backward
 * Task = (batch b, head group g, key block kb): owns dK, dV and dpair of its
 * keys for every kv head of the group; dQ contributions are added to the
 * shared dq under a per-(b, h, query block) lock. */
static void SFX(bwd_task)(job_t *jb, float *ws, int task)
{
    const int E = jb->E, QL = jb->QL, KL = jb->KL, QH = jb->QH, KH = jb->KH, G = jb->G;
    const int rep = QH / KH, GK = G / rep > 0 ? G / rep : 1;
    const int kb = task % jb->nkb, g = (task / jb->nkb) % jb->ngroups, b = task / (jb->nkb * jb->ngroups);
    const int h0 = g * G, kv0 = h0 / rep, k0 = kb * BK, nk = KL - k0 < BK ? KL - k0 : BK;
    float *kt = ws;                                   /* [GK][E][BK] */
    float *vt = kt + (size_t)GK * E * BK;             /* [GK][E][BK] */
    float *kr = vt + (size_t)GK * E * BK;             /* [GK][BK][E] */
    float *dka = kr + (size_t)GK * BK * E;            /* [GK][BK][E] */
    float *dva = dka + (size_t)GK * BK * E;           /* [GK][BK][E] */
    float *qs = dva + (size_t)GK * BK * E;            /* [BQ][E] */
    float *dos = qs + (size_t)BQ * E;                 /* [BQ][E] */
    float *dqc = dos + (size_t)BQ * E;                /* [BQ][E] */
    float *s = dqc + (size_t)BQ * E;                  /* [BQ][BK] -> P */
    float *dp = s + (size_t)BQ * BK;                  /* [BQ][BK] -> dS */
    float *pt = dp + (size_t)BQ * BK;                 /* [BK][BQ] */
    float *dst = pt + (size_t)BK * BQ;                /* [BK][BQ] */
    float *pb = dst + (size_t)BK * BQ;                /* [G][PBS] pair block */
    float *dsb = pb + (size_t)G * PBS;                /* [G][PBS] dS staging for dpair */
    for (int c = 0; c < GK; ++c) {
        const size_t off = (((size_t)b * KH + kv0 + c) * KL + k0) * E;
        SFX(load_keys)(jb->k + off, E, nk, kt + (size_t)c * E * BK, kr + (size_t)c * BK * E);
        SFX(load_keys)(jb->v + off, E, nk, vt + (size_t)c * E * BK, 0);
    }
    memset(dka, 0, (size_t)GK * BK * E * sizeof(float));
    memset(dva, 0, (size_t)GK * BK * E * sizeof(float));
    const int qstart = jb->causal ? k0 / BQ : 0;
    for (int qb = qstart; qb < jb->nqb; ++qb) {
        const int q0 = qb * BQ, nq = QL - q0 < BQ ? QL - q0 : BQ;
        const int masked = SFX(block_masked)(jb, b, q0, k0, nk);
        if (jb->pair)
            SFX(gather_pair)(jb, pb, b, h0, G, q0, nq, k0, nk);
        for (int hh = 0; hh < G; ++hh) {
            const int h = h0 + hh, c = h / rep - kv0;
            const size_t row0 = ((size_t)b * QH + h) * QL + q0;
            SFX(load_rows)(jb->q + row0 * E, E, nq, qs);
            SFX(load_rows)(jb->dout + row0 * E, E, nq, dos);
            SFX(gemm)(BQ, BK, E, qs, E, kt + (size_t)c * E * BK, BK, s, BK, 0);
            SFX(gemm)(BQ, BK, E, dos, E, vt + (size_t)c * E * BK, BK, dp, BK, 0);
            SFX(logits)(jb, s, jb->pair ? pb + (size_t)hh * PBS : 0, b, q0, nq, k0, nk, masked);
            for (int i = 0; i < nq; ++i) {
                const float lse = jb->lse_in[row0 + i], dl = jb->delta[row0 + i];
                for (int j = 0; j < BK; j += VW) {
                    const VF p = SFX(vexp)(SFX(ld)(s + i * BK + j) - lse);
                    SFX(st)(s + i * BK + j, p);
                    SFX(st)(dp + i * BK + j, p * (SFX(ld)(dp + i * BK + j) - dl));
                }
            }
            if (nq < BQ) {
                memset(s + (size_t)nq * BK, 0, (size_t)(BQ - nq) * BK * sizeof(float));
                memset(dp + (size_t)nq * BK, 0, (size_t)(BQ - nq) * BK * sizeof(float));
            }
            for (int i = 0; i < BQ; ++i)
                for (int j = 0; j < BK; ++j) {
                    pt[j * BQ + i] = s[i * BK + j];
                    dst[j * BQ + i] = dp[i * BK + j];
                }
            SFX(gemm)(BK, E, BQ, pt, BQ, dos, E, dva + (size_t)c * BK * E, E, 1);
            SFX(gemm)(BK, E, BQ, dst, BQ, qs, E, dka + (size_t)c * BK * E, E, 1);
            SFX(gemm)(BQ, E, BK, dp, BK, kr + (size_t)c * BK * E, E, dqc, E, 0);
            if (jb->dpair)
                memcpy(dsb + (size_t)hh * PBS, dp, (size_t)BQ * BK * sizeof(float));
            atomic_int *lock = jb->locks + ((size_t)b * QH + h) * jb->nqb + qb;
            for (int spins = 0; atomic_exchange_explicit(lock, 1, memory_order_acquire); ++spins)
                if (spins > 64)
                    sched_yield();
            float *dq = jb->dq + row0 * E;
            for (int i = 0; i < nq; ++i)
                for (int e = 0; e < E; e += VW)
                    SFX(st)(dq + (size_t)i * E + e,
                            SFX(ld)(dq + (size_t)i * E + e) + SFX(ld)(dqc + (size_t)i * E + e) * jb->scale);
            atomic_store_explicit(lock, 0, memory_order_release);
        }
        if (jb->dpair)
            SFX(scatter_dpair)(jb, dsb, b, h0, G, q0, nq, k0, nk);
    }
    for (int c = 0; c < GK; ++c) {
        const size_t off = (((size_t)b * KH + kv0 + c) * KL + k0) * E;
        for (size_t x = 0; x < (size_t)nk * E; ++x) {
            jb->dk[off + x] = dka[(size_t)c * BK * E + x] * jb->scale;
            jb->dv[off + x] = dva[(size_t)c * BK * E + x];
        }
    }
}

#undef VF
#undef VI
#undef SFX
#undef CAT_
#undef CAT2_
