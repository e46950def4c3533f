/* CPU restatement of NNop's flash attention, fp32, multi-threaded and blocked.
 *
 * TEST INFRASTRUCTURE ONLY: the CPU baseline that bench.py times on the host
 * cores (its "cpu_baseline" and the "--impl reference" arm) and a second
 * checker for the tests.  The product (libnnop_b200.so) never links or calls
 * it.
 *
 * What it restates (reference package NNop v0.2.0, Julia):
 *   forward   src/attention.jl:8-143  -- blocks of queries against blocks of
 *             keys, logits (q.k)*scale + pair, causal mask "key j visible to
 *             query i iff j <= i" (src/attention.jl:76-81), key-padding mask,
 *             online softmax with a running max and denominator; saves
 *             lse = max + log(denominator) per query row;
 *   backward  src/attention_bwd.jl:1-175 -- P recomputed as exp(s - lse),
 *             dV = P^T dO, dP = dO V^T, dS = P o (dP - delta) with
 *             delta = rowsum(dO o O) (src/attention_bwd.jl:177-211),
 *             dpair = dS (zero where no key is visible, src/attention_bwd.jl:250),
 *             dK = scale dS^T Q, dQ = scale dS K; GQA query head h reads kv
 *             head h / (QH/KH) and its dK/dV are summed over those heads.
 * Layout: the reference's column-major arrays read as row-major
 *   q, o, dO, dq [B][QH][QL][E]; k, v, dk, dv [B][KH][KL][E];
 *   pair, dpair [B][KL][QL][QH]; kpad mask [B][KL] bytes; lse [B][QH][QL].
 * A query row whose keys are all masked gets NaN output and lse, as the naive
 * softmax of an all -Inf column does.
 *
 * Work is split into independent tasks run by a pool of pthreads (forward:
 * one task per batch, head group and 64-query block; backward: per batch,
 * head group and 64-key block, each owning its keys' dK, dV and dpair, with
 * dQ added under a per-block lock).  With a pair bias the head group is every
 * head, so each pair block is gathered once for all heads; otherwise it is the
 * query heads of one kv head.  Block products are register-tiled with GCC
 * vector extensions, compiled for AVX-512, AVX2+FMA and plain x86-64 and
 * chosen at run time. */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <sched.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define BQ 64
#define BK 64
/* floats per head in the pair / dS staging blocks: one cache line more than a
   block, so the heads' blocks fall in different cache sets */
#define PBS (BQ * BK + 16)

typedef struct job {
    const float *q, *k, *v, *pair, *dout, *lse_in, *o_in;
    const uint8_t *mask;
    uint8_t *kblock_full;      /* [B][nkb]: every key of the block kept by the mask (NULL: no mask) */
    float *o_out, *lse_out, *dq, *dk, *dv, *dpair, *delta;
    int E, QL, KL, QH, KH, B, causal;
    float scale;
    int G, ngroups, nqb, nkb;
    atomic_int *locks;
    int ntasks;
    int *order;
    atomic_int next;
    void (*task)(struct job *, float *, int);
    size_t ws_floats;
} job_t;

#pragma GCC push_options
#pragma GCC target("avx512f,avx512dq,avx512vl,avx2,fma")
#define ISA avx512
#define VW 16
#define ROWS 4
#define CW 4
#include "attention_cpu_impl.h"
#undef ISA
#undef VW
#undef ROWS
#undef CW
#pragma GCC pop_options

#pragma GCC push_options
#pragma GCC target("avx2,fma")
#define ISA avx2
#define VW 8
#define ROWS 4
#define CW 2
#include "attention_cpu_impl.h"
#undef ISA
#undef VW
#undef ROWS
#undef CW
#pragma GCC pop_options

#define ISA generic
#define VW 4
#define ROWS 2
#define CW 2
#include "attention_cpu_impl.h"
#undef ISA
#undef VW
#undef ROWS
#undef CW

enum { ISA_AUTO = 0, ISA_GENERIC = 1, ISA_AVX2 = 2, ISA_AVX512 = 3 };
static int g_forced = ISA_AUTO;

static int pick_isa(void)
{
    __builtin_cpu_init();
    const int best = __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512dq") &&
                             __builtin_cpu_supports("avx512vl")
                         ? ISA_AVX512
                         : (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") ? ISA_AVX2 : ISA_GENERIC);
    return g_forced != ISA_AUTO && g_forced <= best ? g_forced : best;
}

/* Instruction set used by the next call: "avx512", "avx2" or "generic". */
const char *nnop_cpu_isa(void)
{
    static const char *names[] = {"", "generic", "avx2", "avx512"};
    return names[pick_isa()];
}

/* Force an instruction set (0 auto, 1 generic, 2 avx2, 3 avx512) for the
 * tests; a set the CPU lacks falls back to the best it has.  Returns the set
 * now in use. */
int nnop_cpu_force_isa(int isa)
{
    g_forced = isa >= ISA_AUTO && isa <= ISA_AVX512 ? isa : ISA_AUTO;
    return pick_isa();
}

/* ------------------------------------------------------------ thread pool */
typedef struct {
    job_t *jb;
} worker_arg_t;

static void *worker(void *arg)
{
    job_t *jb = ((worker_arg_t *)arg)->jb;
    float *ws = 0;
    if (jb->ws_floats && posix_memalign((void **)&ws, 64, jb->ws_floats * sizeof(float)) != 0)
        return (void *)1;
    for (;;) {
        const int t = atomic_fetch_add_explicit(&jb->next, 1, memory_order_relaxed);
        if (t >= jb->ntasks)
            break;
        jb->task(jb, ws, jb->order ? jb->order[t] : t);
    }
    free(ws);
    return 0;
}

/* Runs every task of the job on nthreads threads (the caller's included). */
static int run_tasks(job_t *jb, int nthreads)
{
    atomic_store(&jb->next, 0);
    if (jb->ntasks <= 0)
        return 0;
    if (nthreads < 1)
        nthreads = 1;
    if (nthreads > jb->ntasks)
        nthreads = jb->ntasks;
    pthread_t *tid = calloc((size_t)nthreads, sizeof(pthread_t));
    if (!tid)
        return -3;
    worker_arg_t arg = {jb};
    int started = 0;                             /* threads that could not start leave their share to the others */
    for (int i = 1; i < nthreads; ++i)
        if (pthread_create(&tid[started], 0, worker, &arg) == 0)
            ++started;
    int rc = worker(&arg) ? -3 : 0;
    for (int i = 0; i < started; ++i) {
        void *r = 0;
        pthread_join(tid[i], &r);
        if (r)
            rc = -3;
    }
    free(tid);
    return rc;
}

/* -------------------------------------------------------- small parallel steps */
typedef struct {
    job_t base;
    void *ptr;
    size_t bytes, chunk;
} zero_job_t;

static void zero_task(job_t *jb, float *ws, int t)
{
    (void)ws;
    zero_job_t *z = (zero_job_t *)jb;
    const size_t lo = (size_t)t * z->chunk, hi = lo + z->chunk < z->bytes ? lo + z->chunk : z->bytes;
    memset((char *)z->ptr + lo, 0, hi - lo);
}

static int parallel_zero(void *ptr, size_t bytes, int nthreads)
{
    if (!ptr || !bytes)
        return 0;
    zero_job_t z;
    memset(&z, 0, sizeof z);
    z.ptr = ptr;
    z.bytes = bytes;
    z.chunk = (size_t)8 << 20;
    z.base.ntasks = (int)((bytes + z.chunk - 1) / z.chunk);
    z.base.task = zero_task;
    return run_tasks(&z.base, nthreads);
}

/* delta[row] = sum_e dO[row][e] * O[row][e] and dq[row] = 0, per (b, h). */
static void delta_task(job_t *jb, float *ws, int t)
{
    (void)ws;
    const size_t row0 = (size_t)t * jb->QL, E = (size_t)jb->E;
    for (int i = 0; i < jb->QL; ++i) {
        const float *d = jb->dout + (row0 + i) * E, *o = jb->o_in + (row0 + i) * E;
        float s = 0.0f;
        for (size_t e = 0; e < E; ++e)
            s += d[e] * o[e];
        jb->delta[row0 + i] = s;
    }
    memset(jb->dq + row0 * E, 0, (size_t)jb->QL * E * sizeof(float));
}

/* ---------------------------------------------------------------- set-up */
static int check_dims(int E, int QL, int KL, int QH, int KH, int B)
{
    if (E <= 0 || E % 16 || E > 512 || QL < 0 || KL < 0 || QH <= 0 || KH <= 0 || B < 0)
        return -1;
    if (QH % KH)
        return -1;
    return 0;
}

static int setup(job_t *jb, const uint8_t *mask, int has_pair)
{
    const int rep = jb->QH / jb->KH;
    jb->G = has_pair ? jb->QH : rep;
    jb->ngroups = jb->QH / jb->G;
    jb->nqb = (jb->QL + BQ - 1) / BQ;
    jb->nkb = (jb->KL + BK - 1) / BK;
    jb->mask = mask;
    jb->kblock_full = 0;
    if (mask && jb->B && jb->nkb) {
        jb->kblock_full = malloc((size_t)jb->B * jb->nkb);
        if (!jb->kblock_full)
            return -3;
        for (int b = 0; b < jb->B; ++b)
            for (int kb = 0; kb < jb->nkb; ++kb) {
                int full = 1;
                for (int j = kb * BK; j < (kb + 1) * BK && j < jb->KL; ++j)
                    full &= mask[(size_t)b * jb->KL + j] != 0;
                jb->kblock_full[(size_t)b * jb->nkb + kb] = (uint8_t)full;
            }
    }
    return 0;
}

/* Task order: most work first (the causal triangle makes blocks unequal). */
static int *largest_first(int ntasks, int nblocks, int causal, int forward)
{
    int *order = malloc((size_t)(ntasks > 0 ? ntasks : 1) * sizeof(int));
    if (!order)
        return 0;
    int n = 0;
    for (int step = 0; step < nblocks; ++step) {
        /* forward: query block nblocks-1 sees the most keys; backward: key block 0 sees the most queries */
        const int blk = causal ? (forward ? nblocks - 1 - step : step) : step;
        for (int t = 0; t < ntasks; ++t)
            if (t % nblocks == blk)
                order[n++] = t;
    }
    return order;
}

/* Forward: o [B][QH][QL][E], lse [B][QH][QL].  Returns 0, -1 for bad
 * dimensions (E a multiple of 16 up to 512, QH a multiple of KH), -3 when
 * memory or threads could not be had. */
int nnop_cpu_attention_fwd(const float *q, const float *k, const float *v, const float *pair,
                           const uint8_t *kpad_mask, float *o, float *lse, int E, int QL, int KL, int QH, int KH,
                           int B, int causal, float scale, int nthreads)
{
    if (check_dims(E, QL, KL, QH, KH, B))
        return -1;
    job_t jb;
    memset(&jb, 0, sizeof jb);
    jb.q = q, jb.k = k, jb.v = v, jb.pair = pair, jb.o_out = o, jb.lse_out = lse;
    jb.E = E, jb.QL = QL, jb.KL = KL, jb.QH = QH, jb.KH = KH, jb.B = B, jb.causal = causal, jb.scale = scale;
    int rc = setup(&jb, kpad_mask, pair != 0);
    if (rc)
        return rc;
    jb.ntasks = B * jb.ngroups * jb.nqb;
    jb.order = largest_first(jb.ntasks, jb.nqb, causal, 1);
    const size_t G = (size_t)jb.G;
    jb.ws_floats = 2 * G * BQ * E + 2 * G * BQ + 2 * (size_t)E * BK + (size_t)BQ * BK + G * PBS;
    const int isa = pick_isa();
    jb.task = isa == ISA_AVX512 ? fwd_task_avx512 : isa == ISA_AVX2 ? fwd_task_avx2 : fwd_task_generic;
    rc = jb.order ? run_tasks(&jb, nthreads) : -3;
    free(jb.order);
    free(jb.kblock_full);
    return rc;
}

/* Backward from the saved (o, lse): dq, dk, dv, and dpair when pair is given
 * (written in full, zero where the forward saw no key).  Same return codes. */
int nnop_cpu_attention_bwd(const float *dout, const float *o, const float *lse, const float *q, const float *k,
                           const float *v, const float *pair, const uint8_t *kpad_mask, float *dq, float *dk,
                           float *dv, float *dpair, int E, int QL, int KL, int QH, int KH, int B, int causal,
                           float scale, int nthreads)
{
    if (check_dims(E, QL, KL, QH, KH, B) || (pair && !dpair))
        return -1;
    job_t jb;
    memset(&jb, 0, sizeof jb);
    jb.dout = dout, jb.o_in = o, jb.lse_in = lse, jb.q = q, jb.k = k, jb.v = v, jb.pair = pair;
    jb.dq = dq, jb.dk = dk, jb.dv = dv, jb.dpair = pair ? dpair : 0;
    jb.E = E, jb.QL = QL, jb.KL = KL, jb.QH = QH, jb.KH = KH, jb.B = B, jb.causal = causal, jb.scale = scale;
    int rc = setup(&jb, kpad_mask, pair != 0);
    if (rc)
        return rc;
    const size_t rows = (size_t)B * QH * QL;
    jb.delta = malloc((rows ? rows : 1) * sizeof(float));
    jb.locks = calloc((size_t)B * QH * (jb.nqb ? jb.nqb : 1) + 1, sizeof(atomic_int));
    if (!jb.delta || !jb.locks)
        rc = -3;
    if (!rc) {                                   /* delta rows and dq = 0, one task per (b, h) */
        jb.ntasks = B * QH, jb.task = delta_task, jb.ws_floats = 0, jb.order = 0;
        rc = run_tasks(&jb, nthreads);
    }
    if (!rc && jb.dpair)
        rc = parallel_zero(jb.dpair, (size_t)B * KL * QL * QH * sizeof(float), nthreads);
    if (!rc) {
        jb.ntasks = B * jb.ngroups * jb.nkb;
        jb.order = largest_first(jb.ntasks, jb.nkb, causal, 0);
        const size_t G = (size_t)jb.G, GK = G / (size_t)(QH / KH) ? G / (size_t)(QH / KH) : 1;
        jb.ws_floats = 5 * GK * E * BK + 3 * (size_t)BQ * E + 4 * (size_t)BQ * BK + 2 * G * PBS;
        const int isa = pick_isa();
        jb.task = isa == ISA_AVX512 ? bwd_task_avx512 : isa == ISA_AVX2 ? bwd_task_avx2 : bwd_task_generic;
        rc = jb.order ? run_tasks(&jb, nthreads) : -3;
    }
    free(jb.order);
    free(jb.delta);
    free(jb.locks);
    free(jb.kblock_full);
    return rc;
}
