// Flash attention forward/backward for f16/bf16 on warp-level tensor-core MMA
// (mma.sync m16n8k16, fp32 accumulation).  This is the general path: every E
// in {16, 32, 64, 128}, pair bias, causal, GQA and key padding.
//
// Reference: `_flash_attention_fwd!` (src/attention.jl:8-143) and
// `_flash_attention_bwd!` (src/attention_bwd.jl:1-175).  The reference's forward
// keeps the softmax state in shared memory with one thread per query row and
// WMMA 16x16x16 tiles; its backward runs one workgroup per (head, batch) over
// every (k-tile, q-tile) pair.  Here:
// * forward: one CTA (4 warps) per (64-query tile, head, batch); each warp owns
//   16 query rows in registers; K/V tiles double-buffered with cp.async; the
//   online softmax runs on the MMA accumulators; causal CTAs skip key tiles
//   above the diagonal, and key tiles past the last kept key are skipped;
// * backward: one CTA per (64-key tile, KV head, batch) looping over the query
//   tiles of every query head of its GQA group, so dK/dV accumulate in
//   registers without atomics; dQ is accumulated in fp32 with atomics;
//   dpair = dS is written for every (query, key) the CTA visits.
#include "fa_common.cuh"

namespace nnop {
namespace fa {
namespace {

constexpr int kThreads = 128;
constexpr int kBM = 64;
constexpr int kBN = 64;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem),
                 "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);

template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                                        uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// cp.async a [64][E] tile (rows row0.., zero-filled past nrows) into smem with
// a padded row stride of E+8 elements (conflict-free ldmatrix).
template <typename T, int E>
__device__ __forceinline__ void load_tile(T* smem, const T* g, int64_t row0, int64_t nrows) {
    constexpr int CPR = E / 8;
    constexpr int SE = E + 8;
    constexpr int ITERS = (64 * CPR + kThreads - 1) / kThreads;
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
        const int c = threadIdx.x + it * kThreads;
        if (c < 64 * CPR) {
            const int r = c / CPR, ch = c % CPR;
            const int64_t gr = row0 + r;
            const bool ok = gr < nrows;
            const T* src = g + (ok ? gr : 0) * E + ch * 8;
            cp_async16(smem + r * SE + ch * 8, src, ok ? 16 : 0);
        }
    }
}

// ============================================================== forward
template <typename T, int E, bool CAUSAL>
__global__ void __launch_bounds__(kThreads) fa_fwd_mma_kernel(const Params p) {
    constexpr int SE = E + 8;
    constexpr int NT = kBN / 8;   // n-tiles of S
    constexpr int KS = E / 16;    // k-steps of QK^T
    constexpr int ET = E / 8;     // n-tiles of O
    extern __shared__ __align__(128) uint8_t smem_raw[];
    T* sQ = reinterpret_cast<T*>(smem_raw);
    T* sK = sQ + kBM * SE;
    T* sV = sK + 2 * kBN * SE;

    const int64_t QL = p.QL, KL = p.KL;
    const int n_qt = (int)((QL + kBM - 1) / kBM);
    const int qt = CAUSAL ? (n_qt - 1 - (int)blockIdx.x) : (int)blockIdx.x;
    const int h = blockIdx.y, b = blockIdx.z;
    const int kvh = h / p.n_rep;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    const int64_t q0 = (int64_t)qt * kBM;

    const T* qg = reinterpret_cast<const T*>(p.q) + ((int64_t)b * p.QH + h) * QL * E;
    const T* kg = reinterpret_cast<const T*>(p.k) + ((int64_t)b * p.KH + kvh) * KL * E;
    const T* vg = reinterpret_cast<const T*>(p.v) + ((int64_t)b * p.KH + kvh) * KL * E;
    const T* pg = p.pair ? reinterpret_cast<const T*>(p.pair) + (int64_t)b * KL * QL * p.QH + h : nullptr;
    const uint8_t* mg = p.kmask ? p.kmask + (int64_t)b * KL : nullptr;

    int64_t kv_len = KL;
    if (mg) kv_len = kv_valid_len_block(mg, KL);
    int n_kt = (int)((kv_len + kBN - 1) / kBN);
    if (CAUSAL) {
        const int64_t i_end = (q0 + kBM < QL ? q0 + kBM : QL);  // exclusive
        const int lim = (int)((i_end + kBN - 1) / kBN);
        n_kt = n_kt < lim ? n_kt : lim;
    }

    load_tile<T, E>(sQ, qg, q0, QL);
    if (n_kt > 0) load_tile<T, E>(sK, kg, 0, KL);
    cp_async_commit();
    if (n_kt > 0) load_tile<T, E>(sV, vg, 0, KL);
    cp_async_commit();

    float o_acc[ET][4];
#pragma unroll
    for (int i = 0; i < ET; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) o_acc[i][j] = 0.f;
    float m_r[2] = {-INFINITY, -INFINITY};
    float l_r[2] = {0.f, 0.f};
    uint32_t qf[KS][4];

    const int r_lo = warp * 16 + g;  // local rows r_lo, r_lo + 8
    const int64_t i_row[2] = {q0 + r_lo, q0 + r_lo + 8};
    const float scale = p.scale;

    for (int kt = 0; kt < n_kt; ++kt) {
        const int buf = kt & 1;
        const int64_t k0 = (int64_t)kt * kBN;
        // Pair values of this thread's fragment, fetched ahead of the MMA.
        float pv[NT][4];
        if (pg) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int64_t i = i_row[e >> 1];
                    const int64_t j = k0 + nt * 8 + 2 * t4 + (e & 1);
                    pv[nt][e] = (i < QL && j < KL) ? to_f(pg[(j * QL + i) * p.QH]) : 0.f;
                }
        }
        cp_async_wait<1>();
        __syncthreads();
        if (kt == 0) {
#pragma unroll
            for (int ks = 0; ks < KS; ++ks)
                ldsm_x4(qf[ks], sQ + (warp * 16 + (lane & 15)) * SE + ks * 16 + (lane >> 4) * 8);
        }
        const T* sKb = sK + buf * kBN * SE;
        float s[NT][4];
#pragma unroll
        for (int i = 0; i < NT; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
            for (int np = 0; np < NT / 2; ++np) {
                uint32_t bf[4];
                ldsm_x4(bf, sKb + (np * 16 + (lane & 7) + (lane >> 4) * 8) * SE + ks * 16 + ((lane >> 3) & 1) * 8);
                mma16816<T>(s[2 * np], qf[ks], bf[0], bf[1]);
                mma16816<T>(s[2 * np + 1], qf[ks], bf[2], bf[3]);
            }
        }
        if (kt + 1 < n_kt) load_tile<T, E>(sK + (buf ^ 1) * kBN * SE, kg, k0 + kBN, KL);
        cp_async_commit();

        // logits, masks, online softmax (natural-log units, exp via exp2)
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int64_t i = i_row[e >> 1];
                const int64_t j = k0 + nt * 8 + 2 * t4 + (e & 1);
                float x = s[nt][e] * scale;
                if (pg) x += pv[nt][e];
                bool valid = j < KL;
                if (CAUSAL) valid = valid && (j <= i);
                if (mg) valid = valid && (j < KL ? mg[j] != 0 : false);
                x = valid ? x : -INFINITY;
                s[nt][e] = x;
                mx[e >> 1] = fmaxf(mx[e >> 1], x);
            }
        float alpha[2], m_use[2];
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            float v = mx[rr];
            v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
            v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
            const float m_new = fmaxf(m_r[rr], v);
            m_use[rr] = (m_new == -INFINITY) ? 0.f : m_new;
            alpha[rr] = exp2f((m_r[rr] - m_use[rr]) * kLog2e);
            m_r[rr] = m_new;
            l_r[rr] *= alpha[rr];
        }
#pragma unroll
        for (int et = 0; et < ET; ++et) {
            o_acc[et][0] *= alpha[0];
            o_acc[et][1] *= alpha[0];
            o_acc[et][2] *= alpha[1];
            o_acc[et][3] *= alpha[1];
        }
        uint32_t pa[NT / 2][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float pe[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                pe[e] = exp2f((s[nt][e] - m_use[e >> 1]) * kLog2e);
                l_r[e >> 1] += pe[e];
            }
            pa[nt >> 1][(nt & 1) * 2 + 0] = pack2<T>(pe[0], pe[1]);
            pa[nt >> 1][(nt & 1) * 2 + 1] = pack2<T>(pe[2], pe[3]);
        }

        cp_async_wait<1>();
        __syncthreads();
        const T* sVb = sV + buf * kBN * SE;
#pragma unroll
        for (int kk = 0; kk < NT / 2; ++kk) {
#pragma unroll
            for (int ep = 0; ep < ET / 2; ++ep) {
                uint32_t bf[4];
                ldsm_x4_t(bf, sVb + (kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * SE + ep * 16 + (lane >> 4) * 8);
                mma16816<T>(o_acc[2 * ep], pa[kk], bf[0], bf[1]);
                mma16816<T>(o_acc[2 * ep + 1], pa[kk], bf[2], bf[3]);
            }
        }
        if (kt + 1 < n_kt) load_tile<T, E>(sV + (buf ^ 1) * kBN * SE, vg, k0 + kBN, KL);
        cp_async_commit();
    }

    // epilogue: O /= l (0/0 = NaN for a fully masked row, as the reference)
    float inv_l[2], lse_v[2];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        float l = l_r[rr];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        inv_l[rr] = 1.0f / l;
        lse_v[rr] = m_r[rr] + logf(l);
    }
    cp_async_wait<0>();
    __syncthreads();
#pragma unroll
    for (int et = 0; et < ET; ++et) {
        const int col = et * 8 + 2 * t4;
        *reinterpret_cast<uint32_t*>(sQ + r_lo * SE + col) = pack2<T>(o_acc[et][0] * inv_l[0], o_acc[et][1] * inv_l[0]);
        *reinterpret_cast<uint32_t*>(sQ + (r_lo + 8) * SE + col) =
            pack2<T>(o_acc[et][2] * inv_l[1], o_acc[et][3] * inv_l[1]);
    }
    __syncthreads();
    T* og = reinterpret_cast<T*>(p.o) + ((int64_t)b * p.QH + h) * QL * E;
    constexpr int CPR = E / 8;
    for (int c = threadIdx.x; c < kBM * CPR; c += kThreads) {
        const int r = c / CPR, ch = c % CPR;
        if (q0 + r < QL)
            *reinterpret_cast<uint4*>(og + (q0 + r) * E + ch * 8) = *reinterpret_cast<const uint4*>(sQ + r * SE + ch * 8);
    }
    if (t4 == 0) {
        float* lg = p.lse + ((int64_t)b * p.QH + h) * QL;
#pragma unroll
        for (int rr = 0; rr < 2; ++rr)
            if (i_row[rr] < QL) lg[i_row[rr]] = lse_v[rr];
    }
}

// ============================================================== backward
template <typename T, int E, bool CAUSAL>
__global__ void __launch_bounds__(kThreads) fa_bwd_mma_kernel(const Params p) {
    constexpr int SE = E + 8;
    constexpr int SS = kBM + 8;   // sdS row stride
    constexpr int NT = kBM / 8;   // n-tiles over the query tile
    constexpr int KS = E / 16;
    constexpr int ET = E / 8;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    T* sK = reinterpret_cast<T*>(smem_raw);
    T* sV = sK + kBN * SE;
    T* sQ = sV + kBN * SE;            // [2][kBM][SE]
    T* sdO = sQ + 2 * kBM * SE;       // [2][kBM][SE]
    T* sdS = sdO + 2 * kBM * SE;      // [kBN][SS]
    float* sLse = reinterpret_cast<float*>(sdS + kBN * SS);  // [2][kBM]
    float* sDel = sLse + 2 * kBM;                             // [2][kBM]

    const int64_t QL = p.QL, KL = p.KL;
    const int kt = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    const int64_t k0 = (int64_t)kt * kBN;
    const int QH = p.QH;

    const T* kg = reinterpret_cast<const T*>(p.k) + ((int64_t)b * p.KH + kvh) * KL * E;
    const T* vg = reinterpret_cast<const T*>(p.v) + ((int64_t)b * p.KH + kvh) * KL * E;
    const uint8_t* mg = p.kmask ? p.kmask + (int64_t)b * KL : nullptr;
    const int64_t kv_len = p.kv_len ? p.kv_len[b] : KL;

    const int n_qt = (int)((QL + kBM - 1) / kBM);
    const int qt0 = CAUSAL ? (int)(k0 / kBM) : 0;
    const int nq = (k0 < kv_len && qt0 < n_qt) ? n_qt - qt0 : 0;
    const int steps = nq * p.n_rep;

    float dk_acc[ET][4], dv_acc[ET][4];
#pragma unroll
    for (int i = 0; i < ET; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) { dk_acc[i][j] = 0.f; dv_acc[i][j] = 0.f; }

    auto issue_step = [&](int step, int buf) {
        const int hh = step / nq, qt = qt0 + step % nq;
        const int h = kvh * p.n_rep + hh;
        const int64_t q0 = (int64_t)qt * kBM;
        const T* qg = reinterpret_cast<const T*>(p.q) + ((int64_t)b * QH + h) * QL * E;
        const T* dg = reinterpret_cast<const T*>(p.dO) + ((int64_t)b * QH + h) * QL * E;
        load_tile<T, E>(sQ + buf * kBM * SE, qg, q0, QL);
        load_tile<T, E>(sdO + buf * kBM * SE, dg, q0, QL);
        if (threadIdx.x < kBM) {
            const int64_t i = q0 + threadIdx.x;
            const int64_t ro = ((int64_t)b * QH + h) * QL;
            sLse[buf * kBM + threadIdx.x] = i < QL ? p.lse[ro + i] : 0.f;
            sDel[buf * kBM + threadIdx.x] = i < QL ? p.delta[ro + i] : 0.f;
        }
    };

    if (steps > 0) {
        load_tile<T, E>(sK, kg, k0, KL);
        load_tile<T, E>(sV, vg, k0, KL);
        issue_step(0, 0);
    }
    cp_async_commit();

    const int j_lo = warp * 16 + g;   // local key rows j_lo, j_lo + 8
    const int64_t j_row[2] = {k0 + j_lo, k0 + j_lo + 8};
    bool jmask[2];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        bool ok = j_row[rr] < KL;
        if (mg) ok = ok && mg[ok ? j_row[rr] : 0] != 0;
        jmask[rr] = ok;
    }
    const float scale = p.scale;

    for (int step = 0; step < steps; ++step) {
        const int buf = step & 1;
        const int hh = step / nq, qt = qt0 + step % nq;
        const int h = kvh * p.n_rep + hh;
        const int64_t q0 = (int64_t)qt * kBM;
        if (step + 1 < steps) issue_step(step + 1, buf ^ 1);
        cp_async_commit();

        const T* pg = p.pair ? reinterpret_cast<const T*>(p.pair) + (int64_t)b * KL * QL * QH + h : nullptr;
        float pv[NT][4];
        if (pg) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int64_t j = j_row[e >> 1];
                    const int64_t i = q0 + nt * 8 + 2 * t4 + (e & 1);
                    pv[nt][e] = (i < QL && j < KL) ? to_f(pg[(j * QL + i) * QH]) : 0.f;
                }
        }
        cp_async_wait<1>();
        __syncthreads();
        const T* sQb = sQ + buf * kBM * SE;
        const T* sdOb = sdO + buf * kBM * SE;

        // S^T = K Q^T and dP^T = V dO^T  (rows: this warp's 16 keys)
        float s[NT][4], dp[NT][4];
#pragma unroll
        for (int i = 0; i < NT; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) { s[i][j] = 0.f; dp[i][j] = 0.f; }
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            uint32_t kf[4], vf[4];
            ldsm_x4(kf, sK + (warp * 16 + (lane & 15)) * SE + ks * 16 + (lane >> 4) * 8);
            ldsm_x4(vf, sV + (warp * 16 + (lane & 15)) * SE + ks * 16 + (lane >> 4) * 8);
#pragma unroll
            for (int np = 0; np < NT / 2; ++np) {
                uint32_t bq[4], bd[4];
                const int roff = (np * 16 + (lane & 7) + (lane >> 4) * 8) * SE + ks * 16 + ((lane >> 3) & 1) * 8;
                ldsm_x4(bq, sQb + roff);
                ldsm_x4(bd, sdOb + roff);
                mma16816<T>(s[2 * np], kf, bq[0], bq[1]);
                mma16816<T>(s[2 * np + 1], kf, bq[2], bq[3]);
                mma16816<T>(dp[2 * np], vf, bd[0], bd[1]);
                mma16816<T>(dp[2 * np + 1], vf, bd[2], bd[3]);
            }
        }

        // P^T = exp(S^T·scale + pair − lse), dS^T = P^T ∘ (dP^T − δ)
        T* dpg = p.dpair ? reinterpret_cast<T*>(p.dpair) + (int64_t)b * KL * QL * QH + h : nullptr;
        uint32_t pa[NT / 2][4], da[NT / 2][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float pe[4], de[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int rr = e >> 1;
                const int li = nt * 8 + 2 * t4 + (e & 1);
                const int64_t i = q0 + li;
                const int64_t j = j_row[rr];
                bool valid = jmask[rr] && i < QL;
                if (CAUSAL) valid = valid && (j <= i);
                float x = s[nt][e] * scale;
                if (pg) x += pv[nt][e];
                const float pr = valid ? exp2f((x - sLse[buf * kBM + li]) * kLog2e) : 0.f;
                const float d = pr * (dp[nt][e] - sDel[buf * kBM + li]);
                pe[e] = pr;
                de[e] = d;
                if (dpg && i < QL && j < KL) dpg[(j * QL + i) * QH] = from_f<T>(d);
            }
            pa[nt >> 1][(nt & 1) * 2 + 0] = pack2<T>(pe[0], pe[1]);
            pa[nt >> 1][(nt & 1) * 2 + 1] = pack2<T>(pe[2], pe[3]);
            da[nt >> 1][(nt & 1) * 2 + 0] = pack2<T>(de[0], de[1]);
            da[nt >> 1][(nt & 1) * 2 + 1] = pack2<T>(de[2], de[3]);
            *reinterpret_cast<uint32_t*>(sdS + j_lo * SS + nt * 8 + 2 * t4) = da[nt >> 1][(nt & 1) * 2 + 0];
            *reinterpret_cast<uint32_t*>(sdS + (j_lo + 8) * SS + nt * 8 + 2 * t4) = da[nt >> 1][(nt & 1) * 2 + 1];
        }

        // dV += P^T dO ; dK += dS^T Q
#pragma unroll
        for (int kk = 0; kk < NT / 2; ++kk) {
#pragma unroll
            for (int ep = 0; ep < ET / 2; ++ep) {
                uint32_t bd[4], bq[4];
                const int roff = (kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * SE + ep * 16 + (lane >> 4) * 8;
                ldsm_x4_t(bd, sdOb + roff);
                ldsm_x4_t(bq, sQb + roff);
                mma16816<T>(dv_acc[2 * ep], pa[kk], bd[0], bd[1]);
                mma16816<T>(dv_acc[2 * ep + 1], pa[kk], bd[2], bd[3]);
                mma16816<T>(dk_acc[2 * ep], da[kk], bq[0], bq[1]);
                mma16816<T>(dk_acc[2 * ep + 1], da[kk], bq[2], bq[3]);
            }
        }
        __syncthreads();

        // dQ[this warp's 16 queries] += dS K · scale  (fp32 atomics)
        float dq[ET][4];
#pragma unroll
        for (int i = 0; i < ET; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) dq[i][j] = 0.f;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
            uint32_t af[4];
            ldsm_x4_t(af, sdS + (kk * 16 + (lane & 7) + (lane >> 4) * 8) * SS + warp * 16 + ((lane >> 3) & 1) * 8);
#pragma unroll
            for (int ep = 0; ep < ET / 2; ++ep) {
                uint32_t bk[4];
                ldsm_x4_t(bk, sK + (kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * SE + ep * 16 + (lane >> 4) * 8);
                mma16816<T>(dq[2 * ep], af, bk[0], bk[1]);
                mma16816<T>(dq[2 * ep + 1], af, bk[2], bk[3]);
            }
        }
        float* dqg = p.dq_acc + ((int64_t)b * QH + h) * QL * E;
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const int64_t i = q0 + warp * 16 + g + rr * 8;
            if (i < QL) {
#pragma unroll
                for (int et = 0; et < ET; ++et) {
                    float* dst = dqg + i * E + et * 8 + 2 * t4;
                    atomicAdd(dst, dq[et][rr * 2] * scale);
                    atomicAdd(dst + 1, dq[et][rr * 2 + 1] * scale);
                }
            }
        }
    }
    cp_async_wait<0>();

    // write dK (·scale) and dV for this CTA's keys
    T* dkg = reinterpret_cast<T*>(p.dk) + ((int64_t)b * p.KH + kvh) * KL * E;
    T* dvg = reinterpret_cast<T*>(p.dv) + ((int64_t)b * p.KH + kvh) * KL * E;
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        const int64_t j = j_row[rr];
        if (j < KL) {
#pragma unroll
            for (int et = 0; et < ET; ++et) {
                const int col = et * 8 + 2 * t4;
                *reinterpret_cast<uint32_t*>(dkg + j * E + col) =
                    pack2<T>(dk_acc[et][rr * 2] * scale, dk_acc[et][rr * 2 + 1] * scale);
                *reinterpret_cast<uint32_t*>(dvg + j * E + col) = pack2<T>(dv_acc[et][rr * 2], dv_acc[et][rr * 2 + 1]);
            }
        }
    }
}

template <typename T, int E, bool CAUSAL>
int launch_fwd_t(const Params& p, cudaStream_t s) {
    constexpr int SE = E + 8;
    const size_t smem = (size_t)(kBM * SE + 4 * kBN * SE) * sizeof(T);
    auto kern = fa_fwd_mma_kernel<T, E, CAUSAL>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return fail(NNOP_ERR_CUDA, "flash_attention_fwd: cannot set shared memory size");
    dim3 grid((unsigned)((p.QL + kBM - 1) / kBM), p.QH, p.B);
    kern<<<grid, kThreads, smem, s>>>(p);
    return check_launch("flash_attention_fwd (mma)");
}

template <typename T, int E, bool CAUSAL>
int launch_bwd_t(const Params& p, cudaStream_t s) {
    constexpr int SE = E + 8;
    const size_t smem = (size_t)(2 * kBN * SE + 4 * kBM * SE + kBN * (kBM + 8)) * sizeof(T) + 4 * kBM * sizeof(float);
    auto kern = fa_bwd_mma_kernel<T, E, CAUSAL>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return fail(NNOP_ERR_CUDA, "flash_attention_bwd: cannot set shared memory size");
    dim3 grid((unsigned)((p.KL + kBN - 1) / kBN), p.KH, p.B);
    kern<<<grid, kThreads, smem, s>>>(p);
    return check_launch("flash_attention_bwd (mma)");
}

template <typename T, bool CAUSAL>
int dispatch_e(const Params& p, cudaStream_t s, bool bwd) {
    switch (p.E) {
        case 16: return bwd ? launch_bwd_t<T, 16, CAUSAL>(p, s) : launch_fwd_t<T, 16, CAUSAL>(p, s);
        case 32: return bwd ? launch_bwd_t<T, 32, CAUSAL>(p, s) : launch_fwd_t<T, 32, CAUSAL>(p, s);
        case 64: return bwd ? launch_bwd_t<T, 64, CAUSAL>(p, s) : launch_fwd_t<T, 64, CAUSAL>(p, s);
        case 128: return bwd ? launch_bwd_t<T, 128, CAUSAL>(p, s) : launch_fwd_t<T, 128, CAUSAL>(p, s);
        default: return fail(NNOP_ERR_SHAPE, "flash_attention: unsupported embedding dim");
    }
}

}  // namespace

template <typename T>
int mma_fwd(const Params& p, bool causal, cudaStream_t s) {
    return causal ? dispatch_e<T, true>(p, s, false) : dispatch_e<T, false>(p, s, false);
}
template <typename T>
int mma_bwd(const Params& p, bool causal, cudaStream_t s) {
    return causal ? dispatch_e<T, true>(p, s, true) : dispatch_e<T, false>(p, s, true);
}
int mma_tile() { return kBN; }

template int mma_fwd<__half>(const Params&, bool, cudaStream_t);
template int mma_fwd<__nv_bfloat16>(const Params&, bool, cudaStream_t);
template int mma_bwd<__half>(const Params&, bool, cudaStream_t);
template int mma_bwd<__nv_bfloat16>(const Params&, bool, cudaStream_t);

}  // namespace fa
}  // namespace nnop
