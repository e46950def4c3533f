// Flash-attention backward on the sm_100a tensor cores for E = 128 (bf16/f16,
// no pair bias): the GQA / RoPE workload's backward.
//
// Reference: `_flash_attention_bwd!` (src/attention_bwd.jl:1-175) -- one
// workgroup per (head, batch) walking every (key tile, query tile) pair with
// five WMMA GEMMs, a read-modify-write of dq in global memory and atomics for
// GQA.  Here one CTA owns a 128-key tile of one KV head of one batch and walks
// 64-query steps of every query head of its GQA group; dK and dV accumulate in
// TMEM for the whole walk.  Consecutive steps alternate between two
// elementwise warpgroups with their own TMEM score buffers, so one step's
// exponentials run while the tensor cores work on the other's products.
//
// TMEM (512 columns) is the binding budget at E = 128: dV and dK take 256
// columns, and each warpgroup's Sᵀ and dPᵀ buffers 64 columns each.  dQ has
// no columns of its own: the elementwise step writes the packed 16-bit Pᵀ and
// dSᵀ of each 16-query chunk back into that chunk's own Sᵀ columns (Pᵀ in the
// first 8, dSᵀ in the next 8), which frees the warpgroup's dPᵀ buffer; dQ is
// computed transposed (E on the TMEM lanes) into it.  Per step t (queries
// q0..q0+63 of head h), warpgroup w = t % 2:
//   Sᵀ  = K·Q_tᵀ              M=128 keys, N=64, K=E    UMMA ss
//   dPᵀ = V·dO_tᵀ                                       UMMA ss
//   Pᵀ  = exp2(Sᵀ·scale·log2e − lse),  dSᵀ = Pᵀ∘(dPᵀ − δ)   (elementwise)
//   dV += Pᵀ·dO_t             N=128 (E), K=64           UMMA ts (Pᵀ from TMEM)
//   dK += dSᵀ·Q_t                                       UMMA ts
//   dQᵀ = Kᵀ·dS_tᵀ            M=128 (E), N=64, K=128    UMMA ss (dS from smem)
//   dq_acc[h][q0..q0+63] += scale·dQ: the dQ warps read dQᵀ from TMEM, stage
//   fp32 [32 queries][32 E] boxes in the step's consumed dS buffer and add
//   them with TMA reduce-adds.
// The next step of the same warpgroup reuses its buffers: Sᵀ(t+2) is issued
// right behind the products of t (the tensor pipe runs one thread's UMMAs in
// order), dPᵀ(t+2) once the dQ warps have read dQᵀ(t).
// Warp roles (512 threads):
//   warp 0      TMA producer (K, V once; Q_t, dO_t into a 3-stage ring)
//   warp 1      MMA issuer (one lane)
//   warps 2-3   step provider: lse (log2 units) and δ of the step's queries
//   warps 4-7   elementwise, even steps (one key per TMEM lane)
//   warps 8-11  elementwise, odd steps
//   warps 12-15 dQ: TMEM dQᵀ -> staged fp32 boxes -> TMA reduce-add
// TMEM columns: dV [0,128), dK [128,256), warpgroup w: Sᵀ [256+128w, 320+128w),
// dPᵀ / dQᵀ [320+128w, 384+128w).
// All mbarrier waits are bounded; a wait that gives up records its site
// (0-13) in the timeout flags and the CTA leaves.
#include <cuda.h>

#include <cstdlib>
#include <cstring>

#include "fa_common.cuh"
#include "fa_sm100.cuh"
#include "sm100.cuh"

namespace nnop {
namespace fa {
namespace {

using namespace sm100;

constexpr int kBN = 128;      // keys per CTA (TMEM lanes)
constexpr int kSM = 64;       // queries per step
constexpr int kE = 128;
constexpr int kStages = 3;    // Q/dO ring
constexpr int kThreads = 512;

enum Bar {
    kKVFull = 0,
    kQFull = 1,       // +stage: Q_t and dO_t landed
    kQEmpty = 4,      // +stage: dV/dK MMAs of the step retired
    kSFull = 7,       // +warpgroup: Sᵀ, dPᵀ of its step in TMEM
    kPFull = 9,       // +warpgroup: elementwise done (128 arrivals)
    kDQFull = 11,     // +warpgroup: dQᵀ of its step in TMEM
    kDQEmpty = 13,    // +warpgroup: dQ warps read dQᵀ (128 arrivals)
    kDSEmpty = 15,    // +warpgroup: dQ staging done with the dS buffer (4 arrivals)
    kTileFull = 17,   // +warpgroup: provider -> elementwise (64 arrivals)
    kTileEmpty = 19,  // +warpgroup: elementwise -> provider (128 arrivals)
    kFinal = 21,      // every MMA retired
    kNumBars = 22
};

struct Lay {
    static constexpr int kKV = kBN * kE * 2;       // K or V: two [128 keys][64 E] SW128 boxes, 32 KB
    static constexpr int kStep = kSM * kE * 2;     // Q_t or dO_t: two [64 q][64 E] boxes, 16 KB
    static constexpr int kK = 0;
    static constexpr int kV = kK + kKV;
    static constexpr int kQ = kV + kKV;                    // kStages x 16 KB
    static constexpr int kDO = kQ + kStages * kStep;       // kStages x 16 KB
    static constexpr int kDS = kDO + kStages * kStep;      // 2 x [128 keys][64 q] MN-major SW128, 16 KB each
    static constexpr int kDSBytes = kBN * kSM * 2;
    static constexpr int kLse = kDS + 2 * kDSBytes;        // [2][64] float (log2 units)
    static constexpr int kDel = kLse + 2 * kSM * 4;        // [2][64] float
    static constexpr int kBar = kDel + 2 * kSM * 4;
    static constexpr int kTmemSlot = kBar + kNumBars * 8;
    static constexpr int kTotal = kTmemSlot + 16;
    static constexpr int kAlloc = kTotal + 1024;
};
static_assert(Lay::kAlloc <= 227 * 1024, "shared memory");
static_assert(Lay::kDSBytes == 4 * 4 * 32 * 32, "dQ staging: 4 warps x one [32][32] fp32 box per round");

template <typename T, bool CAUSAL, bool MASK>
__global__ void __launch_bounds__(kThreads, 1)
fa_bwd128_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_dq, const Params p) {
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Lay::kBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Lay::kTmemSlot);
    float* sLse = reinterpret_cast<float*>(smem + Lay::kLse);
    float* sDel = reinterpret_cast<float*>(smem + Lay::kDel);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t QL = p.QL, KL = p.KL;
    const int QH = p.QH;
    const int kt = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int64_t k0 = (int64_t)kt * kBN;
    const int64_t kv_len = p.kv_len ? p.kv_len[b] : KL;
    const int n_qs = (int)((QL + kSM - 1) / kSM);
    // causal: queries before k0 see none of this CTA's keys (key j visible to query i iff j <= i)
    const int qs0 = CAUSAL ? (int)(k0 / kSM) : 0;
    const int nq = (k0 < kv_len && qs0 < n_qs) ? n_qs - qs0 : 0;
    const int steps = nq * p.n_rep;

    __shared__ int s_abort;   // set by the first wait of this CTA that gives up
    volatile int* ab = &s_abort;
    if (threadIdx.x == 0) {
        s_abort = 0;
        mbar_init(&bars[kKVFull], 1);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars[kQFull + s], 1);
            mbar_init(&bars[kQEmpty + s], 1);
        }
        for (int w = 0; w < 2; ++w) {
            mbar_init(&bars[kSFull + w], 1);
            mbar_init(&bars[kPFull + w], 128);
            mbar_init(&bars[kDQFull + w], 1);
            mbar_init(&bars[kDQEmpty + w], 128);
            mbar_init(&bars[kDSEmpty + w], 4);
            mbar_init(&bars[kTileFull + w], 64);
            mbar_init(&bars[kTileEmpty + w], 128);
        }
        mbar_init(&bars[kFinal], 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tDV = tmem, tDK = tmem + 128;
    // step t's head and first query
    auto step_head = [&](int t) { return kvh * p.n_rep + t / nq; };
    auto step_q0 = [&](int t) { return (qs0 + t % nq) * kSM; };

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0 && steps > 0) {
            tma_prefetch(&tm_q);
            tma_prefetch(&tm_k);
            tma_prefetch(&tm_v);
            tma_prefetch(&tm_do);
            const int bh_k = b * p.KH + kvh;
            mbar_expect_tx(&bars[kKVFull], 2 * Lay::kKV);
#pragma unroll
            for (int e2 = 0; e2 < 2; ++e2) {
                tma_load_3d(smem + Lay::kK + e2 * (Lay::kKV / 2), &tm_k, &bars[kKVFull], e2 * 64, (int)k0, bh_k);
                tma_load_3d(smem + Lay::kV + e2 * (Lay::kKV / 2), &tm_v, &bars[kKVFull], e2 * 64, (int)k0, bh_k);
            }
            int issued = 0;
            for (int t = 0; t < steps; ++t) {
                const int s = t % kStages;
                if (t >= kStages && !wait(&bars[kQEmpty + s], ((t / kStages) - 1) & 1, ab, 0)) break;
                const int bh = b * QH + step_head(t), q0 = step_q0(t);
                mbar_expect_tx(&bars[kQFull + s], 2 * Lay::kStep);
#pragma unroll
                for (int e2 = 0; e2 < 2; ++e2) {
                    tma_load_3d(smem + Lay::kQ + s * Lay::kStep + e2 * (Lay::kStep / 2), &tm_q, &bars[kQFull + s],
                                e2 * 64, q0, bh);
                    tma_load_3d(smem + Lay::kDO + s * Lay::kStep + e2 * (Lay::kStep / 2), &tm_do,
                                &bars[kQFull + s], e2 * 64, q0, bh);
                }
                issued = t + 1;
            }
            // copies in flight land before the CTA leaves (bounded waits)
            wait(&bars[kKVFull], 0, ab, 1);
            for (int t = issued - kStages < 0 ? 0 : issued - kStages; t < issued; ++t)
                wait(&bars[kQFull + t % kStages], (t / kStages) & 1, ab, 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        constexpr uint32_t id_s = idesc_f16<kBF16>(128, kSM, false, false);   // Sᵀ, dPᵀ
        constexpr uint32_t id_kv = idesc_f16<kBF16>(128, kE, false, true);    // dV, dK (A in TMEM)
        constexpr uint32_t id_q = idesc_f16<kBF16>(128, kSM, true, true);     // dQᵀ (A = Kᵀ, B = dS)
        const uint32_t sK = smem_u32(smem + Lay::kK), sV = smem_u32(smem + Lay::kV);
        auto sQ = [&](int t) { return smem_u32(smem + Lay::kQ + (t % kStages) * Lay::kStep); };
        auto sDO = [&](int t) { return smem_u32(smem + Lay::kDO + (t % kStages) * Lay::kStep); };
        // operand descriptors, built once and stepped with desc_add
        const uint64_t dKk = desc_k_sw128(sK), dVk = desc_k_sw128(sV);
        const uint64_t dQk = desc_k_sw128(sQ(0)), dDOk = desc_k_sw128(sDO(0));
        const uint64_t dQmn = desc_mn_sw128(sQ(0), Lay::kStep / 2), dDOmn = desc_mn_sw128(sDO(0), Lay::kStep / 2);
        const uint64_t dKmn = desc_mn_sw128(sK, Lay::kKV / 2);
        const uint64_t dDSmn = desc_mn_sw128(smem_u32(smem + Lay::kDS), 0);
        // K-major SW128 operands stored as two 64-column boxes: K16 step kk of E
        auto kmaj = [](int box_bytes, int kk) { return (uint32_t)((kk >> 2) * box_bytes + (kk & 3) * 32); };
        auto issue_score = [&](int t, bool dp) {   // Sᵀ (or dPᵀ) of step t, lane 0 only
            const int w = t & 1;
            const uint32_t d = tmem + 256 + 128 * w + (dp ? 64 : 0);
            const uint64_t a = dp ? dVk : dKk;
            const uint64_t bq = desc_add(dp ? dDOk : dQk, (uint32_t)(t % kStages) * Lay::kStep);
#pragma unroll
            for (int kk = 0; kk < kE / 16; ++kk)
                umma_ss(d, desc_add(a, kmaj(Lay::kKV / 2, kk)), desc_add(bq, kmaj(Lay::kStep / 2, kk)), id_s,
                        kk > 0 ? 1u : 0u);
        };
        bool ok = steps > 0 && wait_warp(&bars[kKVFull], 0, ab, 2);
        for (int t = 0; ok && t < 2 && t < steps; ++t) {
            if (!wait_warp(&bars[kQFull + t % kStages], (t / kStages) & 1, ab, 3)) { ok = false; break; }
            tc_fence_after();
            if (lane == 0) {
                issue_score(t, false);
                issue_score(t, true);
                umma_commit(&bars[kSFull + (t & 1)]);
            }
            __syncwarp();
        }
        for (int t = 0; ok && t < steps; ++t) {
            const int w = t & 1;
            const uint32_t tSw = tmem + 256 + 128 * w, tDPw = tSw + 64;
            if (!wait_warp(&bars[kPFull + w], (t >> 1) & 1, ab, 4)) break;
            tc_fence_after();
            if (lane == 0) {
                // products of step t: Pᵀ / dSᵀ of query chunk kk at Sᵀ columns 16kk / 16kk + 8
                const uint32_t qoff = (uint32_t)(t % kStages) * Lay::kStep;
                const uint64_t bdo = desc_add(dDOmn, qoff), bq = desc_add(dQmn, qoff);
                const uint32_t acc0 = t > 0 ? 1u : 0u;
#pragma unroll
                for (int kk = 0; kk < kSM / 16; ++kk) {
                    const uint32_t acc = kk > 0 ? 1u : acc0;
                    umma_ts(tDV, tSw + 16 * kk, desc_add(bdo, kk * 16 * 128), id_kv, acc);
                    umma_ts(tDK, tSw + 16 * kk + 8, desc_add(bq, kk * 16 * 128), id_kv, acc);
                }
                umma_commit(&bars[kQEmpty + t % kStages]);
                // dQᵀ = Kᵀ·dSᵀ into the warpgroup's dPᵀ columns (read out by the elementwise step)
                const uint64_t bds = desc_add(dDSmn, (uint32_t)w * Lay::kDSBytes);
#pragma unroll
                for (int kk = 0; kk < kBN / 16; ++kk)
                    umma_ss(tDPw, desc_add(dKmn, kk * 16 * 128), desc_add(bds, kk * 16 * 128), id_q, kk > 0 ? 1u : 0u);
                umma_commit(&bars[kDQFull + w]);
            }
            __syncwarp();
            if (t + 2 < steps) {
                // Sᵀ(t+2) overwrites Pᵀ/dSᵀ(t) only after the products above read
                // them (one thread's UMMAs run in order); dPᵀ(t+2) waits for the
                // dQ warps to have read dQᵀ(t) out of those columns.
                if (!wait_warp(&bars[kQFull + (t + 2) % kStages], ((t + 2) / kStages) & 1, ab, 5)) break;
                tc_fence_after();
                if (lane == 0) issue_score(t + 2, false);
                __syncwarp();
                if (!wait_warp(&bars[kDQEmpty + w], (t >> 1) & 1, ab, 6)) break;
                tc_fence_after();
                if (lane == 0) {
                    issue_score(t + 2, true);
                    umma_commit(&bars[kSFull + w]);
                }
                __syncwarp();
            }
        }
        // every MMA this warp issued retires before TMEM is read out / freed
        if (lane == 0) umma_commit(&bars[kFinal]);
        __syncwarp();
        wait(&bars[kFinal], 0, ab, 7);
    } else if (warp < 4) {
        // ------------------------------------------------------ step provider
        const int u = threadIdx.x - 64;   // one query of the step
        for (int t = 0; t < steps; ++t) {
            const int w = t & 1;
            if (t >= 2 && !wait(&bars[kTileEmpty + w], ((t >> 1) - 1) & 1, ab, 8)) break;
            const int64_t i = step_q0(t) + u;
            const int64_t ro = ((int64_t)b * QH + step_head(t)) * QL;
            sLse[w * kSM + u] = i < QL ? p.lse[ro + i] * kLog2e : 0.f;
            sDel[w * kSM + u] = i < QL ? p.delta[ro + i] : 0.f;
            mbar_arrive(&bars[kTileFull + w]);
        }
    } else if (warp < 12) {
        // ------------------------------------------------------ elementwise
        const int jr = (threadIdx.x - 128) & 127;            // key row = TMEM lane
        const int w = (threadIdx.x - 128) >> 7;              // warpgroup: steps t % 2 == w
        const int64_t j = k0 + jr;
        bool key_ok = j < KL;
        if (MASK && key_ok) key_ok = p.kmask[(int64_t)b * KL + j] != 0;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tSw = tmem + 256 + 128 * w + lane_off, tDPw = tSw + 64;
        const float sl2 = p.scale * kLog2e;
        const uint32_t pw[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
        uint8_t* sDS = smem + Lay::kDS + w * Lay::kDSBytes + jr * 128;
        const float* lse_w = sLse + w * kSM;
        const float* del_w = sDel + w * kSM;
        for (int t = w; t < steps; t += 2) {
            const int n = t >> 1;   // this warpgroup's n-th step
            const int64_t q0 = step_q0(t);
            if (!wait_warp(&bars[kTileFull + w], n & 1, ab, 9)) break;
            if (!wait_warp(&bars[kSFull + w], n & 1, ab, 10)) break;
            if (n >= 1 && !wait_warp(&bars[kDSEmpty + w], (n - 1) & 1, ab, 11)) break;
            tc_fence_after();
            // valid query columns of this key within the step: [cmin, cmax)
            const int64_t nvq = QL - q0;
            const int cmax = key_ok ? (int)(nvq < kSM ? (nvq > 0 ? nvq : 0) : kSM) : 0;
            const int64_t cm = CAUSAL ? j - q0 : 0;
            const int cmin = (int)(cm < 0 ? 0 : (cm > kSM ? kSM : cm));
#pragma unroll 1
            for (int cc = 0; cc < kSM / 16; ++cc) {
                const int col = cc * 16;
                uint32_t sr[16], dr[16];
                tmem_ld16(tSw + col, sr);
                tmem_ld16(tDPw + col, dr);
                float4 l4[4], d4[4];
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    l4[v] = reinterpret_cast<const float4*>(lse_w + col)[v];
                    d4[v] = reinterpret_cast<const float4*>(del_w + col)[v];
                }
                tmem_ld_wait();
                uint32_t pk[8], dk[8];
                const int lo = cmin - col, hi = cmax - col;
                if (lo <= 0 && hi >= 16)
                    elementwise16<T, false, false>(sr, dr, pw, l4, d4, sl2, 0, 16, pk, dk);
                else
                    elementwise16<T, false, true>(sr, dr, pw, l4, d4, sl2, lo, hi, pk, dk);
                // packed Pᵀ and dSᵀ into this chunk's own Sᵀ columns (already read)
                tmem_st8(tSw + col, pk);
                tmem_st8(tSw + col + 8, dk);
                // dS (16-bit) into shared memory for the dQ MMA: row jr, queries
                // col..col+15, canonical MN-major 128-byte swizzle
#pragma unroll
                for (int v = 0; v < 2; ++v) {
                    const int chunk = cc * 2 + v;
                    *reinterpret_cast<uint4*>(sDS + ((chunk ^ (jr & 7)) << 4)) =
                        make_uint4(dk[4 * v], dk[4 * v + 1], dk[4 * v + 2], dk[4 * v + 3]);
                }
            }
            mbar_arrive(&bars[kTileEmpty + w]);
            tmem_st_wait();
            fence_proxy_async_smem();   // dS smem writes -> tensor-core (async proxy) reads
            tc_fence_before();
            mbar_arrive(&bars[kPFull + w]);
        }
        // epilogue: dK (warpgroup 0) and dV (warpgroup 1) rows of this CTA's keys
        if (wait_warp(&bars[kFinal], 0, ab, 12)) {
            tc_fence_after();
            const bool is_dk = w == 0;
            const uint32_t src = (is_dk ? tDK : tDV) + lane_off;
            T* dst = reinterpret_cast<T*>(is_dk ? p.dk : p.dv) + (((int64_t)b * p.KH + kvh) * KL + j) * kE;
            const float mul = is_dk ? p.scale : 1.f;
            if (is_dk && p.rope_cos != nullptr) {
                // fused RoPE backward: dk of the un-rotated k, pairs (e, e + 64)
                // rotated by cos/sin of index e at position j (sin → −sin)
                const int64_t tr = ((p.rope_cb == 1 ? 0 : (int64_t)b) * KL + (j < KL ? j : 0)) * kE;
#pragma unroll 1
                for (int c = 0; c < 2; ++c) {
                    uint32_t ra[32], rb[32];
                    tmem_ld32(src + c * 32, ra);
                    tmem_ld32(src + 64 + c * 32, rb);
                    tmem_ld_wait();
                    if (j < KL) {
                        float4 cw[8], sw[8];   // cos/sin of indices 32c .. 32c+31 at position j
#pragma unroll
                        for (int v = 0; v < 8; ++v) {
                            cw[v] = __ldg(reinterpret_cast<const float4*>(p.rope_cos + tr + 32 * c) + v);
                            sw[v] = __ldg(reinterpret_cast<const float4*>(p.rope_sin + tr + 32 * c) + v);
                        }
                        uint32_t pa[16], pb[16];
#pragma unroll
                        for (int u = 0; u < 32; u += 2) {
                            float oa[2], ob[2];
#pragma unroll
                            for (int v = 0; v < 2; ++v) {
                                const float a = steps > 0 ? __uint_as_float(ra[u + v]) * mul : 0.f;
                                const float bb = steps > 0 ? __uint_as_float(rb[u + v]) * mul : 0.f;
                                const float cs = reinterpret_cast<const float*>(cw)[u + v];
                                const float sn = reinterpret_cast<const float*>(sw)[u + v];
                                oa[v] = a * cs + bb * sn;
                                ob[v] = bb * cs - a * sn;
                            }
                            pa[u >> 1] = pack16<T>(oa[0], oa[1]);
                            pb[u >> 1] = pack16<T>(ob[0], ob[1]);
                        }
                        uint4* da = reinterpret_cast<uint4*>(dst + c * 32);
                        uint4* db = reinterpret_cast<uint4*>(dst + 64 + c * 32);
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            da[v] = make_uint4(pa[4 * v], pa[4 * v + 1], pa[4 * v + 2], pa[4 * v + 3]);
                            db[v] = make_uint4(pb[4 * v], pb[4 * v + 1], pb[4 * v + 2], pb[4 * v + 3]);
                        }
                    }
                }
            } else {
#pragma unroll 1
                for (int c = 0; c < kE / 32; ++c) {
                    uint32_t raw[32];
                    tmem_ld32(src + c * 32, raw);
                    tmem_ld_wait();
                    if (j < KL) {
                        uint32_t pk[16];
#pragma unroll
                        for (int u = 0; u < 16; ++u)
                            pk[u] = steps > 0 ? pack16<T>(__uint_as_float(raw[2 * u]) * mul,
                                                          __uint_as_float(raw[2 * u + 1]) * mul)
                                              : 0u;
                        uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
                        for (int v = 0; v < 4; ++v)
                            d4[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
                    }
                }
            }
        }
    } else {
        // ------------------------------------------------------ dQ reductions
        // warp wi: E columns 32wi..32wi+31 of dQᵀ (TMEM lanes); thread = one E
        // column, 64 query values.  Two passes of one [32 queries][32 E] fp32
        // box per warp (128-byte swizzle) staged in the step's consumed dS
        // buffer, each added to dq_acc with one TMA reduce-add (rows past QL
        // are clipped by the tensor map).
        const int wi = warp & 3;
        const uint32_t lane_off = (uint32_t)(wi * 32) << 16;
        for (int t = 0; t < steps; ++t) {
            const int w = t & 1, n = t >> 1;
            const int bh = b * QH + step_head(t), q0 = step_q0(t);
            if (!wait_warp(&bars[kDQFull + w], n & 1, ab, 13)) break;
            tc_fence_after();
            const uint32_t src = tmem + 256 + 128 * w + 64 + lane_off;
            uint32_t raw[2][32];
            tmem_ld32(src, raw[0]);
            tmem_ld32(src + 32, raw[1]);
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(&bars[kDQEmpty + w]);   // the dPᵀ columns may be overwritten
            uint8_t* stg = smem + Lay::kDS + w * Lay::kDSBytes + wi * 4096;
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (r == 1 && lane == 0) bulk_wait_read<0>();   // the first box has been read
                __syncwarp();
#pragma unroll
                for (int qq = 0; qq < 32; ++qq)
                    *reinterpret_cast<float*>(stg + qq * 128 + (((lane >> 2) ^ (qq & 7)) << 4) + (lane & 3) * 4) =
                        __uint_as_float(raw[r][qq]) * p.scale;
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_reduce_add_3d(&tm_dq, stg, 32 * wi, q0 + 32 * r, bh);
                    bulk_commit();
                }
            }
            if (lane == 0) {
                bulk_wait_read<0>();
                mbar_arrive(&bars[kDSEmpty + w]);
            }
            __syncwarp();
        }
        if (lane == 0) bulk_wait<0>();   // reductions land before the CTA exits
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// 3-D map over the fp32 dQ accumulator [B·QH][QL][128], box (32, 32, 1),
// 128-byte swizzle (the dQ warps' staging layout).
bool make_dq128_map(CUtensorMap* m, float* base, int64_t QL, int64_t bh) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)kE, (cuuint64_t)QL, (cuuint64_t)bh};
    cuuint64_t strides[2] = {(cuuint64_t)kE * 4, (cuuint64_t)QL * kE * 4};
    cuuint32_t box[3] = {32, 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <typename T, bool CAUSAL, bool MASK>
int launch(const Params& p, cudaStream_t s) {
    constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
    CUtensorMap tq, tk, tv, tdo, tdq;
    if (!make_map(&tq, p.q, kE, p.QL, (int64_t)p.B * p.QH, kSM, bf16) ||
        !make_map(&tk, p.k, kE, p.KL, (int64_t)p.B * p.KH, kBN, bf16) ||
        !make_map(&tv, p.v, kE, p.KL, (int64_t)p.B * p.KH, kBN, bf16) ||
        !make_map(&tdo, p.dO, kE, p.QL, (int64_t)p.B * p.QH, kSM, bf16) ||
        !make_dq128_map(&tdq, p.dq_acc, p.QL, (int64_t)p.B * p.QH))
        return fail(NNOP_ERR_CUDA, "flash_attention_bwd: cuTensorMapEncodeTiled failed");
    auto kern = fa_bwd128_sm100_kernel<T, CAUSAL, MASK>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kAlloc) != cudaSuccess)
        return fail(NNOP_ERR_CUDA, "flash_attention_bwd: cannot set shared memory size");
    dim3 grid((unsigned)((p.KL + kBN - 1) / kBN), p.KH, p.B);
    kern<<<grid, kThreads, Lay::kAlloc, s>>>(tq, tk, tv, tdo, tdq, p);
    return check_launch("flash_attention_bwd (sm100, E=128)");
}

template <typename T>
int dispatch(const Params& p, bool causal, cudaStream_t s) {
    const bool mask = p.kmask != nullptr;
    if (causal) return mask ? launch<T, true, true>(p, s) : launch<T, true, false>(p, s);
    return mask ? launch<T, false, true>(p, s) : launch<T, false, false>(p, s);
}

}  // namespace

// Reads and clears the bounded-wait timeout flags of this file's kernel.
int sm100_bwd128_timeouts() {
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, sm100::g_wait_timeout, sizeof(int));
    cudaMemcpyToSymbol(sm100::g_wait_timeout, &z, sizeof(int));
    return v;
}

int sm100_bwd128(const Params& p, int dtype, bool causal, cudaStream_t s) {
    return dtype == NNOP_BF16 ? dispatch<__nv_bfloat16>(p, causal, s) : dispatch<__half>(p, causal, s);
}

}  // namespace fa
}  // namespace nnop
