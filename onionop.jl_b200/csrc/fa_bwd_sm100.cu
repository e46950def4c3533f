// Flash-attention backward on the sm_100a tensor cores (tcgen05 UMMA, TMEM
// accumulators, TMA-fed tiles), bf16/f16, E = 64.
//
// Reference: `_flash_attention_bwd!` (src/attention_bwd.jl:1-175) -- one
// workgroup per (head, batch) walking every (key tile, query tile) pair with
// five WMMA/SIMT GEMMs, a read-modify-write of dq in global memory and atomics
// for GQA.  Here one CTA owns a 128-key tile of one KV head of one batch and
// walks the 128-query tiles of every query head of its GQA group; dK and dV
// stay in TMEM for the whole walk.  Each query tile is processed as two
// 64-query halves, half hf by elementwise warpgroup hf, each with its own
// TMEM score buffers, so the tensor cores work on one half while the other
// half's exponentials run.  Per tile t and half hf:
//   Sᵀ  = K·Q_hfᵀ              (keys on TMEM lanes)     UMMA ts (K from TMEM)
//   dPᵀ = V·dO_hfᵀ                                       UMMA ts (V from TMEM)
//   Pᵀ  = exp(Sᵀ·scale + pairᵀ − lse),  dSᵀ = Pᵀ∘(dPᵀ − δ)   (elementwise)
//   dV += Pᵀ·dO_hf   (Pᵀ from TMEM)                      UMMA ts
//   dK += dSᵀ·Q_hf   (dSᵀ from TMEM)                     UMMA ts
// and per tile: dQ_t = dS·K (dS from shared memory, MN-major, double
// buffered so the next tile's dS can be written meanwhile), then
// dq_acc[t] += scale·dQ_t: the dQ warps stage the fp32 rows in the tile's
// consumed dS buffer (128-byte swizzle) and add them with TMA reduce-adds.
//   dpair[j, i] = dSᵀ (the reference's dpair = dS/scale with its dS ∘ scale),
//                 written per head as key-major dS tiles, see pair_tiles.cu
//                 (through the per-head entry points: straight into the
//                 caller's [B·H][KL][QL] dpair): the MMA warp stores each
//                 finished dS half from shared memory with one TMA store (the
//                 buffer's layout is the tile's box).
// The pair bias is read in the elementwise step from the key-major per-head
// copy pair_tiles() writes: each half tile [128 keys][64 queries] is one TMA
// box (128-byte swizzle), so a thread reads its key's 16 queries as two
// conflict-free 16-byte vectors.  Half tiles rotate through a 4-slot ring (the
// fourth slot is V's shared tile, free once V is in TMEM), so the next tile's
// halves are in flight while the current ones are read.
// Warp roles (512 threads):
//   warp 0      TMA producer (K, V once; Q_t, dO_t into a 2-stage ring; the
//               pair half tiles of (query tile, key tile, head))
//   warp 1      MMA issuer (one lane)
//   warps 2-3   tile provider: lse (log2 units) and δ of the tile's queries
//   warps 4-7   elementwise, query half 0 (one key per TMEM lane)
//   warps 8-11  elementwise, query half 1
//   warps 12-15 dQ: TMEM dQ rows -> staged fp32 boxes -> TMA reduce-add;
//               with a per-head dpair, warp 12 first writes its zeros
// TMEM columns: Sᵀ half 0 [0,64), half 1 [64,128), dPᵀ half 0 [128,192),
// half 1 [192,256), dV [256,320), dK [320,384), dQ [384,448), K [448,480),
// V [480,512) (16-bit pairs).  The 16-bit Pᵀ / dSᵀ of a half overwrite the
// first 32 columns of its own score buffers.  K and V, constant for the whole
// walk, are copied into TMEM once (the elementwise threads move their key's
// row from the TMA-loaded shared tile) so the score MMAs read only Q / dO from
// shared memory: an N = 64 UMMA with both operands in shared memory needs the
// full shared-memory bandwidth (6 KB per 48 cycles) and slows down with every
// other shared-memory user (TMA fills, dS and dQ staging, pair reads); with A
// from TMEM it reads 2 KB.
// All mbarrier waits are bounded; a wait that gives up records its site
// (0-16) in the timeout flags and the CTA leaves.
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

constexpr int kBN = 128;   // keys per CTA (TMEM lanes)
constexpr int kBM = 128;   // queries per tile
constexpr int kHM = 64;    // queries per half
constexpr int kE = 64;
constexpr int kThreads = 512;
constexpr int kPairSlots = 4;   // pair half tiles in flight: 3 slots + V's tile once V is in TMEM

enum Bar {
    kKVFull = 0,
    kQFull = 1,       // +stage: Q_t and dO_t landed
    kQEmpty = 3,      // +stage: dV/dK MMAs of the tile retired
    kSFull = 5,       // +half: Sᵀ, dPᵀ of the half in TMEM
    kPFull = 7,       // +half: elementwise done with the half (128 arrivals)
    kDSEmpty = 9,     // +buffer: dQ staging done with the dS buffer (4 arrivals)
    kDQFull = 11,     // dQ_t in TMEM
    kDQEmpty = 12,    // dQ warps done with TMEM dQ (128 arrivals)
    kTileFull = 13,   // +buffer: provider -> elementwise (64 arrivals)
    kTileEmpty = 15,  // +buffer: elementwise -> provider (256 arrivals)
    kFinal = 17,      // every MMA retired
    kPairFull = 18,   // +slot: pair half tile landed (TMA)
    kPairEmpty = 22,  // +slot: its warpgroup is done with it (128 arrivals)
    kKVTmem = 26,     // K and V copied into TMEM (256 arrivals)
    kNumBars = 27
};

struct Lay {
    static constexpr int kTile = 128 * 64 * 2;      // one [128][64] 16-bit tile, 16 KB
    static constexpr int kK = 0;
    static constexpr int kV = kK + kTile;
    static constexpr int kQ = kV + kTile;           // 2 stages
    static constexpr int kDO = kQ + 2 * kTile;      // 2 stages
    static constexpr int kDS = kDO + 2 * kTile;     // 2 buffers of [2 halves][128 keys][64 queries], MN-major SW128
    static constexpr int kDSBytes = 2 * kTile;
    static constexpr int kPair = kDS + 2 * kDSBytes;   // 3 slots of [BN keys][64 queries] SW128
    static constexpr int kPairSlot = kBN * kHM * 2;
    static constexpr int kLse = kPair + 3 * kPairSlot;  // [2][BM] float (log2 units)
    static constexpr int kDel = kLse + 2 * kBM * 4;     // [2][BM] float
    static constexpr int kZero = kDel + 2 * kBM * 4;    // 4 KB of zeros (per-head dpair fill)
    static constexpr int kZeroBytes = 4096;
    static constexpr int kBar = kZero + kZeroBytes;
    static constexpr int kTmemSlot = kBar + kNumBars * 8;
    static constexpr int kTotal = kTmemSlot + 16;
    static constexpr int kAlloc = kTotal + 1024;
};
static_assert(Lay::kAlloc <= 227 * 1024, "shared memory");

template <typename T, bool CAUSAL, bool PAIR, bool MASK>
__global__ void __launch_bounds__(kThreads, 1)
fa_bwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_pair, const __grid_constant__ CUtensorMap tm_ds,
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
    const int n_qt = (int)((QL + kBM - 1) / kBM);
    const int qt0 = CAUSAL ? (int)(k0 / kBM) : 0;
    const int nq = (k0 < kv_len && qt0 < n_qt) ? n_qt - qt0 : 0;
    const int tiles = nq * p.n_rep;

    __shared__ int s_abort;   // set by the first wait of this CTA that gives up
    volatile int* ab = &s_abort;
    if (threadIdx.x == 0) {
        s_abort = 0;
        mbar_init(&bars[kKVFull], 1);
        mbar_init(&bars[kKVTmem], 256);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&bars[kQFull + s], 1);
            mbar_init(&bars[kQEmpty + s], 1);
            mbar_init(&bars[kSFull + s], 1);
            mbar_init(&bars[kPFull + s], 128);
            mbar_init(&bars[kDSEmpty + s], 4);
            mbar_init(&bars[kTileFull + s], 64);
            mbar_init(&bars[kTileEmpty + s], 256);
        }
        mbar_init(&bars[kDQFull], 1);
        mbar_init(&bars[kDQEmpty], 128);
        mbar_init(&bars[kFinal], 1);
        for (int s = 0; s < kPairSlots; ++s) {
            mbar_init(&bars[kPairFull + s], 1);
            mbar_init(&bars[kPairEmpty + s], 128);
        }
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
    const uint32_t tS = tmem, tDP = tmem + 128, tDV = tmem + 256, tDK = tmem + 320, tDQ = tmem + 384;
    const uint32_t tK = tmem + 448, tV = tmem + 480;
    // pair slot n: three slots of their own, the fourth is V's shared tile
    // (free once V is in TMEM)
    auto pair_slot = [&](int slot) { return smem + (slot < 3 ? Lay::kPair + slot * Lay::kPairSlot : Lay::kV); };
    // pair half tile n = 2t + hf into slot n % 4 once half tile n - 4 is
    // consumed; slot 3 (V's tile) only after V is in TMEM.  The producer
    // issues them after each tile's Q/dO, in step with the tiles (a thread of
    // its own running ahead measured no faster, and slower with the caller's
    // per-head bias, whose scattered 128-byte rows compete with the dpair
    // stores).  With that order the PairEmpty waits never wait: the products
    // of tile t-2, which the QEmpty wait before tile t's loads follows, come
    // after the elementwise reads of the slots' previous half tiles.
    auto load_pair = [&](int n) -> bool {
        const int slot = n % kPairSlots;
        if (n >= kPairSlots && !wait(&bars[kPairEmpty + slot], ((n / kPairSlots) - 1) & 1, ab, 1)) return false;
        if (n == 3 && !wait(&bars[kKVTmem], 0, ab, 1)) return false;
        const int t = n >> 1, hf = n & 1;
        const int h = kvh * p.n_rep + t / nq;
        const int q0 = (qt0 + t % nq) * kBM;
        mbar_expect_tx(&bars[kPairFull + slot], Lay::kPairSlot);
        if (p.pair_per_head)   // [B·H][KL][QL]
            tma_load_3d(pair_slot(slot), &tm_pair, &bars[kPairFull + slot], q0 + hf * kHM, (int)k0, b * QH + h);
        else                   // per-head tiles [B·H][QLp/128][KLp][128]
            tma_load_4d(pair_slot(slot), &tm_pair, &bars[kPairFull + slot], hf * kHM, (int)k0, q0 / kBM, b * QH + h);
        return true;
    };
    auto drain_pairs = [&](int issued) {   // copies in flight land before the CTA leaves
        for (int n = issued - kPairSlots < 0 ? 0 : issued - kPairSlots; n < issued; ++n)
            wait(&bars[kPairFull + n % kPairSlots], (n / kPairSlots) & 1, ab, 2);
    };

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0 && tiles > 0) {
            tma_prefetch(&tm_q);
            tma_prefetch(&tm_k);
            tma_prefetch(&tm_v);
            tma_prefetch(&tm_do);
            if (PAIR) tma_prefetch(&tm_pair);
            const int bh_k = b * p.KH + kvh;
            mbar_expect_tx(&bars[kKVFull], 2 * Lay::kTile);
            tma_load_3d(smem + Lay::kK, &tm_k, &bars[kKVFull], 0, (int)k0, bh_k);
            tma_load_3d(smem + Lay::kV, &tm_v, &bars[kKVFull], 0, (int)k0, bh_k);
            int issued = 0, pair_issued = 0;
            bool run = true;
            for (int t = 0; run && t < tiles; ++t) {
                const int s = t & 1;
                if (t >= 2 && !wait(&bars[kQEmpty + s], ((t >> 1) - 1) & 1, ab, 0)) break;
                const int h = kvh * p.n_rep + t / nq;
                const int q0 = (qt0 + t % nq) * kBM;
                mbar_expect_tx(&bars[kQFull + s], 2 * Lay::kTile);
                tma_load_3d(smem + Lay::kQ + s * Lay::kTile, &tm_q, &bars[kQFull + s], 0, q0, b * QH + h);
                tma_load_3d(smem + Lay::kDO + s * Lay::kTile, &tm_do, &bars[kQFull + s], 0, q0, b * QH + h);
                issued = t + 1;
                for (int hf = 0; PAIR && run && hf < 2; ++hf) {
                    run = load_pair(2 * t + hf);
                    if (run) pair_issued = 2 * t + hf + 1;
                }
            }
            // copies in flight land before the CTA leaves (bounded waits)
            wait(&bars[kKVFull], 0, ab, 2);
            for (int t = issued - 2 < 0 ? 0 : issued - 2; t < issued; ++t)
                wait(&bars[kQFull + (t & 1)], (t >> 1) & 1, ab, 2);
            if (PAIR) drain_pairs(pair_issued);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        constexpr uint32_t id_s = idesc_f16<kBF16>(128, kHM, false, false);   // Sᵀ, dPᵀ of a half
        constexpr uint32_t id_kv = idesc_f16<kBF16>(128, kE, false, true);    // dV, dK (A in TMEM)
        constexpr uint32_t id_q = idesc_f16<kBF16>(128, kE, true, true);      // dQ (A = dS, MN-major)
        const uint32_t sK = smem_u32(smem + Lay::kK), sV = smem_u32(smem + Lay::kV);
        const uint64_t dKmn = desc_mn_sw128(sK, 0);
        const uint64_t dQk = desc_k_sw128(smem_u32(smem + Lay::kQ)), dDOk = desc_k_sw128(smem_u32(smem + Lay::kDO));
        const uint64_t dQmn = desc_mn_sw128(smem_u32(smem + Lay::kQ), 0), dDOmn = desc_mn_sw128(smem_u32(smem + Lay::kDO), 0);
        const uint64_t dDSmn = desc_mn_sw128(smem_u32(smem + Lay::kDS), kBN * 128);
        // Sᵀ/dPᵀ of half hf of tile t into the half's TMEM buffers
        auto issue_s = [&](int t, int hf) -> bool {
            const int s = t & 1;
            if (hf == 0) {
                if (!wait_warp(&bars[kQFull + s], (t >> 1) & 1, ab, 4)) return false;
                tc_fence_after();
            }
            if (lane == 0) {
                const uint32_t off = (uint32_t)(s * Lay::kTile + hf * kHM * 128);
                const uint64_t bq = desc_add(dQk, off), bdo = desc_add(dDOk, off);
                const uint32_t dS = tS + hf * kHM, dDP = tDP + hf * kHM;
#pragma unroll
                for (int kk = 0; kk < kE / 16; ++kk) {
                    umma_ts(dS, tK + kk * 8, desc_add(bq, kk * 32), id_s, kk > 0 ? 1u : 0u);
                    umma_ts(dDP, tV + kk * 8, desc_add(bdo, kk * 32), id_s, kk > 0 ? 1u : 0u);
                }
                umma_commit(&bars[kSFull + hf]);
            }
            __syncwarp();
            return true;
        };
        bool ok = tiles > 0 && wait_warp(&bars[kKVFull], 0, ab, 3) && wait_warp(&bars[kKVTmem], 0, ab, 15);
        if (ok) ok = issue_s(0, 0) && issue_s(0, 1);
        for (int t = 0; ok && t < tiles; ++t) {
            const int s = t & 1;
            for (int hf = 0; hf < 2; ++hf) {
                if (!wait_warp(&bars[kPFull + hf], t & 1, ab, 6)) { ok = false; break; }
                tc_fence_after();
                if (PAIR && lane == 0) {
                    // dS half -> per-head dS tiles; before the half's next score
                    // tile lets its warpgroup refill the other dS buffer, the
                    // store issued two halves ago must have read its source.
                    const int h = kvh * p.n_rep + t / nq;
                    const int q0 = (qt0 + t % nq) * kBM;
                    const uint8_t* src = smem + Lay::kDS + s * Lay::kDSBytes + hf * kBN * 128;
                    if (p.pair_per_head)   // straight into dpair [B·H][KL][QL] (clipped at QL, KL)
                        tma_store_3d(&tm_ds, src, q0 + hf * kHM, (int)k0, b * QH + h);
                    else
                        tma_store_4d(&tm_ds, src, hf * kHM, (int)k0, q0 / kBM, b * QH + h);
                    bulk_commit();
                    bulk_wait_read<2>();
                }
                if (lane == 0) {
                    const uint32_t off = (uint32_t)(s * Lay::kTile + hf * kHM * 128);
                    const uint64_t bq = desc_add(dQmn, off), bdo = desc_add(dDOmn, off);
                    const uint32_t acc0 = (t > 0 || hf > 0) ? 1u : 0u;
#pragma unroll
                    for (int kk = 0; kk < kHM / 16; ++kk) {
                        // packed 16-bit Pᵀ/dSᵀ of the half's queries [16kk, 16kk+16)
                        const uint32_t pcol = hf * kHM + kk * 8;
                        const uint32_t acc = kk > 0 ? 1u : acc0;
                        umma_ts(tDV, tS + pcol, desc_add(bdo, kk * 16 * 128), id_kv, acc);
                        umma_ts(tDK, tDP + pcol, desc_add(bq, kk * 16 * 128), id_kv, acc);
                    }
                    if (hf == 1) umma_commit(&bars[kQEmpty + s]);
                }
                __syncwarp();
                if (t + 1 < tiles && !issue_s(t + 1, hf)) { ok = false; break; }
            }
            if (!ok) break;
            // dQ_t = dS_t·K once the previous dQ has been drained from TMEM
            if (t > 0 && !wait_warp(&bars[kDQEmpty], (t - 1) & 1, ab, 7)) break;
            tc_fence_after();
            if (lane == 0) {
                const uint64_t bds = desc_add(dDSmn, (uint32_t)s * Lay::kDSBytes);
#pragma unroll
                for (int kk = 0; kk < kBN / 16; ++kk)
                    umma_ss(tDQ, desc_add(bds, kk * 16 * 128), desc_add(dKmn, kk * 16 * 128), id_q, kk > 0 ? 1u : 0u);
                // the dQ warps reuse this dS buffer as staging once dQ_t is
                // done: the dS stores must have read it by then
                if (PAIR) bulk_wait_read<0>();
                umma_commit(&bars[kDQFull]);
            }
            __syncwarp();
        }
        // dS stores land before the CTA exits
        if (PAIR && lane == 0) bulk_wait<0>();
        // every MMA this warp issued retires before TMEM is read out / freed
        if (lane == 0) umma_commit(&bars[kFinal]);
        __syncwarp();
        wait(&bars[kFinal], 0, ab, 8);
    } else if (warp < 4) {
        // ------------------------------------------------------ tile provider
        const int tp = threadIdx.x - 64;
        for (int t = 0; t < tiles; ++t) {
            const int buf = t & 1;
            if (t >= 2 && !wait(&bars[kTileEmpty + buf], ((t >> 1) - 1) & 1, ab, 9)) break;
            const int h = kvh * p.n_rep + t / nq;
            const int64_t q0 = (int64_t)(qt0 + t % nq) * kBM;
            const int64_t ro = ((int64_t)b * QH + h) * QL;
            // both queries' loads in flight before the stores
            float lv[kBM / 64], dv[kBM / 64];
#pragma unroll
            for (int r = 0; r < kBM / 64; ++r) {
                const int64_t i = q0 + tp + 64 * r;
                lv[r] = i < QL ? __ldg(p.lse + ro + i) : 0.f;
                dv[r] = i < QL ? __ldg(p.delta + ro + i) : 0.f;
            }
#pragma unroll
            for (int r = 0; r < kBM / 64; ++r) {
                sLse[buf * kBM + tp + 64 * r] = lv[r] * kLog2e;
                sDel[buf * kBM + tp + 64 * r] = dv[r];
            }
            mbar_arrive(&bars[kTileFull + buf]);
        }
    } else if (warp < 12) {
        // ------------------------------------------------------ elementwise
        const int jr = (threadIdx.x - 128) & 127;            // key row = TMEM lane
        const int hf = (threadIdx.x - 128) >> 7;             // query half
        const int64_t j = k0 + jr;
        bool key_ok = j < KL;
        if (MASK && key_ok) key_ok = p.kmask[(int64_t)b * KL + j] != 0;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tSh = tS + hf * kHM + lane_off, tDPh = tDP + hf * kHM + lane_off;
        const float sl2 = p.scale * kLog2e;
        if (tiles > 0 && wait_warp(&bars[kKVFull], 0, ab, 16)) {
            // this key's row of K (half-0 warpgroup) or V (half 1) into TMEM as
            // 16-bit pairs, the A operand of the score MMAs
            const uint8_t* row = smem + (hf ? Lay::kV : Lay::kK) + jr * 128;
            uint32_t kr[32];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint4 u = *reinterpret_cast<const uint4*>(row + ((c ^ (jr & 7)) << 4));
                kr[4 * c] = u.x; kr[4 * c + 1] = u.y; kr[4 * c + 2] = u.z; kr[4 * c + 3] = u.w;
            }
            tmem_st32((hf ? tV : tK) + lane_off, kr);
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&bars[kKVTmem]);
        }
        for (int t = 0; t < tiles; ++t) {
            const int buf = t & 1;
            const int64_t qh0 = (int64_t)(qt0 + t % nq) * kBM + hf * kHM;   // first query of the half
            if (!wait_warp(&bars[kTileFull + buf], (t >> 1) & 1, ab, 10)) break;
            if (!wait_warp(&bars[kSFull + hf], t & 1, ab, 11)) break;
            if (t >= 2 && !wait_warp(&bars[kDSEmpty + buf], ((t >> 1) - 1) & 1, ab, 12)) break;
            const int pn = 2 * t + hf, pslot = pn % kPairSlots;
            if (PAIR && !wait_warp(&bars[kPairFull + pslot], (pn / kPairSlots) & 1, ab, 5)) break;
            tc_fence_after();
            // valid query columns of this key within the half: [cmin, cmax)
            const int64_t nvq = QL - qh0;
            const int cmax = key_ok ? (int)(nvq < kHM ? (nvq > 0 ? nvq : 0) : kHM) : 0;
            const int64_t cm = CAUSAL ? j - qh0 : 0;
            const int cmin = (int)(cm < 0 ? 0 : (cm > kHM ? kHM : cm));
            uint8_t* sDS = smem + Lay::kDS + buf * Lay::kDSBytes + hf * (kBN * 128) + jr * 128;
            const float* lse_h = sLse + buf * kBM + hf * kHM;
            const float* del_h = sDel + buf * kBM + hf * kHM;
            const uint8_t* prow = pair_slot(pslot) + jr * 128;
#pragma unroll 1
            for (int cc = 0; cc < kHM / 16; ++cc) {
                const int col = cc * 16;
                uint32_t sr[16], dr[16];
                tmem_ld16(tSh + col, sr);
                tmem_ld16(tDPh + col, dr);
                float4 l4[4], d4[4];
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    l4[v] = reinterpret_cast<const float4*>(lse_h + col)[v];
                    d4[v] = reinterpret_cast<const float4*>(del_h + col)[v];
                }
                uint32_t pw[8];
                if (PAIR) {
#pragma unroll
                    for (int v = 0; v < 2; ++v) {
                        const uint4 u = *reinterpret_cast<const uint4*>(prow + (((cc * 2 + v) ^ (jr & 7)) << 4));
                        pw[4 * v] = u.x; pw[4 * v + 1] = u.y; pw[4 * v + 2] = u.z; pw[4 * v + 3] = u.w;
                    }
                }
                tmem_ld_wait();
                uint32_t pk[8], dk[8];
                const int lo = cmin - col, hi = cmax - col;
                if (lo <= 0 && hi >= 16)
                    elementwise16<T, PAIR, false>(sr, dr, pw, l4, d4, sl2, 0, 16, pk, dk);
                else
                    elementwise16<T, PAIR, true>(sr, dr, pw, l4, d4, sl2, lo, hi, pk, dk);
                tmem_st8(tSh + cc * 8, pk);
                tmem_st8(tDPh + cc * 8, dk);
                // dS (16-bit) into shared memory for the dQ MMA: row jr, queries
                // col..col+15 of the half, canonical MN-major 128-byte swizzle.
#pragma unroll
                for (int v = 0; v < 2; ++v) {
                    const int chunk = cc * 2 + v;
                    *reinterpret_cast<uint4*>(sDS + ((chunk ^ (jr & 7)) << 4)) =
                        make_uint4(dk[4 * v], dk[4 * v + 1], dk[4 * v + 2], dk[4 * v + 3]);
                }
            }
            mbar_arrive(&bars[kTileEmpty + buf]);
            if (PAIR) mbar_arrive(&bars[kPairEmpty + pslot]);
            tmem_st_wait();
            fence_proxy_async_smem();   // dS smem writes -> tensor-core (async proxy) reads
            tc_fence_before();
            mbar_arrive(&bars[kPFull + hf]);
        }
        // epilogue: dK (half-0 warpgroup) and dV (half-1 warpgroup) rows of this CTA's keys
        if (wait_warp(&bars[kFinal], 0, ab, 13)) {
            tc_fence_after();
            const bool is_dk = hf == 0;
            const uint32_t src = (is_dk ? tDK : tDV) + lane_off;
            T* dst = reinterpret_cast<T*>(is_dk ? p.dk : p.dv) + (((int64_t)b * p.KH + kvh) * KL + j) * kE;
            const float mul = is_dk ? p.scale : 1.f;
            if (is_dk && p.rope_cos != nullptr) {
                // fused RoPE backward: dk of the un-rotated k, pairs (e, e + 32)
                // rotated by cos/sin of index e at position j (sin → −sin)
                const int64_t tr = ((p.rope_cb == 1 ? 0 : (int64_t)b) * KL + (j < KL ? j : 0)) * kE;
#pragma unroll 1
                for (int c = 0; c < 2; ++c) {
                    uint32_t ra[16], rb[16];
                    tmem_ld16(src + c * 16, ra);
                    tmem_ld16(src + 32 + c * 16, rb);
                    tmem_ld_wait();
                    if (j < KL) {
                        float4 cw[4], sw[4];   // cos/sin of indices 16c .. 16c+15 at position j
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            cw[v] = __ldg(reinterpret_cast<const float4*>(p.rope_cos + tr + 16 * c) + v);
                            sw[v] = __ldg(reinterpret_cast<const float4*>(p.rope_sin + tr + 16 * c) + v);
                        }
                        uint32_t pa[8], pb[8];
#pragma unroll
                        for (int u = 0; u < 16; u += 2) {
                            float oa[2], ob[2];
#pragma unroll
                            for (int v = 0; v < 2; ++v) {
                                const float a = tiles > 0 ? __uint_as_float(ra[u + v]) * mul : 0.f;
                                const float bb = tiles > 0 ? __uint_as_float(rb[u + v]) * mul : 0.f;
                                const float cs = reinterpret_cast<const float*>(cw)[u + v];
                                const float sn = reinterpret_cast<const float*>(sw)[u + v];
                                oa[v] = a * cs + bb * sn;
                                ob[v] = bb * cs - a * sn;
                            }
                            pa[u >> 1] = pack16<T>(oa[0], oa[1]);
                            pb[u >> 1] = pack16<T>(ob[0], ob[1]);
                        }
                        uint4* da = reinterpret_cast<uint4*>(dst + c * 16);
                        uint4* db = reinterpret_cast<uint4*>(dst + 32 + c * 16);
                        da[0] = make_uint4(pa[0], pa[1], pa[2], pa[3]);
                        da[1] = make_uint4(pa[4], pa[5], pa[6], pa[7]);
                        db[0] = make_uint4(pb[0], pb[1], pb[2], pb[3]);
                        db[1] = make_uint4(pb[4], pb[5], pb[6], pb[7]);
                    }
                }
            } else {
#pragma unroll
                for (int c = 0; c < kE / 16; ++c) {
                    uint32_t raw[16];
                    tmem_ld16(src + c * 16, raw);
                    tmem_ld_wait();
                    if (j < KL) {
                        uint32_t pk[8];
#pragma unroll
                        for (int u = 0; u < 8; ++u)
                            pk[u] = tiles > 0 ? pack16<T>(__uint_as_float(raw[2 * u]) * mul,
                                                          __uint_as_float(raw[2 * u + 1]) * mul)
                                              : 0u;
                        uint4* d4 = reinterpret_cast<uint4*>(dst + c * 16);
                        d4[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                        d4[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                    }
                }
            }
        }
    } else {
        // ------------------------------------------------------ dQ reductions
        // warp w: query rows 32w..32w+31 of the tile (TMEM lanes), staged as
        // two [32 rows][32 floats] boxes, 128-byte swizzle, in the tile's dS
        // buffer, then one TMA reduce-add per box into dq_acc (rows past QL
        // are clipped by the tensor map)
        const int w = warp & 3;
        const uint32_t lane_off = (uint32_t)(w * 32) << 16;
        // A per-head dpair gets its zeros here, before the first dQ tile: this
        // CTA's key rows, queries [0, i_lo) of every head of the group -- the
        // part no tile covers (above the causal diagonal; all of it past the
        // last kept key).  Bulk copies from a zeroed 4 KB buffer, in flight
        // while the tiles run; under the causal mask the CTAs with the most
        // zeros (late key tiles) are the ones with the fewest tiles.
        int64_t i_lo = 0;
        if (PAIR && p.pair_per_head) i_lo = nq == 0 ? QL : (CAUSAL ? (k0 < QL ? k0 : QL) : 0);
        if (w == 0 && i_lo > 0) {
            uint8_t* zb = smem + Lay::kZero;
            for (int u = lane; u < Lay::kZeroBytes / 16; u += 32)
                reinterpret_cast<uint4*>(zb)[u] = make_uint4(0u, 0u, 0u, 0u);
            fence_proxy_async_smem();   // generic zero writes -> bulk-copy (async proxy) reads
            __syncwarp();
            // lane 1: its own bulk groups, apart from lane 0's reduce-adds
            if (lane == 1) {
                const int64_t rows = KL - k0 < kBN ? KL - k0 : kBN;
                const int64_t row_bytes = i_lo * 2;
                for (int r = 0; r < p.n_rep; ++r) {
                    uint8_t* base = reinterpret_cast<uint8_t*>(p.dpair) +
                                    (((int64_t)b * QH + kvh * p.n_rep + r) * KL + k0) * QL * 2;
                    for (int64_t jr = 0; jr < rows; ++jr)
                        for (int64_t off = 0; off < row_bytes; off += Lay::kZeroBytes) {
                            const int64_t n = row_bytes - off < Lay::kZeroBytes ? row_bytes - off : Lay::kZeroBytes;
                            bulk_store(base + jr * QL * 2 + off, zb, (uint32_t)n);
                        }
                }
                bulk_commit();
            }
            __syncwarp();
        }
        for (int t = 0; t < tiles; ++t) {
            const int h = kvh * p.n_rep + t / nq;
            const int q0 = (qt0 + t % nq) * kBM;
            if (!wait_warp(&bars[kDQFull], t & 1, ab, 14)) break;
            tc_fence_after();
            uint32_t raw[4][16];
#pragma unroll
            for (int c = 0; c < 4; ++c) tmem_ld16(tDQ + lane_off + c * 16, raw[c]);
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(&bars[kDQEmpty]);   // TMEM dQ may be overwritten
            uint8_t* stg = smem + Lay::kDS + (t & 1) * Lay::kDSBytes + w * 8192;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    const int chunk = (c & 1) * 4 + v;
                    *reinterpret_cast<float4*>(stg + (c >> 1) * 4096 + lane * 128 + ((chunk ^ (lane & 7)) << 4)) =
                        make_float4(__uint_as_float(raw[c][4 * v]) * p.scale, __uint_as_float(raw[c][4 * v + 1]) * p.scale,
                                    __uint_as_float(raw[c][4 * v + 2]) * p.scale,
                                    __uint_as_float(raw[c][4 * v + 3]) * p.scale);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_reduce_add_3d(&tm_dq, stg, 0, q0 + 32 * w, b * QH + h);
                tma_reduce_add_3d(&tm_dq, stg + 4096, 32, q0 + 32 * w, b * QH + h);
                bulk_commit();
                bulk_wait_read<0>();
                mbar_arrive(&bars[kDSEmpty + (t & 1)]);
            }
            __syncwarp();
        }
        if (lane == 0 || (lane == 1 && w == 0 && i_lo > 0)) bulk_wait<0>();   // reductions, zeros land before exit
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// 3-D map over the fp32 dQ accumulator [B·QH][QL][64], box (32, 32, 1),
// 128-byte swizzle (the dQ warps' staging layout).
bool make_dq_map(CUtensorMap* m, float* base, int64_t QL, int64_t bh) {
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

template <typename T, bool CAUSAL, bool PAIR, bool MASK>
int launch(const Params& p, const void* pair_tiles, void* ds_tiles, cudaStream_t s) {
    constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
    const int64_t qlp = (p.QL + 127) / 128 * 128, klp = (p.KL + 127) / 128 * 128;
    CUtensorMap tq, tk, tv, tdo, tp, tds, tdq;
    memset(&tp, 0, sizeof(tp));
    memset(&tds, 0, sizeof(tds));
    if (!make_map(&tq, p.q, kE, p.QL, (int64_t)p.B * p.QH, kBM, bf16) ||
        !make_map(&tk, p.k, kE, p.KL, (int64_t)p.B * p.KH, kBN, bf16) ||
        !make_map(&tv, p.v, kE, p.KL, (int64_t)p.B * p.KH, kBN, bf16) ||
        !make_map(&tdo, p.dO, kE, p.QL, (int64_t)p.B * p.QH, kBM, bf16) ||
        !make_dq_map(&tdq, p.dq_acc, p.QL, (int64_t)p.B * p.QH) ||
        (PAIR && !p.pair_per_head &&
         (!make_tiles_map(&tp, pair_tiles, qlp, klp, (int64_t)p.B * p.QH, bf16) ||
          !make_tiles_map(&tds, ds_tiles, qlp, klp, (int64_t)p.B * p.QH, bf16))) ||
        (PAIR && p.pair_per_head &&
         (!make_per_head_map(&tp, p.pair, p.QL, p.KL, (int64_t)p.B * p.QH, bf16) ||
          !make_per_head_map(&tds, p.dpair, p.QL, p.KL, (int64_t)p.B * p.QH, bf16))))
        return fail(NNOP_ERR_CUDA, "flash_attention_bwd: cuTensorMapEncodeTiled failed");
    auto kern = fa_bwd_sm100_kernel<T, CAUSAL, PAIR, MASK>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kAlloc) != cudaSuccess)
        return fail(NNOP_ERR_CUDA, "flash_attention_bwd: cannot set shared memory size");
    dim3 grid((unsigned)((p.KL + kBN - 1) / kBN), p.KH, p.B);
    kern<<<grid, kThreads, Lay::kAlloc, s>>>(tq, tk, tv, tdo, tp, tds, tdq, p);
    return check_launch("flash_attention_bwd (sm100)");
}

template <typename T, bool CAUSAL>
int dispatch_flags(const Params& p, const void* pt, void* dt, cudaStream_t s) {
    const bool pair = p.pair != nullptr, mask = p.kmask != nullptr;
    if (pair && mask) return launch<T, CAUSAL, true, true>(p, pt, dt, s);
    if (pair) return launch<T, CAUSAL, true, false>(p, pt, dt, s);
    if (mask) return launch<T, CAUSAL, false, true>(p, pt, dt, s);
    return launch<T, CAUSAL, false, false>(p, pt, dt, s);
}

}  // namespace

int sm100_bwd128(const Params& p, int dtype, bool causal, cudaStream_t s);

// Shapes the tcgen05 backward kernels cover: E = 64 (with or without the pair
// bias, this file) and E = 128 without it (fa_bwd128_sm100.cu); the others
// use the mma.sync kernels.
bool sm100_bwd_supported(const Params& p, int dtype) {
    if (dtype != NNOP_BF16 && dtype != NNOP_F16) return false;
    return p.E == kE || (p.E == 128 && p.pair == nullptr);
}

int sm100_bwd_tile() { return kBN; }

// Reads and clears the bounded-wait timeout flags of this file's kernels.
int sm100_bwd_timeouts() {
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, sm100::g_wait_timeout, sizeof(int));
    cudaMemcpyToSymbol(sm100::g_wait_timeout, &z, sizeof(int));
    return v;
}

int sm100_bwd(const Params& p, const void* pair_tiles, void* ds_tiles, int dtype, bool causal, cudaStream_t s) {
    if (p.E == 128) return sm100_bwd128(p, dtype, causal, s);
    if (dtype == NNOP_BF16)
        return causal ? dispatch_flags<__nv_bfloat16, true>(p, pair_tiles, ds_tiles, s)
                      : dispatch_flags<__nv_bfloat16, false>(p, pair_tiles, ds_tiles, s);
    return causal ? dispatch_flags<__half, true>(p, pair_tiles, ds_tiles, s)
                  : dispatch_flags<__half, false>(p, pair_tiles, ds_tiles, s);
}

}  // namespace fa
}  // namespace nnop
