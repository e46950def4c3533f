// Flash-attention backward on the sm_100a tensor cores (tcgen05 UMMA, TMEM
// accumulators, TMA-fed tiles), bf16/f16, E = 64.
//
// Reference: `_flash_attention_bwd!` (src/attention_bwd.jl:1-175) -- one
// workgroup per (head, batch) walking every (key tile, query tile) pair with
// five WMMA/SIMT GEMMs, a read-modify-write of dq in global memory and atomics
// for GQA.  Here one CTA owns a 128-key tile of one KV head of one batch and
// walks the 128-query tiles of every query head of its GQA group; dK and dV
// stay in TMEM for the whole walk.  Per step (query tile i):
//   Sᵀ  = K·Q_iᵀ (+ c·I·pairᵀ)  (keys on TMEM lanes)   UMMA ss
//   dPᵀ = V·dO_iᵀ                                       UMMA ss
//   Pᵀ  = exp(Sᵀ·scale − lse_i),  dSᵀ = Pᵀ∘(dPᵀ − δ_i)   (elementwise)
//   dV += Pᵀ·dO_i   (Pᵀ from TMEM)                      UMMA ts
//   dK += dSᵀ·Q_i   (dSᵀ from TMEM)                     UMMA ts
//   dQ_i = dS·K     (dS from shared memory, MN-major)   UMMA ss
//   dq_acc[i] += scale·dQ_i  (fp32 vector reductions, red.global.add.v4.f32)
//   dpair[j, i] = dSᵀ (the reference's dpair = dS/scale with its dS ∘ scale),
//                 written per head as key-major dS tiles, see pair_tiles.cu.
// The pair bias enters through the tensor cores: c = 1/scale (a power of two,
// so c·pair is exact in the fp32 accumulator) times the shifted identity of
// fa_sm100.cuh as A, the pair tile [key][query] of the key-major per-head copy
// pair_tiles() writes as the MN-major B operand.
// Warp roles (512 threads):
//   warp 0      TMA producer (K, V once; Q_i, dO_i into a 2-stage ring)
//   warp 1      MMA issuer (one lane)
//   warps 2-3   tile provider: lse_i (log2 units) and δ_i
//   (the pair tile of (query tile, key tile, head), two 64-query boxes of
//   [B][H][KL][QL], is also loaded by warp 0; dS goes out as 32-byte row
//   pieces in the same layout and dpair_from_tiles() turns it into dpair)
//   warps 4-11  elementwise: two warpgroups on the same 128 TMEM lanes
//               (one key per lane), query columns [0,64) and [64,128)
//   warps 12-15 dQ: TMEM dQ rows -> fp32 reductions into the accumulator
// TMEM columns: Sᵀ [0,128), dPᵀ [128,256), dV [256,320), dK [320,384),
// dQ [384,448).  The 16-bit Pᵀ / dSᵀ overwrite their own warpgroup's score
// columns (query c -> column c/2 + 32·[c >= 64]) so neither warpgroup can
// overwrite scores the other has not read yet.  All mbarrier waits are bounded.
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
constexpr int kBM = 128;   // queries per step
constexpr int kE = 64;
constexpr int kThreads = 512;

enum Bar {
    kKVFull = 0,
    kQFull = 1,       // +stage: Q_i and dO_i landed
    kQEmpty = 3,      // +stage: dV/dK MMAs of the step retired
    kSFull = 5,       // Sᵀ, dPᵀ in TMEM
    kPFull = 6,       // elementwise done (256 arrivals)
    kDQFull = 7,      // dQ_i in TMEM
    kDQEmpty = 8,     // dQ warps done with TMEM dQ (128 arrivals)
    kTileFull = 9,    // +buffer: provider -> elementwise (64 arrivals)
    kTileEmpty = 11,  // +buffer: elementwise -> provider (256 arrivals)
    kFinal = 13,      // every MMA retired
    kPairFull = 14,   // +buffer: pair tile landed (TMA)
    kPairEmpty = 16,  // +buffer: its UMMAs retired
    kNumBars = 18
};

struct Lay {
    static constexpr int kTile = 128 * 64 * 2;      // one [128][64] 16-bit tile, 16 KB
    static constexpr int kK = 0;
    static constexpr int kV = kK + kTile;
    static constexpr int kQ = kV + kTile;           // 2 stages
    static constexpr int kDO = kQ + 2 * kTile;      // 2 stages
    static constexpr int kDS = kDO + 2 * kTile;     // [2 halves][128 keys][64 queries], MN-major SW128
    static constexpr int kPair = kDS + 2 * kTile;   // 2 buffers of [2 halves][BN keys][64 queries] SW128
    static constexpr int kPairBytes = kBM * kBN * 2;
    static constexpr int kEye = kPair + 2 * kPairBytes;   // shifted identity (1024-aligned)
    static constexpr int kLse = kEye + kEyeBytes;         // [2][BM] float (log2 units)
    static constexpr int kDel = kLse + 2 * kBM * 4;       // [2][BM] float
    static constexpr int kBar = kDel + 2 * kBM * 4;
    static constexpr int kTmemSlot = kBar + kNumBars * 8;
    static constexpr int kTotal = kTmemSlot + 16;
    static constexpr int kAlloc = kTotal + 1024;
};

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}
// Warp-uniform bounded wait: true only if every lane saw the phase complete
// (guards warp-wide tcgen05.ld/st, which must not run divergent).
__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t parity, volatile int* ab, int site) {
    const bool ok = wait(bar, parity, ab, site);
    return __all_sync(0xffffffffu, ok);
}

template <typename T, bool CAUSAL, bool PAIR, bool MASK>
__global__ void __launch_bounds__(kThreads, 1)
fa_bwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_pair, const Params p, uint16_t* __restrict__ ds_tiles,
                    int64_t qlp, int64_t klp) {
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
    const int steps = nq * p.n_rep;

    __shared__ int s_abort;   // set by the first wait of this CTA that gives up
    volatile int* ab = &s_abort;
    if (threadIdx.x == 0) {
        s_abort = 0;
        mbar_init(&bars[kKVFull], 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&bars[kQFull + s], 1);
            mbar_init(&bars[kQEmpty + s], 1);
            mbar_init(&bars[kTileFull + s], 64);
            mbar_init(&bars[kTileEmpty + s], 256);
            mbar_init(&bars[kPairFull + s], 1);
            mbar_init(&bars[kPairEmpty + s], 1);
        }
        mbar_init(&bars[kSFull], 1);
        mbar_init(&bars[kPFull], 256);
        mbar_init(&bars[kDQFull], 1);
        mbar_init(&bars[kDQEmpty], 128);
        mbar_init(&bars[kFinal], 1);
        fence_mbar_init();
    }
    if (PAIR) {
        build_eye<T>(smem + Lay::kEye, 1.f / p.scale, threadIdx.x, kThreads);
        fence_proxy_async_smem();   // identity writes -> UMMA reads
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

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0 && steps > 0) {
            tma_prefetch(&tm_q);
            tma_prefetch(&tm_k);
            tma_prefetch(&tm_v);
            tma_prefetch(&tm_do);
            if (PAIR) tma_prefetch(&tm_pair);
            const int bh_k = b * p.KH + kvh;
            mbar_expect_tx(&bars[kKVFull], 2 * Lay::kTile);
            tma_load_3d(smem + Lay::kK, &tm_k, &bars[kKVFull], 0, (int)k0, bh_k);
            tma_load_3d(smem + Lay::kV, &tm_v, &bars[kKVFull], 0, (int)k0, bh_k);
            int issued = 0;
            for (int st = 0; st < steps; ++st) {
                const int s = st & 1;
                if (st >= 2 && !wait(&bars[kQEmpty + s], ((st >> 1) - 1) & 1, ab, 1)) break;
                if (PAIR && st >= 2 && !wait(&bars[kPairEmpty + s], ((st >> 1) - 1) & 1, ab, 14)) break;
                issued = st + 1;
                const int h = kvh * p.n_rep + st / nq;
                const int q0 = (qt0 + st % nq) * kBM;
                mbar_expect_tx(&bars[kQFull + s], 2 * Lay::kTile);
                tma_load_3d(smem + Lay::kQ + s * Lay::kTile, &tm_q, &bars[kQFull + s], 0, q0, b * QH + h);
                tma_load_3d(smem + Lay::kDO + s * Lay::kTile, &tm_do, &bars[kQFull + s], 0, q0, b * QH + h);
                if (PAIR) {
                    mbar_expect_tx(&bars[kPairFull + s], Lay::kPairBytes);
#pragma unroll
                    for (int half = 0; half < 2; ++half)
                        tma_load_3d(smem + Lay::kPair + s * Lay::kPairBytes + half * kBN * 128, &tm_pair,
                                    &bars[kPairFull + s], q0 + half * 64, (int)k0, b * QH + h);
                }
            }
            // copies in flight land before the CTA leaves (bounded waits)
            wait(&bars[kKVFull], 0, ab, 2);
            for (int st = issued - 2 < 0 ? 0 : issued - 2; st < issued; ++st) {
                wait(&bars[kQFull + (st & 1)], (st >> 1) & 1, ab, 3);
                if (PAIR) wait(&bars[kPairFull + (st & 1)], (st >> 1) & 1, ab, 15);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        constexpr uint32_t id_s = idesc_f16<kBF16>(128, 128, false, false);   // Sᵀ, dPᵀ
        constexpr uint32_t id_kv = idesc_f16<kBF16>(128, 64, false, true);    // dV, dK (A in TMEM)
        constexpr uint32_t id_q = idesc_f16<kBF16>(128, 64, true, true);      // dQ (A = dS, MN-major)
        const uint32_t sK = smem_u32(smem + Lay::kK), sV = smem_u32(smem + Lay::kV);
        constexpr uint32_t id_p = idesc_f16<kBF16>(128, 128, false, true);   // Sᵀ += c·I·pairᵀ
        const uint32_t sDS = smem_u32(smem + Lay::kDS);
        const uint32_t sEye = smem_u32(smem + Lay::kEye);
        bool ok = steps > 0 && wait_warp(&bars[kKVFull], 0, ab, 4);
        for (int st = 0; ok && st < steps; ++st) {
            const int s = st & 1;
            if (!wait_warp(&bars[kQFull + s], (st >> 1) & 1, ab, 5)) break;
            if (PAIR && !wait_warp(&bars[kPairFull + s], (st >> 1) & 1, ab, 16)) break;
            tc_fence_after();
            const uint32_t sQ = smem_u32(smem + Lay::kQ + s * Lay::kTile);
            const uint32_t sDO = smem_u32(smem + Lay::kDO + s * Lay::kTile);
            if (lane == 0) {
#pragma unroll
                for (int kk = 0; kk < kE / 16; ++kk) {
                    umma_ss(tS, desc_k_sw128(sK + kk * 32), desc_k_sw128(sQ + kk * 32), id_s, kk > 0 ? 1u : 0u);
                    umma_ss(tDP, desc_k_sw128(sV + kk * 32), desc_k_sw128(sDO + kk * 32), id_s, kk > 0 ? 1u : 0u);
                }
                if (PAIR) {
                    // B = pair tile [key][query]: MN-major over queries, K = keys
                    const uint32_t sP = smem_u32(smem + Lay::kPair + s * Lay::kPairBytes);
#pragma unroll
                    for (int kk = 0; kk < kBN / 16; ++kk)
                        umma_ss(tS, desc_k_sw128(eye_step(sEye, kk)), desc_mn_sw128(sP + kk * 16 * 128, kBN * 128),
                                id_p, 1u);
                    umma_commit(&bars[kPairEmpty + s]);
                }
                umma_commit(&bars[kSFull]);
            }
            __syncwarp();
            if (!wait_warp(&bars[kPFull], st & 1, ab, 6)) break;
            tc_fence_after();
            if (lane == 0) {
#pragma unroll
                for (int kk = 0; kk < kBM / 16; ++kk) {
                    // packed 16-bit Pᵀ/dSᵀ of queries [16kk, 16kk+16)
                    const uint32_t pcol = kk * 8 + (kk >= 4 ? 32 : 0);
                    const uint32_t acc = (st > 0 || kk > 0) ? 1u : 0u;
                    umma_ts(tDV, tS + pcol, desc_mn_sw128(sDO + kk * 16 * 128, 0), id_kv, acc);
                    umma_ts(tDK, tDP + pcol, desc_mn_sw128(sQ + kk * 16 * 128, 0), id_kv, acc);
                }
                umma_commit(&bars[kQEmpty + s]);
            }
            __syncwarp();
            if (st > 0 && !wait_warp(&bars[kDQEmpty], (st - 1) & 1, ab, 7)) break;
            tc_fence_after();
            if (lane == 0) {
#pragma unroll
                for (int kk = 0; kk < kBN / 16; ++kk)
                    umma_ss(tDQ, desc_mn_sw128(sDS + kk * 16 * 128, 128 * 128), desc_mn_sw128(sK + kk * 16 * 128, 0),
                            id_q, kk > 0 ? 1u : 0u);
                umma_commit(&bars[kDQFull]);
            }
            __syncwarp();
        }
        // every MMA this warp issued retires before TMEM is read out / freed
        if (lane == 0) umma_commit(&bars[kFinal]);
        __syncwarp();
        wait(&bars[kFinal], 0, ab, 8);
    } else if (warp < 4) {
        // ------------------------------------------------------ tile provider
        const int tp = threadIdx.x - 64;
        for (int st = 0; st < steps; ++st) {
            const int buf = st & 1;
            if (st >= 2 && !wait(&bars[kTileEmpty + buf], ((st >> 1) - 1) & 1, ab, 9)) break;
            const int h = kvh * p.n_rep + st / nq;
            const int64_t q0 = (int64_t)(qt0 + st % nq) * kBM;
            const int64_t ro = ((int64_t)b * QH + h) * QL;
            for (int t = tp; t < kBM; t += 64) {
                const int64_t i = q0 + t;
                sLse[buf * kBM + t] = i < QL ? p.lse[ro + i] * kLog2e : 0.f;
                sDel[buf * kBM + t] = i < QL ? p.delta[ro + i] : 0.f;
            }
            mbar_arrive(&bars[kTileFull + buf]);
        }
    } else if (warp < 12) {
        // ------------------------------------------------------ elementwise
        const int jr = (threadIdx.x - 128) & 127;            // key row = TMEM lane
        const int c0 = ((threadIdx.x - 128) >> 7) * 64;       // query columns [c0, c0+64)
        const int64_t j = k0 + jr;
        bool key_ok = j < KL;
        if (MASK && key_ok) key_ok = p.kmask[(int64_t)b * KL + j] != 0;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const float sl2 = p.scale * kLog2e;
        uint8_t* sDS = smem + Lay::kDS;
        for (int st = 0; st < steps; ++st) {
            const int buf = st & 1;
            const int h = kvh * p.n_rep + st / nq;
            const int64_t q0 = (int64_t)(qt0 + st % nq) * kBM;
            if (!wait_warp(&bars[kTileFull + buf], (st >> 1) & 1, ab, 10)) break;
            if (!wait_warp(&bars[kSFull], st & 1, ab, 11)) break;
            tc_fence_after();
            // dS tile row of this key: [b][h][key][query]
            uint16_t* dst_row = PAIR ? ds_tiles + (((int64_t)b * QH + h) * klp + j) * qlp + q0 : nullptr;
#pragma unroll 1
            for (int cc = 0; cc < 4; ++cc) {
                const int col = c0 + cc * 16;
                uint32_t sr[16], dr[16];
                tmem_ld16(tS + lane_off + col, sr);
                tmem_ld16(tDP + lane_off + col, dr);
                tmem_ld_wait();
                uint32_t pk[8], dk[8];
#pragma unroll
                for (int t = 0; t < 16; t += 2) {
                    float pv[2], dv[2];
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const int c = col + t + u;
                        const int64_t i = q0 + c;
                        bool valid = key_ok && i < QL;
                        if (CAUSAL) valid = valid && (j <= i);
                        const float x = __uint_as_float(sr[t + u]) * sl2 - sLse[buf * kBM + c];
                        const float pr = valid ? ex2(x) : 0.f;
                        pv[u] = pr;
                        dv[u] = pr * (__uint_as_float(dr[t + u]) - sDel[buf * kBM + c]);
                    }
                    pk[t >> 1] = pack16<T>(pv[0], pv[1]);
                    dk[t >> 1] = pack16<T>(dv[0], dv[1]);
                }
                const uint32_t pcol = col / 2 + (c0 ? 32 : 0);
                tmem_st8(tS + lane_off + pcol, pk);
                tmem_st8(tDP + lane_off + pcol, dk);
                // dS (16-bit) into shared memory for the dQ MMA: row jr, queries
                // col..col+15, canonical MN-major 128-byte-swizzle layout.
#pragma unroll
                for (int v = 0; v < 2; ++v) {
                    const int q8 = col + v * 8;
                    const int half = q8 >> 6, chunk = (q8 & 63) >> 3;
                    uint4* dst = reinterpret_cast<uint4*>(sDS + half * (128 * 128) + jr * 128 + ((chunk ^ (jr & 7)) << 4));
                    *dst = make_uint4(dk[4 * v], dk[4 * v + 1], dk[4 * v + 2], dk[4 * v + 3]);
                }
                if (PAIR) {
#pragma unroll
                    for (int v = 0; v < 2; ++v)
                        __stcs(reinterpret_cast<uint4*>(dst_row + col + v * 8),
                               make_uint4(dk[4 * v], dk[4 * v + 1], dk[4 * v + 2], dk[4 * v + 3]));
                }
            }
            mbar_arrive(&bars[kTileEmpty + buf]);
            tmem_st_wait();
            fence_proxy_async_smem();   // dS smem writes -> tensor-core (async proxy) reads
            tc_fence_before();
            mbar_arrive(&bars[kPFull]);
        }
        // epilogue: dK (warpgroup 0) and dV (warpgroup 1) rows of this CTA's keys
        if (wait_warp(&bars[kFinal], 0, ab, 12)) {
            tc_fence_after();
            const bool is_dk = c0 == 0;
            const uint32_t src = (is_dk ? tDK : tDV) + lane_off;
            T* dst = reinterpret_cast<T*>(is_dk ? p.dk : p.dv) + (((int64_t)b * p.KH + kvh) * KL + j) * kE;
            const float mul = is_dk ? p.scale : 1.f;
#pragma unroll
            for (int c = 0; c < kE / 16; ++c) {
                uint32_t raw[16];
                tmem_ld16(src + c * 16, raw);
                tmem_ld_wait();
                if (j < KL) {
                    uint32_t pk[8];
#pragma unroll
                    for (int t = 0; t < 8; ++t)
                        pk[t] = steps > 0 ? pack16<T>(__uint_as_float(raw[2 * t]) * mul, __uint_as_float(raw[2 * t + 1]) * mul)
                                          : 0u;
                    uint4* d4 = reinterpret_cast<uint4*>(dst + c * 16);
                    d4[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    d4[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                }
            }
        }
    } else {
        // ------------------------------------------------------ dQ reductions
        const int r = threadIdx.x - 384;                      // query row = TMEM lane
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        for (int st = 0; st < steps; ++st) {
            const int h = kvh * p.n_rep + st / nq;
            const int64_t i = (int64_t)(qt0 + st % nq) * kBM + r;
            if (!wait_warp(&bars[kDQFull], st & 1, ab, 13)) break;
            tc_fence_after();
            float* dq = p.dq_acc + (((int64_t)b * QH + h) * QL + i) * kE;
#pragma unroll
            for (int c = 0; c < kE / 16; ++c) {
                uint32_t raw[16];
                tmem_ld16(tDQ + lane_off + c * 16, raw);
                tmem_ld_wait();
                if (i < QL) {
#pragma unroll
                    for (int v = 0; v < 4; ++v)
                        red_add_v4(dq + c * 16 + 4 * v, __uint_as_float(raw[4 * v]) * p.scale,
                                   __uint_as_float(raw[4 * v + 1]) * p.scale, __uint_as_float(raw[4 * v + 2]) * p.scale,
                                   __uint_as_float(raw[4 * v + 3]) * p.scale);
                }
            }
            tc_fence_before();
            mbar_arrive(&bars[kDQEmpty]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

template <typename T, bool CAUSAL, bool PAIR, bool MASK>
int launch(const Params& p, const void* pair_tiles, void* ds_tiles, cudaStream_t s) {
    constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
    const int64_t qlp = (p.QL + 127) / 128 * 128, klp = (p.KL + 127) / 128 * 128;
    CUtensorMap tq, tk, tv, tdo, tp;
    memset(&tp, 0, sizeof(tp));
    if (!make_map(&tq, p.q, kE, p.QL, (int64_t)p.B * p.QH, kBM, bf16) ||
        !make_map(&tk, p.k, kE, p.KL, (int64_t)p.B * p.KH, kBN, bf16) ||
        !make_map(&tv, p.v, kE, p.KL, (int64_t)p.B * p.KH, kBN, bf16) ||
        !make_map(&tdo, p.dO, kE, p.QL, (int64_t)p.B * p.QH, kBM, bf16) ||
        (PAIR && !make_map(&tp, pair_tiles, (int)qlp, klp, (int64_t)p.B * p.QH, kBN, bf16)))
        return fail(NNOP_ERR_CUDA, "flash_attention_bwd: cuTensorMapEncodeTiled failed");
    auto kern = fa_bwd_sm100_kernel<T, CAUSAL, PAIR, MASK>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kAlloc) != cudaSuccess)
        return fail(NNOP_ERR_CUDA, "flash_attention_bwd: cannot set shared memory size");
    dim3 grid((unsigned)((p.KL + kBN - 1) / kBN), p.KH, p.B);
    kern<<<grid, kThreads, Lay::kAlloc, s>>>(tq, tk, tv, tdo, tp, p, static_cast<uint16_t*>(ds_tiles), qlp, klp);
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

bool sm100_bwd_supported(const Params& p, int dtype) {
    return (dtype == NNOP_BF16 || dtype == NNOP_F16) && p.E == kE;
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
    if (dtype == NNOP_BF16)
        return causal ? dispatch_flags<__nv_bfloat16, true>(p, pair_tiles, ds_tiles, s)
                      : dispatch_flags<__nv_bfloat16, false>(p, pair_tiles, ds_tiles, s);
    return causal ? dispatch_flags<__half, true>(p, pair_tiles, ds_tiles, s)
                  : dispatch_flags<__half, false>(p, pair_tiles, ds_tiles, s);
}

}  // namespace fa
}  // namespace nnop
