// Flash-attention forward on the sm_100a tensor cores, two query tiles per
// CTA in ping-pong (bf16/f16; E in {64, 128}, E = 64 with a pair bias).
//
// Reference: `_flash_attention_fwd!` (src/attention.jl:8-143).
//
// The one-tile kernel (fa_fwd_sm100.cu) is bound by its softmax warpgroup:
// per 128-key tile the tensor cores need ~1000 cycles (E = 128) but the one
// warpgroup's TMEM-load → max → exp2 → store chain takes ~3000.  Here a CTA
// owns two 128-query tiles of one head (tiles 2p and 2p+1) with a softmax
// warpgroup each, a TMEM score buffer S_t and an accumulator O_t per tile, and
// one K/V stream both tiles use.  Per key tile j the tensor pipe runs
//   PV_0(j), S_0(j+1), PV_1(j), S_1(j+1)
// so one tile's softmax overlaps the other tile's MMAs, the two warpgroups'
// latency stalls interleave on the same schedulers, and each K/V tile is
// loaded once for 256 queries.
//
// Warp roles (384 threads):
//   warp 0      TMA producer: Q_0, Q_1 once, then K_j / V_j into a ring
//   warp 1      MMA issuer (one lane)
//   warps 2-3   (only the key-validity bits at start)
//   warps 4-7   softmax of tile 0, warps 8-11 softmax of tile 1: thread r
//               owns query row r of its tile (TMEM lane r); it reads its 128
//               scores, masks, keeps a running max (rescaling O only when the
//               max grows by more than 2^8, warp-uniform), writes P as 16-bit
//               values over the first half of its score columns, and at the
//               end normalises O and writes o and lse.
// TMEM: tile t: S_t [t·W, t·W+128), O_t [t·W+128, t·W+128+E), W = 128 + E.
// S_t is single-buffered: S_t(j+1) is issued behind PV_t(j), which reads P_t(j)
// from the same columns (one thread's UMMAs run in order).
// With a pair bias (E = 64) the producer also loads the pair tile of every
// (tile, key tile) -- from the per-head tiles pair_tiles() writes or, through
// the per-head entry points, from the caller's [B][H][KL][QL] buffer -- into
// a 3-slot ring shared by both tiles in the order the scores are issued
// (key tile major, tile minor), and the MMA warp adds it to S_t as
// c·I·pairᵀ (c = 1/scale, exact) with the shifted identity of fa_sm100.cuh.
// With a causal mask the second tile sees one more key tile than the first.
// Every mbarrier wait is bounded; waits guarding warp-wide tcgen05.ld/st are
// warp-uniform.
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

constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kThreads = 384;
constexpr int kMaxKeyWords = 2048;   // validity bits for up to 65536 keys
constexpr unsigned kFull = 0xffffffffu;

enum Bar {
    kQFull = 0,
    kKFull = 1,      // +stage (up to 3)
    kVFull = 4,      // +stage
    kKVEmpty = 7,    // +stage
    kSFull = 10,     // +tile: S_t(j) in TMEM
    kPFull = 12,     // +tile: softmax done, P_t(j) in TMEM (128 arrivals)
    kOStep = 14,     // +tile: PV_t(j) retired
    kOFinal = 16,    // +tile: every PV_t retired
    kMmaDone = 18,
    kPairFull = 19,  // +slot (TMA -> MMA)
    kPairEmpty = 22, // +slot (its UMMAs retired -> producer)
    kNumBars = 25
};

constexpr int kPairSlots = 3;

template <int E, bool PAIR>
struct Layout2 {
    static constexpr int kStages = (E == 64 && !PAIR) ? 3 : 2;
    static constexpr int kQBytes = kBM * E * 2;
    static constexpr int kKVBytes = kBN * E * 2;
    static constexpr int kPairBytes = PAIR ? kBN * kBM * 2 : 0;
    static constexpr int kQ = 0;                               // 2 tiles
    static constexpr int kK = kQ + 2 * kQBytes;
    static constexpr int kV = kK + kStages * kKVBytes;
    static constexpr int kPair = kV + kStages * kKVBytes;
    static constexpr int kEye = kPair + kPairSlots * kPairBytes;   // 1024-aligned
    static constexpr int kBits = kEye + (PAIR ? kEyeBytes : 0);
    static constexpr int kBar = kBits + kMaxKeyWords * 4;
    static constexpr int kTmemSlot = kBar + kNumBars * 8;
    static constexpr int kTotal = kTmemSlot + 16;
    static constexpr int kAlloc = kTotal + 1024;               // slack for 1024-byte alignment
};
static_assert(Layout2<128, false>::kAlloc <= 227 * 1024, "shared memory");
static_assert(Layout2<64, false>::kAlloc <= 227 * 1024, "shared memory");
static_assert(Layout2<64, true>::kAlloc <= 227 * 1024, "shared memory");

template <typename T, int E, bool CAUSAL, bool PAIR, bool MASK>
__global__ void __launch_bounds__(kThreads, 1)
fa_fwd2_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_pair,
                     const Params p) {
    static_assert(!PAIR || E == 64, "pair tiles fit shared memory only for E = 64");
    using L = Layout2<E, PAIR>;
    constexpr int S = L::kStages;
    constexpr int W = kBN + E;   // TMEM columns per tile
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlot);
    uint32_t* bits = reinterpret_cast<uint32_t*>(smem + L::kBits);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t QL = p.QL, KL = p.KL;
    const int n_qt = (int)((QL + kBM - 1) / kBM);
    const int n_pairs = (n_qt + 1) / 2;
    const int pr = CAUSAL ? n_pairs - 1 - (int)blockIdx.y : (int)blockIdx.y;   // heavy pairs first
    const int h = blockIdx.x, b = blockIdx.z;
    const int kvh = h / p.n_rep;

    __shared__ int s_abort;
    __shared__ int s_kvlen;
    volatile int* ab = &s_abort;

    const int n_words = (int)((KL + 31) / 32);
    if (threadIdx.x == 0) s_kvlen = MASK ? 0 : (int)KL;
    __syncthreads();
    if (MASK) {
        const uint8_t* mg = p.kmask + (int64_t)b * KL;
        int best = 0;
        for (int w = threadIdx.x; w < n_words; w += kThreads) {
            uint32_t word = 0;
            for (int t = 0; t < 32; ++t) {
                const int64_t key = (int64_t)w * 32 + t;
                if (key < KL && mg[key]) word |= 1u << t;
            }
            bits[w] = word;
            if (word) best = max(best, w * 32 + 32 - __clz(word));
        }
        if (best) atomicMax(&s_kvlen, best);
    } else {
        for (int w = threadIdx.x; w < n_words; w += kThreads) {
            const int64_t n = KL - (int64_t)w * 32;
            bits[w] = n >= 32 ? 0xffffffffu : ((1u << n) - 1u);
        }
    }
    if (PAIR) {
        build_eye<T>(smem + L::kEye, 1.f / p.scale, threadIdx.x, kThreads);
        fence_proxy_async_smem();   // identity writes -> UMMA reads
    }
    if (threadIdx.x == 0) {
        s_abort = 0;
        mbar_init(&bars[kQFull], 1);
        for (int s = 0; s < S; ++s) {
            mbar_init(&bars[kKFull + s], 1);
            mbar_init(&bars[kVFull + s], 1);
            mbar_init(&bars[kKVEmpty + s], 1);
        }
        for (int t = 0; t < 2; ++t) {
            mbar_init(&bars[kSFull + t], 1);
            mbar_init(&bars[kPFull + t], 128);
            mbar_init(&bars[kOStep + t], 1);
            mbar_init(&bars[kOFinal + t], 1);
        }
        for (int i = 0; i < kPairSlots; ++i) {
            mbar_init(&bars[kPairFull + i], 1);
            mbar_init(&bars[kPairEmpty + i], 1);
        }
        mbar_init(&bars[kMmaDone], 1);
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
    const int64_t kv_len = s_kvlen;
    const int kv_tiles = (int)((kv_len + kBN - 1) / kBN);
    // key tiles of tile t (0 when the tile lies past QL)
    auto key_tiles = [&](int t) {
        const int64_t q0 = (int64_t)(2 * pr + t) * kBM;
        int n = q0 < QL ? kv_tiles : 0;
        if (CAUSAL && n > 0) {
            const int64_t i_end = q0 + kBM < QL ? q0 + kBM : QL;
            const int lim = (int)((i_end + kBN - 1) / kBN);
            n = n < lim ? n : lim;
        }
        return n;
    };
    const int nkt0 = key_tiles(0), nkt1 = key_tiles(1);
    const int n_kt = nkt0 > nkt1 ? nkt0 : nkt1;

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0 && n_kt > 0) {
            tma_prefetch(&tm_q);
            tma_prefetch(&tm_k);
            tma_prefetch(&tm_v);
            if (PAIR) tma_prefetch(&tm_pair);
            const int bh_q = b * p.QH + h, bh_k = b * p.KH + kvh;
            const int nq = nkt1 > 0 ? 2 : 1;
            mbar_expect_tx(&bars[kQFull], nq * L::kQBytes);
            for (int t = 0; t < nq; ++t)
#pragma unroll
                for (int e2 = 0; e2 < E / 64; ++e2)
                    tma_load_3d(smem + L::kQ + t * L::kQBytes + e2 * kBM * 128, &tm_q, &bars[kQFull], e2 * 64,
                                (2 * pr + t) * kBM, bh_q);
            // pair tiles of key tile j (both query tiles), the u-th into slot
            // u % 3 once the scores that read tile u - 3 have retired
            int pair_issued = 0;
            auto load_pairs = [&](int j) -> bool {
                for (int t = 0; t < 2; ++t) {
                    if (j >= (t ? nkt1 : nkt0)) continue;
                    const int u = pair_issued, slot = u % kPairSlots;
                    if (u >= kPairSlots && !wait(&bars[kPairEmpty + slot], ((u / kPairSlots) - 1) & 1, ab, 13))
                        return false;
                    mbar_expect_tx(&bars[kPairFull + slot], L::kPairBytes);
                    const int qt = 2 * pr + t;
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        uint8_t* dst = smem + L::kPair + slot * L::kPairBytes + half * kBN * 128;
                        if (p.pair_per_head)   // [B·H][KL][QL]: queries qt·128 + half·64.., keys j·128..
                            tma_load_3d(dst, &tm_pair, &bars[kPairFull + slot], qt * kBM + half * 64, j * kBN, bh_q);
                        else                   // per-head tiles [B·H][QLp/128][KLp][128]
                            tma_load_4d(dst, &tm_pair, &bars[kPairFull + slot], half * 64, j * kBN, qt, bh_q);
                    }
                    pair_issued = u + 1;
                }
                return true;
            };
            int issued = 0;
            bool run = !PAIR || load_pairs(0);
            for (int j = 0; run && j < n_kt; ++j) {
                const int s = j % S;
                if (j >= S && !wait(&bars[kKVEmpty + s], ((j / S) - 1) & 1, ab, 1)) break;
                issued = j + 1;
                mbar_expect_tx(&bars[kKFull + s], L::kKVBytes);
#pragma unroll
                for (int e2 = 0; e2 < E / 64; ++e2)
                    tma_load_3d(smem + L::kK + s * L::kKVBytes + e2 * kBN * 128, &tm_k, &bars[kKFull + s], e2 * 64,
                                j * kBN, bh_k);
                mbar_expect_tx(&bars[kVFull + s], L::kKVBytes);
#pragma unroll
                for (int e2 = 0; e2 < E / 64; ++e2)
                    tma_load_3d(smem + L::kV + s * L::kKVBytes + e2 * kBN * 128, &tm_v, &bars[kVFull + s], e2 * 64,
                                j * kBN, bh_k);
                if (PAIR && j + 1 < n_kt) run = load_pairs(j + 1);
            }
            // copies still in flight land before the CTA exits
            wait(&bars[kQFull], 0, ab, 2);
            for (int j = issued - S < 0 ? 0 : issued - S; j < issued; ++j) {
                wait(&bars[kKFull + j % S], (j / S) & 1, ab, 3);
                wait(&bars[kVFull + j % S], (j / S) & 1, ab, 3);
            }
            for (int u = pair_issued - kPairSlots < 0 ? 0 : pair_issued - kPairSlots; u < pair_issued; ++u)
                wait(&bars[kPairFull + u % kPairSlots], (u / kPairSlots) & 1, ab, 14);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        constexpr uint32_t idesc_s = idesc_f16<kBF16>(kBM, kBN, false, false);
        constexpr uint32_t idesc_o = idesc_f16<kBF16>(kBM, E, false, true);
        bool ok = n_kt > 0 && wait_warp(&bars[kQFull], 0, ab, 4);
        const uint32_t sEye = smem_u32(smem + L::kEye);
        int u_pair = 0;   // pair tiles consumed, in the producer's order
        // the pair tile of the next score MMA has landed (warp-uniform)
        auto pair_ready = [&]() -> bool {
            return !PAIR || wait_warp(&bars[kPairFull + u_pair % kPairSlots], (u_pair / kPairSlots) & 1, ab, 15);
        };
        // operand descriptors, built once and stepped with desc_add
        const uint64_t dQ0 = desc_k_sw128(smem_u32(smem + L::kQ)), dK0 = desc_k_sw128(smem_u32(smem + L::kK));
        const uint64_t dV0 = desc_mn_sw128(smem_u32(smem + L::kV), kBN * 128);
        const uint64_t dEye = desc_k_sw128(sEye), dP0 = desc_k_sw128(smem_u32(smem + L::kPair));
        auto issue_s = [&](int t, int j) {   // S_t(j) = Q_t·K_jᵀ (+ c·I·pairᵀ), lane 0
            const uint64_t bq = desc_add(dQ0, (uint32_t)t * L::kQBytes);
            const uint64_t bk = desc_add(dK0, (uint32_t)(j % S) * L::kKVBytes);
#pragma unroll
            for (int kk = 0; kk < E / 16; ++kk) {
                const uint32_t off_q = (kk / 4) * kBM * 128 + (kk % 4) * 32;
                const uint32_t off_k = (kk / 4) * kBN * 128 + (kk % 4) * 32;
                umma_ss(tmem + t * W, desc_add(bq, off_q), desc_add(bk, off_k), idesc_s, kk > 0 ? 1u : 0u);
            }
            if (PAIR) {
                // B = pair tile [key][query], K-major over queries
                const int slot = u_pair % kPairSlots;
                const uint64_t bp = desc_add(dP0, (uint32_t)slot * L::kPairBytes);
#pragma unroll
                for (int kk = 0; kk < kBM / 16; ++kk)
                    umma_ss(tmem + t * W, desc_add(dEye, eye_step(0, kk)),
                            desc_add(bp, (kk / 4) * kBN * 128 + (kk % 4) * 32), idesc_s, 1u);
                umma_commit(&bars[kPairEmpty + slot]);
            }
            umma_commit(&bars[kSFull + t]);
        };
        if (ok) ok = wait_warp(&bars[kKFull], 0, ab, 5);
        for (int t = 0; ok && t < 2; ++t) {
            if ((t ? nkt1 : nkt0) == 0) continue;
            if (!pair_ready()) { ok = false; break; }
            tc_fence_after();
            if (lane == 0) issue_s(t, 0);
            __syncwarp();
            if (PAIR) ++u_pair;
        }
        for (int j = 0; ok && j < n_kt; ++j) {
            const int s = j % S;
            if (!wait_warp(&bars[kVFull + s], (j / S) & 1, ab, 6)) break;
            const bool next = j + 1 < n_kt;
            if (next && !wait_warp(&bars[kKFull + (j + 1) % S], ((j + 1) / S) & 1, ab, 7)) break;
            for (int t = 0; t < 2; ++t) {
                const int nk_t = t ? nkt1 : nkt0;
                if (j >= nk_t) continue;
                if (!wait_warp(&bars[kPFull + t], j & 1, ab, 8)) { ok = false; break; }
                const bool more = j + 1 < nk_t;
                if (more && !pair_ready()) { ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
                    const uint64_t bv = desc_add(dV0, (uint32_t)s * L::kKVBytes);
                    const uint32_t acc0 = j > 0 ? 1u : 0u;
#pragma unroll
                    for (int kk = 0; kk < kBN / 16; ++kk)
                        umma_ts(tmem + t * W + kBN, tmem + t * W + kk * 8, desc_add(bv, kk * 16 * 128), idesc_o,
                                kk > 0 ? 1u : acc0);
                    umma_commit(&bars[kOStep + t]);
                    if (!more) umma_commit(&bars[kOFinal + t]);
                    else issue_s(t, j + 1);   // behind PV_t(j), which reads P_t(j) from the same columns
                }
                __syncwarp();
                if (PAIR && more) ++u_pair;
            }
            if (!ok) break;
            if (lane == 0) umma_commit(&bars[kKVEmpty + s]);   // K_j, V_j read by every MMA issued so far
            __syncwarp();
        }
        if (n_kt > 0) {
            if (lane == 0) umma_commit(&bars[kMmaDone]);
            __syncwarp();
            wait(&bars[kMmaDone], 0, ab, 9);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------ softmax (tile t)
        const int t = (warp - 4) >> 2;
        const int r = (threadIdx.x - 128) & 127;
        const int64_t q0 = (int64_t)(2 * pr + t) * kBM;
        const int64_t i = q0 + r;
        const int nk = t ? nkt1 : nkt0;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + t * W + lane_off, tO = tS + kBN;
        const float sl2 = p.scale * kLog2e;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nk; ++j) {
            const int64_t k0 = (int64_t)j * kBN;
            if (!wait_warp(&bars[kSFull + t], j & 1, ab, 10)) { ok = false; break; }
            tc_fence_after();
            uint32_t raw[kBN];
#pragma unroll
            for (int c = 0; c < kBN / 32; ++c)
                tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(raw + c * 32));
            uint32_t vb[kBN / 32];
#pragma unroll
            for (int c = 0; c < kBN / 32; ++c) vb[c] = (k0 + c * 32 < KL) ? bits[(k0 >> 5) + c] : 0u;
            const int64_t kr64 = i - k0;
            const int kr = (int)(kr64 < 0 ? -1 : (kr64 > kBN ? kBN : kr64));
            const bool full = (!CAUSAL || kr >= kBN - 1) && (vb[0] & vb[1] & vb[2] & vb[3]) == 0xffffffffu;
            tmem_ld_wait();
            if (!full) {
#pragma unroll
                for (int u = 0; u < kBN; ++u) {
                    bool valid = (vb[u >> 5] >> (u & 31)) & 1u;
                    if (CAUSAL) valid = valid && (u <= kr);
                    raw[u] = valid ? raw[u] : __float_as_uint(-INFINITY);
                }
            }
            float mp[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) mp[u] = __uint_as_float(raw[u]);
#pragma unroll
            for (int u = 8; u < kBN; ++u) mp[u & 7] = fmaxf(mp[u & 7], __uint_as_float(raw[u]));
            const float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                                   fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7]))) * sl2;
            float alpha = 1.f;
            const float m_new = fmaxf(m, mx);
            if (m_new > m + 8.f) {
                alpha = ex2(m - m_new);
                m = m_new;
            }
            const float m_use = (m == -INFINITY) ? 0.f : m;
            float sp[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) sp[u] = 0.f;
#pragma unroll
            for (int c = 0; c < kBN / 32; ++c) {
                uint32_t pk[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    const float p0 = ex2(fmaf(__uint_as_float(raw[c * 32 + 2 * u]), sl2, -m_use));
                    const float p1 = ex2(fmaf(__uint_as_float(raw[c * 32 + 2 * u + 1]), sl2, -m_use));
                    sp[(2 * u) & 7] += p0;
                    sp[(2 * u + 1) & 7] += p1;
                    pk[u] = pack16<T>(p0, p1);
                }
                tmem_st16(tS + c * 16, pk);
            }
            const float ls = ((sp[0] + sp[1]) + (sp[2] + sp[3])) + ((sp[4] + sp[5]) + (sp[6] + sp[7]));
            l = l * alpha + ls;
            if (__any_sync(kFull, j > 0 && alpha != 1.f)) {
                // O_t holds Σ_{<j} P·V: PV_t(j-1) must have retired
                if (!wait_warp(&bars[kOStep + t], (j - 1) & 1, ab, 11)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < E / 32; ++c) {
                    uint32_t ov[32];
                    tmem_ld32(tO + c * 32, ov);
                    tmem_ld_wait();
#pragma unroll
                    for (int u = 0; u < 32; ++u) ov[u] = __float_as_uint(__uint_as_float(ov[u]) * alpha);
                    tmem_st32(tO + c * 32, ov);
                }
            }
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&bars[kPFull + t]);
        }
        // epilogue
        if (q0 < QL) {
            T* og = reinterpret_cast<T*>(p.o) + (((int64_t)b * p.QH + h) * QL) * E;
            if (i < QL) {
                const float m_use = (m == -INFINITY) ? 0.f : m;
                p.lse[((int64_t)b * p.QH + h) * QL + i] = m_use * 0.6931471805599453f + logf(l);
            }
            bool have_o = nk > 0 && __all_sync(kFull, ok);
            if (have_o) have_o = wait_warp(&bars[kOFinal + t], 0, ab, 12);
            if (have_o) {
                tc_fence_after();
                const float inv = 1.0f / l;
#pragma unroll
                for (int c = 0; c < E / 32; ++c) {
                    uint32_t ov[32];
                    tmem_ld32(tO + c * 32, ov);
                    tmem_ld_wait();
                    if (i < QL) {
                        uint32_t pk[16];
#pragma unroll
                        for (int u = 0; u < 16; ++u)
                            pk[u] = pack16<T>(__uint_as_float(ov[2 * u]) * inv, __uint_as_float(ov[2 * u + 1]) * inv);
                        uint4* dst = reinterpret_cast<uint4*>(og + i * E + c * 32);
#pragma unroll
                        for (int v = 0; v < 4; ++v)
                            dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
                    }
                }
            } else if (i < QL) {
                // no visible key (or a timed-out wait): 0/0, as the reference yields
                const T nanv = from_f<T>(__int_as_float(0x7fc00000));
                for (int e = 0; e < E; ++e) og[i * E + e] = nanv;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

template <typename T, int E, bool CAUSAL, bool PAIR, bool MASK>
int launch2(const Params& p, const void* pair_tiles, cudaStream_t s) {
    using Lay = Layout2<E, PAIR>;
    constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
    const int64_t qlp = (p.QL + 127) / 128 * 128, klp = (p.KL + 127) / 128 * 128;
    CUtensorMap tq, tk, tv, tp;
    memset(&tp, 0, sizeof(tp));
    if (!make_map(&tq, p.q, E, p.QL, (int64_t)p.B * p.QH, kBM, bf16) ||
        !make_map(&tk, p.k, E, p.KL, (int64_t)p.B * p.KH, kBN, bf16) ||
        !make_map(&tv, p.v, E, p.KL, (int64_t)p.B * p.KH, kBN, bf16) ||
        (PAIR && !(p.pair_per_head ? make_per_head_map(&tp, p.pair, p.QL, p.KL, (int64_t)p.B * p.QH, bf16)
                                   : make_tiles_map(&tp, pair_tiles, qlp, klp, (int64_t)p.B * p.QH, bf16))))
        return fail(NNOP_ERR_CUDA, "flash_attention_fwd: cuTensorMapEncodeTiled failed");
    auto kern = fa_fwd2_sm100_kernel<T, E, CAUSAL, PAIR, MASK>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kAlloc) != cudaSuccess)
        return fail(NNOP_ERR_CUDA, "flash_attention_fwd: cannot set shared memory size");
    const int n_qt = (int)((p.QL + kBM - 1) / kBM);
    dim3 grid(p.QH, (unsigned)((n_qt + 1) / 2), p.B);
    kern<<<grid, kThreads, Lay::kAlloc, s>>>(tq, tk, tv, tp, p);
    return check_launch("flash_attention_fwd (sm100, two tiles)");
}

template <typename T, int E, bool CAUSAL>
int dispatch2_flags(const Params& p, const void* pair_tiles, cudaStream_t s) {
    const bool pair = p.pair != nullptr, mask = p.kmask != nullptr;
    if constexpr (E == 64) {
        if (pair) return mask ? launch2<T, 64, CAUSAL, true, true>(p, pair_tiles, s)
                              : launch2<T, 64, CAUSAL, true, false>(p, pair_tiles, s);
    }
    return mask ? launch2<T, E, CAUSAL, false, true>(p, pair_tiles, s)
                : launch2<T, E, CAUSAL, false, false>(p, pair_tiles, s);
}

template <typename T, int E>
int dispatch2(const Params& p, const void* pair_tiles, bool causal, cudaStream_t s) {
    return causal ? dispatch2_flags<T, E, true>(p, pair_tiles, s) : dispatch2_flags<T, E, false>(p, pair_tiles, s);
}

}  // namespace

// Reads and clears the bounded-wait timeout flags of this file's kernel.
int sm100_fwd2_timeouts() {
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, sm100::g_wait_timeout, sizeof(int));
    cudaMemcpyToSymbol(sm100::g_wait_timeout, &z, sizeof(int));
    return v;
}

// The forward for bf16/f16, E 64 or 128; with a pair bias E = 64 only, the
// bias from the per-head tiles (pair_tiles) or, with p.pair_per_head, from
// the caller's per-head buffer.
int sm100_fwd2(const Params& p, const void* pair_tiles, int dtype, bool causal, cudaStream_t s) {
    if (dtype == NNOP_BF16)
        return p.E == 64 ? dispatch2<__nv_bfloat16, 64>(p, pair_tiles, causal, s)
                         : dispatch2<__nv_bfloat16, 128>(p, pair_tiles, causal, s);
    return p.E == 64 ? dispatch2<__half, 64>(p, pair_tiles, causal, s) : dispatch2<__half, 128>(p, pair_tiles, causal, s);
}

}  // namespace fa
}  // namespace nnop
