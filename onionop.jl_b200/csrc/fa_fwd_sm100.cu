// Flash-attention forward on the sm_100a tensor cores (tcgen05 UMMA, TMEM
// accumulators, TMA-fed tiles), bf16/f16, E in {64, 128}.
//
// Reference: `_flash_attention_fwd!` (src/attention.jl:8-143) -- one thread
// per query row with the scores in shared memory and WMMA 16x16x16 tiles.
//
// One CTA per (128-query tile, query head, batch); 256 threads:
//   warp 0     TMA producer: Q once, then K_j / V_j into a 2-stage ring and,
//              with a pair bias, the pair tile of (q-tile, k-tile j, head)
//              from the key-major per-head copy pair_tiles() writes
//              ([B][H][QL/128][KL][128], two 64-query boxes: [key][query]);
//   warp 1     MMA issuer: S_j = Q·K_jᵀ into one of two TMEM score buffers,
//              plus, with a pair bias, S_j += c·I·pair_jᵀ (c = 1/scale; the
//              pair tile is the K-major B operand of a 128x128x128 UMMA
//              whose A is the shifted identity of fa_sm100.cuh -- exact,
//              since c is a power of two and products accumulate in fp32),
//              O += P_j·V_j with P_j read from TMEM (tcgen05 "ts" form);
//   warps 4-7  softmax: thread r owns query row r (TMEM lane r): it reads
//              its 128 scores (bias included), masks, updates the running
//              max (rescaling O in TMEM only when the max grows by more than
//              2^8 -- the stale max keeps exp2 values <= 256), writes P as
//              16-bit values back into the score columns, and finally
//              normalises O and writes o and lse.
// Key validity (padding mask, ragged tail) is one bit per key, built once per
// CTA in shared memory.  TMEM: S0 [0,128), S1 [128,256), O [256, 256+E).
// Every mbarrier wait is bounded (sm100::wait); waits that guard warp-wide
// tcgen05.ld/st are made warp-uniform (__all_sync) so a timed-out lane never
// leaves its warp divergent at an .aligned instruction.
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
constexpr int kStages = 2;
constexpr int kPairSlots = 3;        // pair tiles in flight (loaded two key tiles ahead)
constexpr int kThreads = 256;
constexpr int kMaxKeyWords = 2048;   // validity bits for up to 65536 keys
constexpr unsigned kFull = 0xffffffffu;

enum Bar {
    kQFull = 0,
    kKFull = 1,      // +stage
    kVFull = 3,      // +stage
    kKVEmpty = 5,    // +stage
    kSFull = 7,      // +buffer
    kPFull = 9,      // +buffer
    kOFinal = 11,
    kOStep = 12,
    kPairFull = 13,  // +slot (TMA -> MMA)
    kPairEmpty = 16, // +slot (its UMMAs retired -> producer)
    kMmaDone = 19,   // MMA warp's own "all my MMAs retired" barrier
    kNumBars = 20
};

template <int E, bool PAIR>
struct Layout {
    static constexpr int kQBytes = kBM * E * 2;
    static constexpr int kKVBytes = kBN * E * 2;
    static constexpr int kQ = 0;
    static constexpr int kK = kQ + kQBytes;
    static constexpr int kV = kK + kStages * kKVBytes;
    static constexpr int kPairBytes = PAIR ? kBN * kBM * 2 : 0;
    static constexpr int kPair = kV + kStages * kKVBytes;
    static constexpr int kEye = kPair + kPairSlots * kPairBytes;  // shifted identity (1024-aligned)
    static constexpr int kBits = kEye + (PAIR ? kEyeBytes : 0); // kMaxKeyWords uint32
    static constexpr int kBar = kBits + kMaxKeyWords * 4;
    static constexpr int kTmemSlot = kBar + kNumBars * 8;
    static constexpr int kTotal = kTmemSlot + 16;
    static constexpr int kAlloc = kTotal + 1024;                // slack for 1024-byte alignment
};

template <typename T, int E, bool CAUSAL, bool PAIR, bool MASK>
__global__ void __launch_bounds__(kThreads, 1)
fa_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_pair,
                    const Params p) {
    using L = Layout<E, PAIR>;
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlot);
    uint32_t* bits = reinterpret_cast<uint32_t*>(smem + L::kBits);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t QL = p.QL, KL = p.KL;
    const int n_qt = (int)((QL + kBM - 1) / kBM);
    const int qt = CAUSAL ? n_qt - 1 - (int)blockIdx.y : (int)blockIdx.y;
    const int h = blockIdx.x, b = blockIdx.z;
    const int kvh = h / p.n_rep;
    const int64_t q0 = (int64_t)qt * kBM;

    __shared__ int s_abort;   // set by the first wait of this CTA that gives up
    __shared__ int s_kvlen;   // last kept key + 1
    volatile int* ab = &s_abort;

    // key-validity bits (padding mask and ragged tail) and the kept length
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
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars[kKFull + s], 1);
            mbar_init(&bars[kVFull + s], 1);
            mbar_init(&bars[kKVEmpty + s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars[kSFull + i], 1);
            mbar_init(&bars[kPFull + i], 128);
        }
        for (int i = 0; i < kPairSlots; ++i) {
            mbar_init(&bars[kPairFull + i], 1);
            mbar_init(&bars[kPairEmpty + i], 1);
        }
        mbar_init(&bars[kOFinal], 1);
        mbar_init(&bars[kOStep], 1);
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
    const uint32_t tS0 = tmem, tS1 = tmem + kBN, tO = tmem + 2 * kBN;
    const int64_t kv_len = s_kvlen;
    int n_kt = (int)((kv_len + kBN - 1) / kBN);
    if (CAUSAL) {
        const int64_t i_end = q0 + kBM < QL ? q0 + kBM : QL;
        const int lim = (int)((i_end + kBN - 1) / kBN);
        n_kt = n_kt < lim ? n_kt : lim;
    }

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0 && n_kt > 0) {
            tma_prefetch(&tm_q);
            tma_prefetch(&tm_k);
            tma_prefetch(&tm_v);
            if (PAIR) tma_prefetch(&tm_pair);
            const int bh_q = b * p.QH + h, bh_k = b * p.KH + kvh;
            mbar_expect_tx(&bars[kQFull], L::kQBytes);
#pragma unroll
            for (int half = 0; half < E / 64; ++half)
                tma_load_3d(smem + L::kQ + half * kBM * 128, &tm_q, &bars[kQFull], half * 64, (int)q0, bh_q);
            int issued = 0, pair_issued = 0;
            // pair tile of key tile j into slot j % 3 once tile j - 3 has been consumed
            auto load_pair = [&](int j) -> bool {
                const int slot = j % kPairSlots;
                if (j >= kPairSlots && !wait(&bars[kPairEmpty + slot], ((j / kPairSlots) - 1) & 1, ab, 2))
                    return false;
                mbar_expect_tx(&bars[kPairFull + slot], L::kPairBytes);
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint8_t* dst = smem + L::kPair + slot * L::kPairBytes + half * kBN * 128;
                    if (p.pair_per_head)   // [B·H][KL][QL]: queries qt·128 + half·64.., keys j·128..
                        tma_load_3d(dst, &tm_pair, &bars[kPairFull + slot], qt * kBM + half * 64, j * kBN, bh_q);
                    else                   // per-head tiles [B·H][QLp/128][KLp][128]
                        tma_load_4d(dst, &tm_pair, &bars[kPairFull + slot], half * 64, j * kBN, qt, bh_q);
                }
                pair_issued = j + 1;
                return true;
            };
            bool run = true;
            if (PAIR) run = load_pair(0) && (n_kt < 2 || load_pair(1));
            for (int j = 0; run && j < n_kt; ++j) {
                const int s = j % kStages;
                if (j >= kStages && !wait(&bars[kKVEmpty + s], ((j / kStages) - 1) & 1, ab, 1)) break;
                issued = j + 1;
                const int k0 = j * kBN;
                mbar_expect_tx(&bars[kKFull + s], L::kKVBytes);
#pragma unroll
                for (int half = 0; half < E / 64; ++half)
                    tma_load_3d(smem + L::kK + s * L::kKVBytes + half * kBN * 128, &tm_k, &bars[kKFull + s],
                                half * 64, k0, bh_k);
                mbar_expect_tx(&bars[kVFull + s], L::kKVBytes);
#pragma unroll
                for (int half = 0; half < E / 64; ++half)
                    tma_load_3d(smem + L::kV + s * L::kKVBytes + half * kBN * 128, &tm_v, &bars[kVFull + s],
                                half * 64, k0, bh_k);
                if (PAIR && j + 2 < n_kt) run = load_pair(j + 2);
            }
            // Copies still in flight must land before the CTA can exit (they
            // have, unless a consumer gave up): bounded waits on the last ones.
            wait(&bars[kQFull], 0, ab, 3);
            for (int j = issued - kStages < 0 ? 0 : issued - kStages; j < issued; ++j) {
                wait(&bars[kKFull + j % kStages], (j / kStages) & 1, ab, 4);
                wait(&bars[kVFull + j % kStages], (j / kStages) & 1, ab, 5);
            }
            for (int j = pair_issued - kPairSlots < 0 ? 0 : pair_issued - kPairSlots; j < pair_issued; ++j)
                wait(&bars[kPairFull + j % kPairSlots], (j / kPairSlots) & 1, ab, 6);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        constexpr uint32_t idesc_s = idesc_f16<kBF16>(kBM, kBN, false, false);
        constexpr uint32_t idesc_o = idesc_f16<kBF16>(kBM, E, false, true);
        const uint32_t sQ = smem_u32(smem + L::kQ);
        bool ok = n_kt > 0 && wait_warp(&bars[kQFull], 0, ab, 7);
        const uint32_t sEye = smem_u32(smem + L::kEye);
        auto issue_s = [&](int j) -> bool {
            const int s = j % kStages;
            if (!wait_warp(&bars[kKFull + s], (j / kStages) & 1, ab, 8)) return false;
            if (PAIR && !wait_warp(&bars[kPairFull + j % kPairSlots], (j / kPairSlots) & 1, ab, 12)) return false;
            tc_fence_after();
            if (lane == 0) {
                const uint32_t sK = smem_u32(smem + L::kK + s * L::kKVBytes);
                const uint32_t d = (j & 1) ? tS1 : tS0;
#pragma unroll
                for (int kk = 0; kk < E / 16; ++kk) {
                    const uint32_t off_q = (kk / 4) * kBM * 128 + (kk % 4) * 32;
                    const uint32_t off_k = (kk / 4) * kBN * 128 + (kk % 4) * 32;
                    umma_ss(d, desc_k_sw128(sQ + off_q), desc_k_sw128(sK + off_k), idesc_s, kk > 0 ? 1u : 0u);
                }
                if (PAIR) {
                    // S += c·I·pairᵀ: B = pair tile [key][query], K-major over queries
                    const uint32_t sP = smem_u32(smem + L::kPair + (j % kPairSlots) * L::kPairBytes);
#pragma unroll
                    for (int kk = 0; kk < kBM / 16; ++kk)
                        umma_ss(d, desc_k_sw128(eye_step(sEye, kk)),
                                desc_k_sw128(sP + (kk / 4) * kBN * 128 + (kk % 4) * 32), idesc_s, 1u);
                    umma_commit(&bars[kPairEmpty + j % kPairSlots]);
                }
                umma_commit(&bars[kSFull + (j & 1)]);
            }
            __syncwarp();
            return true;
        };
        if (ok) ok = issue_s(0);
        for (int j = 0; ok && j < n_kt; ++j) {
            if (j + 1 < n_kt && !issue_s(j + 1)) break;
            const int s = j % kStages;
            if (!wait_warp(&bars[kPFull + (j & 1)], (j >> 1) & 1, ab, 9)) break;
            if (!wait_warp(&bars[kVFull + s], (j / kStages) & 1, ab, 10)) break;
            tc_fence_after();
            if (lane == 0) {
                const uint32_t sV = smem_u32(smem + L::kV + s * L::kKVBytes);
                const uint32_t a = (j & 1) ? tS1 : tS0;
#pragma unroll
                for (int kk = 0; kk < kBN / 16; ++kk) {
                    umma_ts(tO, a + kk * 8, desc_mn_sw128(sV + kk * 16 * 128, kBN * 128), idesc_o,
                            (j > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(&bars[kKVEmpty + s]);
                umma_commit(&bars[kOStep]);
                if (j == n_kt - 1) umma_commit(&bars[kOFinal]);
            }
            __syncwarp();
        }
        // Every MMA this warp issued retires before TMEM is released.
        if (n_kt > 0) {
            if (lane == 0) umma_commit(&bars[kMmaDone]);
            __syncwarp();
            wait(&bars[kMmaDone], 0, ab, 11);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------ softmax
        const int r = threadIdx.x - 128;
        const int64_t i = q0 + r;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const float sl2 = p.scale * kLog2e;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < n_kt; ++j) {
            const int buf = j & 1;
            const int64_t k0 = (int64_t)j * kBN;
            if (!wait_warp(&bars[kSFull + buf], (j >> 1) & 1, ab, 13)) { ok = false; break; }
            tc_fence_after();
            const uint32_t tS = (buf ? tS1 : tS0) + lane_off;
            // all four 32-column loads in flight at once
            uint32_t raw[kBN];
#pragma unroll
            for (int c = 0; c < kBN / 32; ++c)
                tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(raw + c * 32));
            // words past the last key are never read: k0 + c·32 < n_words·32 here
            uint32_t vb[kBN / 32];
#pragma unroll
            for (int c = 0; c < kBN / 32; ++c) vb[c] = (k0 + c * 32 < KL) ? bits[(k0 >> 5) + c] : 0u;
            // keys k0 + t visible to this row: t <= kr (causal)
            const int64_t kr64 = i - k0;
            const int kr = (int)(kr64 < 0 ? -1 : (kr64 > kBN ? kBN : kr64));
            const bool full = (!CAUSAL || kr >= kBN - 1) && (vb[0] & vb[1] & vb[2] & vb[3]) == 0xffffffffu;
            tmem_ld_wait();
            float x[kBN];
            if (full) {
#pragma unroll
                for (int t = 0; t < kBN; ++t) x[t] = __uint_as_float(raw[t]) * sl2;
            } else {
#pragma unroll
                for (int t = 0; t < kBN; ++t) {
                    bool valid = (vb[t >> 5] >> (t & 31)) & 1u;
                    if (CAUSAL) valid = valid && (t <= kr);
                    x[t] = valid ? __uint_as_float(raw[t]) * sl2 : -INFINITY;
                }
            }
            // row max and sum over 8 independent partials (short dependency chains)
            float mp[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) mp[u] = x[u];
#pragma unroll
            for (int t = 8; t < kBN; ++t) mp[t & 7] = fmaxf(mp[t & 7], x[t]);
            const float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                                   fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
            float alpha = 1.f;
            const float m_new = fmaxf(m, mx);
            const bool resc = m_new > m + 8.f;
            if (resc) {
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
                for (int t = 0; t < 16; ++t) {
                    const float p0 = ex2(x[c * 32 + 2 * t] - m_use);
                    const float p1 = ex2(x[c * 32 + 2 * t + 1] - m_use);
                    sp[(2 * t) & 7] += p0;
                    sp[(2 * t + 1) & 7] += p1;
                    pk[t] = pack16<T>(p0, p1);
                }
                tmem_st16(tS + c * 16, pk);
            }
            const float ls = ((sp[0] + sp[1]) + (sp[2] + sp[3])) + ((sp[4] + sp[5]) + (sp[6] + sp[7]));
            l = l * alpha + ls;
            // O rescale: the decision is per row, the TMEM access per warp, so
            // the whole warp takes the branch when any of its rows needs it
            // (the others multiply by alpha = 1).
            if (__any_sync(kFull, j > 0 && alpha != 1.f)) {
                // O holds Σ_{<j} P·V; PV_{j-1} must be complete before rescaling.
                if (!wait_warp(&bars[kOStep], (j - 1) & 1, ab, 14)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < E / 32; ++c) {
                    uint32_t raw[32];
                    tmem_ld32(tO + lane_off + c * 32, raw);
                    tmem_ld_wait();
#pragma unroll
                    for (int t = 0; t < 32; ++t) raw[t] = __float_as_uint(__uint_as_float(raw[t]) * alpha);
                    tmem_st32(tO + lane_off + c * 32, raw);
                }
            }
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&bars[kPFull + buf]);
        }
        // epilogue
        T* og = reinterpret_cast<T*>(p.o) + (((int64_t)b * p.QH + h) * QL) * E;
        if (i < QL) {
            const float m_use = (m == -INFINITY) ? 0.f : m;
            p.lse[((int64_t)b * p.QH + h) * QL + i] = m_use * 0.6931471805599453f + logf(l);
        }
        bool have_o = n_kt > 0 && __all_sync(kFull, ok);
        if (have_o) have_o = wait_warp(&bars[kOFinal], 0, ab, 15);
        if (have_o) {
            tc_fence_after();
            const float inv = 1.0f / l;
#pragma unroll
            for (int c = 0; c < E / 32; ++c) {
                uint32_t raw[32];
                tmem_ld32(tO + lane_off + c * 32, raw);
                tmem_ld_wait();
                if (i < QL) {
                    uint32_t pk[16];
#pragma unroll
                    for (int t = 0; t < 16; ++t)
                        pk[t] = pack16<T>(__uint_as_float(raw[2 * t]) * inv, __uint_as_float(raw[2 * t + 1]) * inv);
                    uint4* dst = reinterpret_cast<uint4*>(og + i * E + c * 32);
#pragma unroll
                    for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
                }
            }
        } else if (i < QL) {
            // no visible key (or a timed-out wait): 0/0, as the reference yields
            const T nanv = from_f<T>(__int_as_float(0x7fc00000));
            for (int e = 0; e < E; ++e) og[i * E + e] = nanv;
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
int launch(const Params& p, const void* pair_tiles, cudaStream_t s) {
    using Lay = Layout<E, PAIR>;
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
    auto kern = fa_fwd_sm100_kernel<T, E, CAUSAL, PAIR, MASK>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kAlloc) != cudaSuccess)
        return fail(NNOP_ERR_CUDA, "flash_attention_fwd: cannot set shared memory size");
    dim3 grid(p.QH, (unsigned)((p.QL + kBM - 1) / kBM), p.B);
    kern<<<grid, kThreads, Lay::kAlloc, s>>>(tq, tk, tv, tp, p);
    return check_launch("flash_attention_fwd (sm100)");
}

template <typename T, int E, bool CAUSAL>
int dispatch_flags(const Params& p, const void* pair_tiles, cudaStream_t s) {
    const bool pair = p.pair != nullptr, mask = p.kmask != nullptr;
    if constexpr (E == 64) {
        if (pair && mask) return launch<T, 64, CAUSAL, true, true>(p, pair_tiles, s);
        if (pair) return launch<T, 64, CAUSAL, true, false>(p, pair_tiles, s);
    }
    if (mask) return launch<T, E, CAUSAL, false, true>(p, pair_tiles, s);
    return launch<T, E, CAUSAL, false, false>(p, pair_tiles, s);
}

}  // namespace

// Shapes this kernel covers; the others use the mma.sync kernels.  With a pair
// bias the per-head pair tiles must have been written to the workspace.
bool sm100_fwd_supported(const Params& p, int dtype, bool have_pair_tiles) {
    if (dtype != NNOP_BF16 && dtype != NNOP_F16) return false;
    if ((p.KL + 31) / 32 > kMaxKeyWords) return false;
    if (p.pair) return p.E == 64 && have_pair_tiles;   // E=128 pair tiles exceed shared memory
    return p.E == 64 || p.E == 128;
}

// Reads and clears the bounded-wait timeout flags of this file's kernels.
int sm100_fwd_timeouts() {
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, sm100::g_wait_timeout, sizeof(int));
    cudaMemcpyToSymbol(sm100::g_wait_timeout, &z, sizeof(int));
    return v;
}

int sm100_fwd2(const Params& p, const void* pair_tiles, int dtype, bool causal, cudaStream_t s);

int sm100_fwd(const Params& p, const void* pair_tiles, int dtype, bool causal, cudaStream_t s) {
    // two query tiles per CTA in ping-pong (fa_fwd2_sm100.cu) for every shape
    // this file's kernel takes; NNOP_B200_FA=one_tile selects this file's
    // kernel (the tests check both)
    const char* v = getenv("NNOP_B200_FA");
    if (!(v && strcmp(v, "one_tile") == 0)) return sm100_fwd2(p, pair_tiles, dtype, causal, s);
    if (dtype == NNOP_BF16) {
        if (p.E == 64)
            return causal ? dispatch_flags<__nv_bfloat16, 64, true>(p, pair_tiles, s)
                          : dispatch_flags<__nv_bfloat16, 64, false>(p, pair_tiles, s);
        return causal ? dispatch_flags<__nv_bfloat16, 128, true>(p, pair_tiles, s)
                      : dispatch_flags<__nv_bfloat16, 128, false>(p, pair_tiles, s);
    }
    if (p.E == 64)
        return causal ? dispatch_flags<__half, 64, true>(p, pair_tiles, s) : dispatch_flags<__half, 64, false>(p, pair_tiles, s);
    return causal ? dispatch_flags<__half, 128, true>(p, pair_tiles, s) : dispatch_flags<__half, 128, false>(p, pair_tiles, s);
}

}  // namespace fa
}  // namespace nnop
