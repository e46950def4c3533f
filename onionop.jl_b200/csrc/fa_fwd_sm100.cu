// Flash-attention forward on the sm_100a tensor cores (tcgen05 UMMA, TMEM
// accumulators, TMA-fed K/V tiles), bf16/f16, E in {64, 128}.
//
// Reference: `_flash_attention_fwd!` (src/attention.jl:40-175) -- one thread
// per query row with the scores in shared memory and WMMA 16x16x16 tiles.
//
// One CTA per (128-query tile, query head, batch); 256 threads in four roles:
//   warp 0     TMA producer: Q once, then K_j / V_j into a 2-stage ring;
//   warp 1     MMA issuer: S_j = Q·K_jᵀ into one of two TMEM score buffers,
//              O += P_j·V_j with P_j read from TMEM (tcgen05 "ts" form);
//   warps 2-3  tile provider: key-validity bits (padding mask, ragged tail)
//              and the pair-bias tile, rearranged to [key/8][query][8];
//              with XC > 0 the XC = H CTAs of one (q-tile, batch) form a
//              thread-block cluster and share the pair bias: CTA r TMA-loads
//              keys [r·BN/H, (r+1)·BN/H) of the tile for ALL heads (the pair is
//              head-innermost, so this is one dense box), transposes it in
//              registers and pushes each head's slab into that head's CTA with
//              st.async (peer shared memory, completing the peer's mbarrier
//              transaction count) -- every pair byte crosses L2 once;
//   warps 4-7  softmax: thread r owns query row r (TMEM lane r): it reads
//              its 128 scores, adds the pair bias, masks, updates the running
//              max (rescaling O in TMEM only when the max grows by more than
//              2^8 -- the stale max keeps exp2 values <= 256), writes P as
//              16-bit values back into the score columns, and finally
//              normalises O and writes o and lse.
// TMEM: S0 [0,128), S1 [128,256), O [256, 256+E) of a 512-column allocation.
// Every mbarrier wait is bounded (sm100::wait); on a timeout all roles stop,
// the CTA frees its TMEM and returns.
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
constexpr int kThreads = 256;

enum Bar {
    kQFull = 0,
    kKFull = 1,      // +stage
    kVFull = 3,      // +stage
    kKVEmpty = 5,    // +stage
    kSFull = 7,      // +buffer
    kPFull = 9,      // +buffer
    kOFinal = 11,
    kOStep = 12,
    kTileFull = 13,  // +buffer (provider -> softmax)
    kTileEmpty = 15, // +buffer (softmax -> provider)
    kMmaDone = 17,   // MMA warp's own "all my MMAs retired" barrier
    kStageFull = 18, // exchange: own slice of the all-heads pair box landed
    kPairEmpty = 19, // +buffer, exchange: every receiver consumed the slot
    kNumBars = 21
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
    static constexpr int kStage = kPair + 2 * kPairBytes;       // exchange staging box [BN/H][BM][H]
    static constexpr int kStageBytes = PAIR ? kBN * kBM * 2 : 0;
    static constexpr int kBits = kStage + kStageBytes;          // 2 x (kBN/32) uint32
    static constexpr int kBar = kBits + 2 * (kBN / 32) * 4;
    static constexpr int kTmemSlot = kBar + kNumBars * 8;
    static constexpr int kTotal = kTmemSlot + 16;
    static constexpr int kAlloc = kTotal + 1024;                // slack for 1024-byte alignment
};

template <typename T, int E, bool CAUSAL, bool PAIR, bool MASK, int XC>
__global__ void __launch_bounds__(kThreads, 1)
fa_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_pair,
                    const Params p) {
    using L = Layout<E, PAIR>;
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
    constexpr bool kProvider = PAIR || MASK;
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
    const uint8_t* mg = MASK ? p.kmask + (int64_t)b * KL : nullptr;

    int64_t kv_len = KL;
    if (MASK) kv_len = kv_valid_len_block(mg, KL);
    int n_kt = (int)((kv_len + kBN - 1) / kBN);
    if (CAUSAL) {
        const int64_t i_end = q0 + kBM < QL ? q0 + kBM : QL;
        const int lim = (int)((i_end + kBN - 1) / kBN);
        n_kt = n_kt < lim ? n_kt : lim;
    }

    __shared__ int s_abort;   // set by the first wait of this CTA that gives up
    volatile int* ab = &s_abort;
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
            mbar_init(&bars[kTileFull + i], XC ? 1 : 64);
            mbar_init(&bars[kTileEmpty + i], 128);
            mbar_init(&bars[kPairEmpty + i], XC ? XC : 1);
        }
        mbar_init(&bars[kStageFull], 1);
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
    if (XC) cluster_sync();   // peers' barriers are initialised before any remote access
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS0 = tmem, tS1 = tmem + kBN, tO = tmem + 2 * kBN;

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0 && n_kt > 0) {
            tma_prefetch(&tm_q);
            tma_prefetch(&tm_k);
            tma_prefetch(&tm_v);
            const int bh_q = b * p.QH + h, bh_k = b * p.KH + kvh;
            mbar_expect_tx(&bars[kQFull], L::kQBytes);
#pragma unroll
            for (int half = 0; half < E / 64; ++half)
                tma_load_3d(smem + L::kQ + half * kBM * 128, &tm_q, &bars[kQFull], half * 64, (int)q0, bh_q);
            int issued = 0;
            for (int j = 0; j < n_kt; ++j) {
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
            }
            // Copies still in flight must land before the CTA can exit (they
            // have, unless a consumer gave up): bounded waits on the last ones.
            wait(&bars[kQFull], 0, ab, 2);
            for (int j = issued - kStages < 0 ? 0 : issued - kStages; j < issued; ++j) {
                wait(&bars[kKFull + j % kStages], (j / kStages) & 1, ab, 3);
                wait(&bars[kVFull + j % kStages], (j / kStages) & 1, ab, 4);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        constexpr uint32_t idesc_s = idesc_f16<kBF16>(kBM, kBN, false, false);
        constexpr uint32_t idesc_o = idesc_f16<kBF16>(kBM, E, false, true);
        const uint32_t sQ = smem_u32(smem + L::kQ);
        bool ok = n_kt > 0 && wait(&bars[kQFull], 0, ab, 5);
        auto issue_s = [&](int j) -> bool {
            const int s = j % kStages;
            if (!wait(&bars[kKFull + s], (j / kStages) & 1, ab, 6)) return false;
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
                umma_commit(&bars[kSFull + (j & 1)]);
            }
            __syncwarp();
            return true;
        };
        if (ok) ok = issue_s(0);
        for (int j = 0; ok && j < n_kt; ++j) {
            if (j + 1 < n_kt && !issue_s(j + 1)) break;
            const int s = j % kStages;
            if (!wait(&bars[kPFull + (j & 1)], (j >> 1) & 1, ab, 7)) break;
            if (!wait(&bars[kVFull + s], (j / kStages) & 1, ab, 8)) break;
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
            wait(&bars[kMmaDone], 0, ab, 9);
        }
    } else if (warp < 4) {
        // ------------------------------------------------------ tile provider
        if constexpr (XC > 0) {
            // ---- cluster exchange of the pair bias (see header comment)
            constexpr int KS = kBN / XC;   // keys this CTA stages per tile
            const int tp = threadIdx.x - 64;
            const uint32_t rank = cluster_rank();
            const uint8_t* stage = smem + L::kStage;
            const uint32_t recv0 = smem_u32(smem + L::kPair);
            for (int j = 0; j < n_kt; ++j) {
                const int buf = j & 1;
                const int64_t k0 = (int64_t)j * kBN;
                if (j >= 2) {
                    // my softmax is done with slot `buf` (tile j-2): tell every sender
                    if (!wait(&bars[kTileEmpty + buf], ((j >> 1) - 1) & 1, ab, 10)) break;
                    if (tp == 0) {
                        const uint32_t eb = smem_u32(&bars[kPairEmpty + buf]);
                        for (int d = 0; d < XC; ++d) mbar_arrive_remote(mapa(eb, d));
                    }
                    // and every receiver is done with it before I overwrite it
                    if (!wait_cluster(&bars[kPairEmpty + buf], ((j >> 1) - 1) & 1, ab, 11)) break;
                }
                if (tp == 0) {
                    mbar_expect_tx(&bars[kStageFull], L::kStageBytes);
                    tma_load_4d(smem + L::kStage, &tm_pair, &bars[kStageFull], 0, (int)q0, (int)(k0 + rank * KS), b);
                }
                if (tp < kBN / 32) {
                    uint32_t w = 0;
                    for (int t = 0; t < 32; ++t) {
                        const int64_t key = k0 + tp * 32 + t;
                        bool v = key < KL;
                        if (MASK && v) v = mg[key] != 0;
                        w |= (v ? 1u : 0u) << t;
                    }
                    bits[buf * (kBN / 32) + tp] = w;
                }
                if (!wait(&bars[kStageFull], j & 1, ab, 12)) break;
                named_bar_sync(1, 64);
                if (tp == 0) mbar_expect_tx_cluster(&bars[kTileFull + buf], kBN * kBM * 2);
                const uint32_t full_bar = smem_u32(&bars[kTileFull + buf]);
#pragma unroll 1
                for (int rr = 0; rr < kBM / 64; ++rr) {
                    const int q = tp + rr * 64;
#pragma unroll
                    for (int kk = 0; kk < KS / 8; ++kk) {
                        // in[k][w]: keys kk*8+k of query q, word w = heads (2w, 2w+1)
                        uint32_t in[8][XC / 2];
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            const uint4* src = reinterpret_cast<const uint4*>(stage + (((kk * 8 + k) * kBM + q) * XC) * 2);
#pragma unroll
                            for (int v = 0; v < XC / 8; ++v) {
                                const uint4 u = src[v];
                                in[k][4 * v] = u.x; in[k][4 * v + 1] = u.y; in[k][4 * v + 2] = u.z; in[k][4 * v + 3] = u.w;
                            }
                        }
                        const uint32_t off = (uint32_t)(((rank * KS / 8 + kk) * kBM + q) * 16);
#pragma unroll
                        for (int hd = 0; hd < XC; ++hd) {
                            const uint32_t sel = (hd & 1) ? 0x7632u : 0x5410u;
                            uint4 o;
                            o.x = __byte_perm(in[0][hd >> 1], in[1][hd >> 1], sel);
                            o.y = __byte_perm(in[2][hd >> 1], in[3][hd >> 1], sel);
                            o.z = __byte_perm(in[4][hd >> 1], in[5][hd >> 1], sel);
                            o.w = __byte_perm(in[6][hd >> 1], in[7][hd >> 1], sel);
                            st_async16(mapa(recv0 + buf * L::kPairBytes + off, hd), o, mapa(full_bar, hd));
                        }
                    }
                }
                named_bar_sync(1, 64);   // staging reads done before the next TMA overwrites it
            }
        } else if (kProvider) {
            const int tp = threadIdx.x - 64;
            const T* pg = PAIR ? reinterpret_cast<const T*>(p.pair) + (int64_t)b * KL * QL * p.QH + h : nullptr;
            for (int j = 0; j < n_kt; ++j) {
                const int buf = j & 1;
                if (j >= 2 && !wait(&bars[kTileEmpty + buf], ((j >> 1) - 1) & 1, ab, 13)) break;
                const int64_t k0 = (int64_t)j * kBN;
                if (tp < kBN / 32) {
                    uint32_t w = 0;
                    for (int t = 0; t < 32; ++t) {
                        const int64_t key = k0 + tp * 32 + t;
                        bool v = key < KL;
                        if (MASK && v) v = mg[key] != 0;
                        w |= (v ? 1u : 0u) << t;
                    }
                    bits[buf * (kBN / 32) + tp] = w;
                }
                if (PAIR) {
                    uint8_t* dst = smem + L::kPair + buf * L::kPairBytes;
#pragma unroll 1
                    for (int rr = 0; rr < kBM / 64; ++rr) {
                        const int r = tp + rr * 64;
                        const int64_t i = q0 + r;
#pragma unroll 2
                        for (int g = 0; g < kBN / 8; ++g) {
                            T v8[8];
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                const int64_t key = k0 + g * 8 + e;
                                v8[e] = (i < QL && key < KL) ? pg[(key * QL + i) * p.QH] : from_f<T>(0.f);
                            }
                            *reinterpret_cast<uint4*>(dst + ((g * kBM + r) * 8) * 2) = *reinterpret_cast<uint4*>(v8);
                        }
                    }
                }
                mbar_arrive(&bars[kTileFull + buf]);
            }
        }
    } else {
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
            if (kProvider) {
                const bool got = XC ? wait_cluster(&bars[kTileFull + buf], (j >> 1) & 1, ab, 14)
                                    : wait(&bars[kTileFull + buf], (j >> 1) & 1, ab, 14);
                if (!got) { ok = false; break; }
            }
            if (!wait(&bars[kSFull + buf], (j >> 1) & 1, ab, 15)) { ok = false; break; }
            tc_fence_after();
            const uint32_t tS = (buf ? tS1 : tS0) + lane_off;
            float x[kBN];
#pragma unroll
            for (int c = 0; c < kBN / 32; ++c) {
                uint32_t raw[32];
                tmem_ld32(tS + c * 32, raw);
                tmem_ld_wait();
                uint32_t vbits = 0xffffffffu;
                if (kProvider) {
                    vbits = bits[buf * (kBN / 32) + c];
                } else if (k0 + c * 32 + 32 > KL) {
                    const int64_t n = KL - (k0 + c * 32);
                    vbits = n <= 0 ? 0u : (n >= 32 ? 0xffffffffu : ((1u << n) - 1u));
                }
                float pb[32];
                if (PAIR) {
                    const uint8_t* src = smem + L::kPair + buf * L::kPairBytes;
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        const uint4 u = *reinterpret_cast<const uint4*>(src + (((c * 4 + g) * kBM + r) * 8) * 2);
                        float f8[8];
                        unpack8<T>(u, f8);
#pragma unroll
                        for (int e = 0; e < 8; ++e) pb[g * 8 + e] = f8[e] * kLog2e;
                    }
                }
#pragma unroll
                for (int t = 0; t < 32; ++t) {
                    float v = __uint_as_float(raw[t]) * sl2;
                    if (PAIR) v += pb[t];
                    bool valid = (vbits >> t) & 1u;
                    if (CAUSAL) valid = valid && (k0 + c * 32 + t <= i);
                    x[c * 32 + t] = valid ? v : -INFINITY;
                }
            }
            if (kProvider) mbar_arrive(&bars[kTileEmpty + buf]);
            float mx = x[0];
#pragma unroll
            for (int t = 1; t < kBN; ++t) mx = fmaxf(mx, x[t]);
            float alpha = 1.f;
            const float m_new = fmaxf(m, mx);
            const bool resc = m_new > m + 8.f;
            if (resc) {
                alpha = ex2(m - m_new);
                m = m_new;
            }
            const float m_use = (m == -INFINITY) ? 0.f : m;
            float ls = 0.f;
#pragma unroll
            for (int c = 0; c < kBN / 32; ++c) {
                uint32_t pk[16];
#pragma unroll
                for (int t = 0; t < 16; ++t) {
                    const float p0 = ex2(x[c * 32 + 2 * t] - m_use);
                    const float p1 = ex2(x[c * 32 + 2 * t + 1] - m_use);
                    ls += p0 + p1;
                    pk[t] = pack16<T>(p0, p1);
                }
                tmem_st16(tS + c * 16, pk);
            }
            l = l * alpha + ls;
            if (resc && j > 0 && alpha != 1.f) {
                // O holds Σ_{<j} P·V; PV_{j-1} must be complete before rescaling.
                if (!wait(&bars[kOStep], (j - 1) & 1, ab, 16)) { ok = false; break; }
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
        if (n_kt > 0 && ok && wait(&bars[kOFinal], 0, ab, 17)) {
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
    if (XC) cluster_sync();   // no peer may still write into this CTA's shared memory
}

// 4-D map over the pair bias [B][KL][QL][H] (Julia (H, QL, KL, B)), box
// (H, BM, BN/H, 1): one CTA's key slice of a tile for every head, no swizzle.
bool make_pair_map(CUtensorMap* m, const void* base, int H, int64_t QL, int64_t KL, int64_t B, int keys, bool bf16) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[4] = {(cuuint64_t)H, (cuuint64_t)QL, (cuuint64_t)KL, (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)H * 2, (cuuint64_t)QL * H * 2, (cuuint64_t)KL * QL * H * 2};
    cuuint32_t box[4] = {(cuuint32_t)H, (cuuint32_t)kBM, (cuuint32_t)keys, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// NNOP_B200_PAIR_XCH=0 disables the cluster exchange (the gather provider
// then reads the pair bias per head); used by the tests to cover both.
bool xch_enabled() {
    const char* e = getenv("NNOP_B200_PAIR_XCH");
    return !(e != nullptr && e[0] == '0');
}

template <typename T, int E, bool CAUSAL, bool PAIR, bool MASK, int XC>
int launch(const Params& p, cudaStream_t s, bool* launched) {
    using Lay = Layout<E, PAIR>;
    constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
    *launched = false;
    CUtensorMap tq, tk, tv, tp;
    memset(&tp, 0, sizeof(tp));
    if (!make_map(&tq, p.q, E, p.QL, (int64_t)p.B * p.QH, kBM, bf16) ||
        !make_map(&tk, p.k, E, p.KL, (int64_t)p.B * p.KH, kBN, bf16) ||
        !make_map(&tv, p.v, E, p.KL, (int64_t)p.B * p.KH, kBN, bf16) ||
        (XC && !make_pair_map(&tp, p.pair, p.QH, p.QL, p.KL, p.B, kBN / XC, bf16)))
        return fail(NNOP_ERR_CUDA, "flash_attention_fwd: cuTensorMapEncodeTiled failed");
    auto kern = fa_fwd_sm100_kernel<T, E, CAUSAL, PAIR, MASK, XC>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kAlloc) != cudaSuccess)
        return fail(NNOP_ERR_CUDA, "flash_attention_fwd: cannot set shared memory size");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.QH, (unsigned)((p.QL + kBM - 1) / kBM), p.B);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Lay::kAlloc;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    if (XC) {
        if (XC > 8) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = XC;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int nclusters = 0;
        if (cudaOccupancyMaxActiveClusters(&nclusters, kern, &cfg) != cudaSuccess || nclusters < 1) {
            cudaGetLastError();
            return NNOP_OK;   // not launchable here: caller falls back to the gather provider
        }
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tq, tk, tv, tp, p);
    if (e != cudaSuccess) return fail(NNOP_ERR_CUDA, std::string("flash_attention_fwd (sm100): ") + cudaGetErrorString(e));
    *launched = true;
    return check_launch("flash_attention_fwd (sm100)");
}

template <typename T, int E, bool CAUSAL>
int dispatch_flags(const Params& p, cudaStream_t s) {
    const bool pair = p.pair != nullptr, mask = p.kmask != nullptr;
    bool done = false;
    int st = NNOP_OK;
    if (pair && xch_enabled() && (p.QH == 8 || p.QH == 16) && E == 64) {
        if (p.QH == 16)
            st = mask ? launch<T, E, CAUSAL, true, true, 16>(p, s, &done) : launch<T, E, CAUSAL, true, false, 16>(p, s, &done);
        else
            st = mask ? launch<T, E, CAUSAL, true, true, 8>(p, s, &done) : launch<T, E, CAUSAL, true, false, 8>(p, s, &done);
        if (st || done) return st;
    }
    if (pair && mask) return launch<T, E, CAUSAL, true, true, 0>(p, s, &done);
    if (pair) return launch<T, E, CAUSAL, true, false, 0>(p, s, &done);
    if (mask) return launch<T, E, CAUSAL, false, true, 0>(p, s, &done);
    return launch<T, E, CAUSAL, false, false, 0>(p, s, &done);
}

}  // namespace

// Shapes this kernel covers; the others use the mma.sync kernels.
bool sm100_fwd_supported(const Params& p, int dtype) {
    if (dtype != NNOP_BF16 && dtype != NNOP_F16) return false;
    if (p.E == 64) return true;
    if (p.E == 128) return p.pair == nullptr;   // pair tiles at E=128 exceed shared memory
    return false;
}

// Reads and clears the bounded-wait timeout flag of this file's kernels.
int sm100_fwd_timeouts() {
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, sm100::g_wait_timeout, sizeof(int));
    cudaMemcpyToSymbol(sm100::g_wait_timeout, &z, sizeof(int));
    return v;
}

int sm100_fwd(const Params& p, int dtype, bool causal, cudaStream_t s) {
    if (dtype == NNOP_BF16) {
        if (p.E == 64) return causal ? dispatch_flags<__nv_bfloat16, 64, true>(p, s) : dispatch_flags<__nv_bfloat16, 64, false>(p, s);
        return causal ? dispatch_flags<__nv_bfloat16, 128, true>(p, s) : dispatch_flags<__nv_bfloat16, 128, false>(p, s);
    }
    if (p.E == 64) return causal ? dispatch_flags<__half, 64, true>(p, s) : dispatch_flags<__half, 64, false>(p, s);
    return causal ? dispatch_flags<__half, 128, true>(p, s) : dispatch_flags<__half, 128, false>(p, s);
}

}  // namespace fa


}  // namespace nnop
