// Re-layout of the pair bias between the reference's head-innermost layout and
// the per-head tiles the tcgen05 attention kernels load with TMA.
//
// The pair bias is (H, QL, KL, B) in Julia (src/attention.jl:72,104), i.e. the
// buffer [B][KL][QL][H]: one head's element is 2 bytes of every 32-byte sector
// (H = 16), so a CTA that owns one head cannot read it efficiently.  The
// attention kernels instead read, per head, the key-major copy
//   tiles[b][h][query/128][key][query%128]   (QL, KL padded to multiples of 128)
// in which a (128-query, 128-key) tile is one contiguous 32 KB block, two
// 64-query TMA boxes.  The forward uses
// it as the K-major, the backward as the MN-major B operand of an identity
// UMMA that adds the bias to the scores (fa_fwd_sm100.cu, fa_bwd_sm100.cu);
// the backward writes its dS tiles in the same layout and dpair_from_tiles
// turns them back into dpair [B][KL][QL][H], writing zeros for the (query,
// key) tiles the backward does not visit (above the causal diagonal, key
// tiles past the last kept key), so every dpair element is written once.
//
// A pair value of −Inf (a masked entry) is written to the tiles as the most
// negative finite value of the dtype: the identity UMMA multiplies every tile
// element, and 0·(−Inf) would turn the whole 16-wide K block into NaN.  Its
// probability stays exactly 0 (exp2 of < −9e4 underflows) whenever the row
// has another finite score.
//
// Both kernels move [8 keys][128 queries][H] blocks through shared memory: on
// the reference side 8 contiguous runs of 128·H elements (16-byte vectors, all
// eight in flight per thread), on the per-head side 16-byte pieces of 8
// queries, threads walking heads fastest so each head's pieces form whole
// 32-byte sectors.  Blocks the attention kernels never read are skipped.
#include "fa_common.cuh"

namespace nnop {
namespace {

constexpr int kTB = 256;    // threads per block
constexpr int kTile = 128;  // attention tile (queries and keys)
constexpr int kKeys = 8;    // keys per block

// 16-bit patterns of −Inf and of the most negative finite value
template <typename T> struct NegInf;
template <> struct NegInf<__nv_bfloat16> { static constexpr uint32_t kInf = 0xFF80u, kLowest = 0xFF7Fu; };
template <> struct NegInf<__half> { static constexpr uint32_t kInf = 0xFC00u, kLowest = 0xFBFFu; };

template <typename T>
__device__ __forceinline__ uint32_t finite_lo(uint32_t x) {
    return x == NegInf<T>::kInf ? NegInf<T>::kLowest : x;
}

__device__ __forceinline__ bool aligned_rows(const void* p, int64_t elems_per_row) {
    return ((reinterpret_cast<uintptr_t>(p) & 15) == 0) && (elems_per_row % 8 == 0);
}

// Loads pair[b][g*8 .. g*8+8)[i0 .. i0+128)[0 .. H) into s[8][128·H]
// (zeros outside the tensor).
template <typename T>
__device__ __forceinline__ void load_block(const T* __restrict__ pair, T* s, int b, int64_t g, int64_t i0,
                                           int64_t QL, int64_t KL, int H) {
    const int row = kTile * H;
    const T* src = pair + (((int64_t)b * KL + g * kKeys) * QL + i0) * H;
    const int64_t rs = QL * H;   // elements between consecutive keys
    if (g * kKeys + kKeys <= KL && i0 + kTile <= QL && aligned_rows(pair, rs)) {
        for (int v = threadIdx.x; v < row / 8; v += kTB) {
            uint4 u[kKeys];
#pragma unroll
            for (int e = 0; e < kKeys; ++e) u[e] = __ldcs(reinterpret_cast<const uint4*>(src + e * rs) + v);
#pragma unroll
            for (int e = 0; e < kKeys; ++e) reinterpret_cast<uint4*>(s + e * row)[v] = u[e];
        }
    } else {
        for (int e = 0; e < kKeys; ++e) {
            const bool key_ok = g * kKeys + e < KL;
            for (int x = threadIdx.x; x < row; x += kTB) {
                const bool ok = key_ok && i0 + x / H < QL;
                s[e * row + x] = ok ? src[e * rs + x] : from_f<T>(0.f);
            }
        }
    }
}

// True when the attention kernels read the (query tile c, key group g) block.
__device__ __forceinline__ bool visited(int c, int64_t g, int b, const int* kv_len, int causal) {
    const int64_t kt = g * kKeys / kTile;
    if (causal && kt > c) return false;
    if (kv_len != nullptr && kt * kTile >= kv_len[b]) return false;
    return true;
}

// tiles[b][h][c][g*8+kk][i] = pair[b][g*8+kk][c*128+i][h];
// block = (query chunk c, key group g, b)
template <typename T>
__global__ void __launch_bounds__(kTB, 2) pair_tiles_kernel(const T* __restrict__ pair, T* __restrict__ out,
                                                         const int* __restrict__ kv_len, int64_t QL, int64_t KL,
                                                         int H, int64_t qlp, int64_t klp, int causal) {
    extern __shared__ __align__(16) uint8_t sm_raw[];
    T* s = reinterpret_cast<T*>(sm_raw);   // [8][128][H]
    const int c = blockIdx.x;
    const int64_t g = blockIdx.y;
    const int b = blockIdx.z;
    if (!visited(c, g, b, kv_len, causal)) return;
    const int64_t i0 = (int64_t)c * kTile;
    load_block(pair, s, b, g, i0, QL, KL, H);
    __syncthreads();
    // thread -> (key kk, 8-query piece v, head h), heads fastest
    for (int x = threadIdx.x; x < H * (kTile / 8) * kKeys; x += kTB) {
        const int h = x % H, v = (x / H) % (kTile / 8), kk = x / (H * (kTile / 8));
        const uint16_t* col = reinterpret_cast<const uint16_t*>(s) + (kk * kTile + v * 8) * H + h;
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
            w[e] = finite_lo<T>(col[(2 * e) * H]) | (finite_lo<T>(col[(2 * e + 1) * H]) << 16);
        T* dst = out + ((((int64_t)b * H + h) * (qlp / kTile) + c) * klp + g * kKeys + kk) * kTile + v * 8;
        __stcs(reinterpret_cast<uint4*>(dst), make_uint4(w[0], w[1], w[2], w[3]));
    }
}

// dpair[b][g*8+kk][c*128+i][h] = tiles[b][h][c][g*8+kk][i] on visited blocks, 0 elsewhere.
template <typename T>
__global__ void __launch_bounds__(kTB) dpair_from_tiles_kernel(const T* __restrict__ tiles, T* __restrict__ dpair,
                                                               const int* __restrict__ kv_len, int64_t QL,
                                                               int64_t KL, int H, int64_t qlp, int64_t klp,
                                                               int causal) {
    extern __shared__ __align__(16) uint8_t sm_raw[];
    T* s = reinterpret_cast<T*>(sm_raw);   // [8][128][H]
    const int c = blockIdx.x;
    const int64_t g = blockIdx.y;
    const int b = blockIdx.z;
    const int64_t i0 = (int64_t)c * kTile;
    const bool vis = visited(c, g, b, kv_len, causal);
    const int row = kTile * H;
    if (vis) {
        const int total = H * (kTile / 8) * kKeys;
        for (int base = 0; base < total; base += 8 * kTB) {
            uint4 u[8];
#pragma unroll
            for (int it = 0; it < 8; ++it) {
                const int x = base + it * kTB + threadIdx.x;
                if (x < total) {
                    const int h = x % H, v = (x / H) % (kTile / 8), kk = x / (H * (kTile / 8));
                    u[it] = __ldcs(reinterpret_cast<const uint4*>(
                        tiles + ((((int64_t)b * H + h) * (qlp / kTile) + c) * klp + g * kKeys + kk) * kTile + v * 8));
                }
            }
#pragma unroll
            for (int it = 0; it < 8; ++it) {
                const int x = base + it * kTB + threadIdx.x;
                if (x < total) {
                    const int h = x % H, v = (x / H) % (kTile / 8), kk = x / (H * (kTile / 8));
                    uint16_t* col = reinterpret_cast<uint16_t*>(s) + (kk * kTile + v * 8) * H + h;
                    const uint32_t w[4] = {u[it].x, u[it].y, u[it].z, u[it].w};
#pragma unroll
                    for (int e = 0; e < 8; ++e) col[e * H] = (uint16_t)(w[e >> 1] >> (16 * (e & 1)));
                }
            }
        }
        __syncthreads();
    }
    const bool full_q = i0 + kTile <= QL;
    const int64_t rs = QL * H;
    T* dst0 = dpair + (((int64_t)b * KL + g * kKeys) * QL + i0) * H;
    if (g * kKeys + kKeys <= KL && full_q && aligned_rows(dpair, rs)) {
        for (int v = threadIdx.x; v < row / 8; v += kTB) {
#pragma unroll
            for (int kk = 0; kk < kKeys; ++kk) {
                const uint4 u = vis ? reinterpret_cast<const uint4*>(s + kk * row)[v] : make_uint4(0, 0, 0, 0);
                __stcs(reinterpret_cast<uint4*>(dst0 + kk * rs) + v, u);
            }
        }
    } else {
        const int n = (int)((full_q ? kTile : QL - i0) * H);
        for (int kk = 0; kk < kKeys && g * kKeys + kk < KL; ++kk)
            for (int x = threadIdx.x; x < n; x += kTB) dst0[kk * rs + x] = vis ? s[kk * row + x] : from_f<T>(0.f);
    }
}


// ---------------------------------------------------------------------------
// Fast path for H = 8·CQ heads, CQ in {1, 2, 4, 8}: the block's key rows sit in
// shared memory as 16-byte chunks (CQ per query: 8 heads each), chunk L of a
// row stored at swz(L); a thread moves 8 heads × 8 queries at a time: eight
// 16-byte shared accesses and an 8×8 transpose of 16-bit values in registers
// (byte permutes).  The swizzle spreads the query pieces a warp touches at
// once over distinct bank groups, so the 16-byte accesses need the minimum
// four wavefronts.
// word i of a 16-byte vector (i a compile-time constant after unrolling)
__device__ __forceinline__ uint32_t word(const uint4& u, int i) {
    return i == 0 ? u.x : i == 1 ? u.y : i == 2 ? u.z : u.w;
}

template <int CQ>
__device__ __forceinline__ int swz(int L) {
    constexpr int NV = 8 / CQ;
    return L ^ (((L / (8 * CQ)) % NV) * CQ);
}

// −Inf -> most negative finite on two packed 16-bit values (NaN kept)
template <typename T>
__device__ __forceinline__ uint32_t finite2(uint32_t x);
template <>
__device__ __forceinline__ uint32_t finite2<__nv_bfloat16>(uint32_t x) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&x);
    const uint32_t lo = 0xFF7FFF7Fu;
    v = __hmax2_nan(v, *reinterpret_cast<const __nv_bfloat162*>(&lo));
    return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t finite2<__half>(uint32_t x) {
    __half2 v = *reinterpret_cast<__half2*>(&x);
    const uint32_t lo = 0xFBFFFBFFu;
    v = __hmax2_nan(v, *reinterpret_cast<const __half2*>(&lo));
    return *reinterpret_cast<uint32_t*>(&v);
}

template <typename T, int CQ>
__global__ void __launch_bounds__(kTB, 3) pair_tiles_fast_kernel(const T* __restrict__ pair, T* __restrict__ out,
                                                              const int* __restrict__ kv_len, int64_t QL,
                                                              int64_t KL, int64_t qlp, int64_t klp, int causal) {
    constexpr int H = 8 * CQ;
    constexpr int RC = kTile * CQ;   // 16-byte chunks per key row
    extern __shared__ __align__(16) uint8_t sm_raw[];
    uint4* s4 = reinterpret_cast<uint4*>(sm_raw);          // [8][RC] swizzled
    const int c = blockIdx.x;
    const int64_t g = blockIdx.y;
    const int b = blockIdx.z;
    if (!visited(c, g, b, kv_len, causal)) return;
    const int64_t i0 = (int64_t)c * kTile;
    const int64_t rs = QL * H;
    const T* src = pair + (((int64_t)b * KL + g * kKeys) * QL + i0) * H;
    if (g * kKeys + kKeys <= KL && i0 + kTile <= QL && aligned_rows(pair, rs)) {
#pragma unroll
        for (int L0 = 0; L0 < RC; L0 += kTB) {
            const int L = L0 + threadIdx.x;
            if (RC % kTB == 0 || L < RC) {
                uint4 u[kKeys];
#pragma unroll
                for (int e = 0; e < kKeys; ++e) u[e] = __ldcs(reinterpret_cast<const uint4*>(src + e * rs) + L);
#pragma unroll
                for (int e = 0; e < kKeys; ++e) s4[e * RC + swz<CQ>(L)] = u[e];
            }
        }
    } else {
        uint16_t* s16 = reinterpret_cast<uint16_t*>(sm_raw);
        for (int e = 0; e < kKeys; ++e) {
            const bool key_ok = g * kKeys + e < KL;
            for (int x = threadIdx.x; x < kTile * H; x += kTB) {
                const bool ok = key_ok && i0 + x / H < QL;
                const T val = ok ? src[e * rs + x] : from_f<T>(0.f);
                s16[(e * RC + swz<CQ>(x / 8)) * 8 + x % 8] = *reinterpret_cast<const uint16_t*>(&val);
            }
        }
    }
    __syncthreads();
    // thread -> (key kk, 8-query piece v, head octet ho), octets fastest
    constexpr int kItems = kKeys * (kTile / 8) * CQ;
    for (int x = threadIdx.x; x < kItems; x += kTB) {
        const int ho = x % CQ, v = (x / CQ) % (kTile / 8), kk = x / (CQ * (kTile / 8));
        uint4 r[8];   // r[e]: heads 8ho..8ho+7 of query v*8+e
#pragma unroll
        for (int e = 0; e < 8; ++e) r[e] = s4[kk * RC + swz<CQ>((v * 8 + e) * CQ + ho)];
        T* dst = out + ((((int64_t)b * H + 8 * ho) * (qlp / kTile) + c) * klp + g * kKeys + kk) * kTile + v * 8;
#pragma unroll
        for (int j = 0; j < 8; ++j) {   // head 8ho+j: queries (2m, 2m+1) in word m
            const uint32_t sel = (j & 1) ? 0x7632u : 0x5410u;
            uint32_t o[4];
#pragma unroll
            for (int m = 0; m < 4; ++m) o[m] = finite2<T>(__byte_perm(word(r[2 * m], j >> 1), word(r[2 * m + 1], j >> 1), sel));
            __stcs(reinterpret_cast<uint4*>(dst + (int64_t)j * klp * qlp), make_uint4(o[0], o[1], o[2], o[3]));
        }
    }
}

template <typename T, int CQ>
__global__ void __launch_bounds__(kTB, CQ >= 4 ? 2 : 3) dpair_from_tiles_fast_kernel(const T* __restrict__ tiles,
                                                                    T* __restrict__ dpair,
                                                                    const int* __restrict__ kv_len, int64_t QL,
                                                                    int64_t KL, int64_t qlp, int64_t klp,
                                                                    int causal) {
    constexpr int H = 8 * CQ;
    constexpr int RC = kTile * CQ;
    extern __shared__ __align__(16) uint8_t sm_raw[];
    uint4* s4 = reinterpret_cast<uint4*>(sm_raw);
    const int c = blockIdx.x;
    const int64_t g = blockIdx.y;
    const int b = blockIdx.z;
    const int64_t i0 = (int64_t)c * kTile;
    const bool vis = visited(c, g, b, kv_len, causal);
    if (vis) {
        // thread -> (key kk, 8-query piece v, head octet ho): eight 16-byte
        // loads (one per head) in flight, transposed into eight query chunks
        constexpr int kItems = kKeys * (kTile / 8) * CQ;
        for (int x = threadIdx.x; x < kItems; x += kTB) {
            const int ho = x % CQ, v = (x / CQ) % (kTile / 8), kk = x / (CQ * (kTile / 8));
            const T* p0 = tiles + ((((int64_t)b * H + 8 * ho) * (qlp / kTile) + c) * klp + g * kKeys + kk) * kTile + v * 8;
            uint4 in[8];   // in[j]: queries v*8..v*8+7 of head 8ho+j
#pragma unroll
            for (int j = 0; j < 8; ++j) in[j] = __ldcs(reinterpret_cast<const uint4*>(p0 + (int64_t)j * klp * qlp));
#pragma unroll
            for (int e = 0; e < 8; ++e) {   // query v*8+e: heads (2w, 2w+1) in word w
                const uint32_t sel = (e & 1) ? 0x7632u : 0x5410u;
                s4[kk * RC + swz<CQ>((v * 8 + e) * CQ + ho)] =
                    make_uint4(__byte_perm(word(in[0], e >> 1), word(in[1], e >> 1), sel),
                               __byte_perm(word(in[2], e >> 1), word(in[3], e >> 1), sel),
                               __byte_perm(word(in[4], e >> 1), word(in[5], e >> 1), sel),
                               __byte_perm(word(in[6], e >> 1), word(in[7], e >> 1), sel));
            }
        }
        __syncthreads();
    }
    const int64_t rs = QL * H;
    T* dst0 = dpair + (((int64_t)b * KL + g * kKeys) * QL + i0) * H;
    if (g * kKeys + kKeys <= KL && i0 + kTile <= QL && aligned_rows(dpair, rs)) {
#pragma unroll
        for (int L0 = 0; L0 < RC; L0 += kTB) {
            const int L = L0 + threadIdx.x;
            if (RC % kTB == 0 || L < RC) {
#pragma unroll
                for (int kk = 0; kk < kKeys; ++kk) {
                    const uint4 u = vis ? s4[kk * RC + swz<CQ>(L)] : make_uint4(0, 0, 0, 0);
                    __stcs(reinterpret_cast<uint4*>(dst0 + kk * rs) + L, u);
                }
            }
        }
    } else {
        const uint16_t* s16 = reinterpret_cast<const uint16_t*>(sm_raw);
        const int n = (int)((i0 + kTile <= QL ? kTile : QL - i0) * H);
        for (int kk = 0; kk < kKeys && g * kKeys + kk < KL; ++kk)
            for (int x = threadIdx.x; x < n; x += kTB) {
                const uint16_t bits = vis ? s16[(kk * RC + swz<CQ>(x / 8)) * 8 + x % 8] : (uint16_t)0;
                dst0[kk * rs + x] = *reinterpret_cast<const T*>(&bits);
            }
    }
}

template <typename KernelT>
int set_smem(KernelT kern, size_t smem, const char* what) {
    if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return fail(NNOP_ERR_CUDA, std::string(what) + ": cannot set shared memory size");
    return NNOP_OK;
}

}  // namespace

namespace fa_host {

int64_t pad_tile(int64_t n) { return (n + kTile - 1) / kTile * kTile; }

size_t pair_tiles_bytes(int64_t QL, int64_t KL, int64_t H, int64_t B) {
    return (size_t)B * H * pad_tile(QL) * pad_tile(KL) * 2;
}

template <typename T>
int launch_pair_tiles(const T* pair, T* out, const int* kv_len, int64_t QL, int64_t KL, int H, int B, bool causal,
                      cudaStream_t s) {
    const int64_t qlp = pad_tile(QL), klp = pad_tile(KL);
    const size_t smem = (size_t)kKeys * kTile * H * sizeof(T);
    dim3 grid((unsigned)(qlp / kTile), (unsigned)(klp / kKeys), B);
    const int cz = causal ? 1 : 0;
    int st = NNOP_OK;
#define NNOP_TILES_FAST(CQ)                                                                              \
    case 8 * CQ:                                                                                          \
        st = set_smem(pair_tiles_fast_kernel<T, CQ>, smem, "pair_tiles");                               \
        if (st) return st;                                                                                \
        pair_tiles_fast_kernel<T, CQ><<<grid, kTB, smem, s>>>(pair, out, kv_len, QL, KL, qlp, klp, cz); \
        return check_launch("pair_tiles");
    switch (H) {
        NNOP_TILES_FAST(1)
        NNOP_TILES_FAST(2)
        NNOP_TILES_FAST(4)
        NNOP_TILES_FAST(8)
        default:
            break;
    }
#undef NNOP_TILES_FAST
    st = set_smem(pair_tiles_kernel<T>, smem, "pair_tiles");
    if (st) return st;
    pair_tiles_kernel<T><<<grid, kTB, smem, s>>>(pair, out, kv_len, QL, KL, H, qlp, klp, cz);
    return check_launch("pair_tiles");
}

template <typename T>
int launch_dpair_from_tiles(const T* tiles, T* dpair, const int* kv_len, int64_t QL, int64_t KL, int H, int B,
                            bool causal, cudaStream_t s) {
    const int64_t qlp = pad_tile(QL), klp = pad_tile(KL);
    const size_t smem = (size_t)kKeys * kTile * H * sizeof(T);
    dim3 grid((unsigned)(qlp / kTile), (unsigned)(klp / kKeys), B);
    const int cz = causal ? 1 : 0;
    int st = NNOP_OK;
#define NNOP_DPAIR_FAST(CQ)                                                                                    \
    case 8 * CQ:                                                                                                \
        st = set_smem(dpair_from_tiles_fast_kernel<T, CQ>, smem, "dpair_from_tiles");                         \
        if (st) return st;                                                                                      \
        dpair_from_tiles_fast_kernel<T, CQ><<<grid, kTB, smem, s>>>(tiles, dpair, kv_len, QL, KL, qlp, klp, cz); \
        return check_launch("dpair_from_tiles");
    switch (H) {
        NNOP_DPAIR_FAST(1)
        NNOP_DPAIR_FAST(2)
        NNOP_DPAIR_FAST(4)
        NNOP_DPAIR_FAST(8)
        default:
            break;
    }
#undef NNOP_DPAIR_FAST
    st = set_smem(dpair_from_tiles_kernel<T>, smem, "dpair_from_tiles");
    if (st) return st;
    dpair_from_tiles_kernel<T><<<grid, kTB, smem, s>>>(tiles, dpair, kv_len, QL, KL, H, qlp, klp, cz);
    return check_launch("dpair_from_tiles");
}

template int launch_pair_tiles<__half>(const __half*, __half*, const int*, int64_t, int64_t, int, int, bool,
                                       cudaStream_t);
template int launch_pair_tiles<__nv_bfloat16>(const __nv_bfloat16*, __nv_bfloat16*, const int*, int64_t, int64_t, int,
                                              int, bool, cudaStream_t);
template int launch_dpair_from_tiles<__half>(const __half*, __half*, const int*, int64_t, int64_t, int, int, bool,
                                             cudaStream_t);
template int launch_dpair_from_tiles<__nv_bfloat16>(const __nv_bfloat16*, __nv_bfloat16*, const int*, int64_t,
                                                    int64_t, int, int, bool, cudaStream_t);

}  // namespace fa_host
}  // namespace nnop
