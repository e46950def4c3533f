// Re-layout of the pair bias between the reference's head-innermost layout and
// per-head tiles the tcgen05 attention kernels load with one TMA box.
//
// The pair bias is (H, QL, KL, B) in Julia (src/attention.jl:72,104), i.e. the
// buffer [B][KL][QL][H]: one head's element is 2 bytes of every 32-byte sector
// (H = 16), so a CTA that owns one head cannot read it efficiently.  These
// kernels move whole [8 keys][128 queries][H] (or [128 keys][8 queries][H])
// blocks through shared memory -- every global read and write is a contiguous
// run -- and write, per head:
//   pair_tiles_fwd: F[b][h][key/8][query][key%8]   (QL, KL padded to 128)
//   pair_tiles_bwd: T[b][h][query/8][key][query%8]
// The backward writes its dS tiles in layout T; dpair_from_tiles turns them
// back into dpair [B][KL][QL][H], writing zeros for the (query, key) tiles the
// backward did not visit (above the causal diagonal, fully masked key tiles),
// so every dpair element is written exactly once.
// Blocks the attention kernels never read (causal upper triangle) are skipped.
#include "fa_common.cuh"

namespace nnop {
namespace {

constexpr int kTB = 256;    // threads per block
constexpr int kTile = 128;  // attention tile (queries and keys)

inline __device__ bool vec_ok(const void* p, int64_t elems_per_row) {
    return ((reinterpret_cast<uintptr_t>(p) & 15) == 0) && (elems_per_row % 8 == 0);
}

// F[b][h][g][i][e] = pair[b][g*8+e][i][h]; block = (q chunk c, key group g, b)
template <typename T>
__global__ void __launch_bounds__(kTB) pair_tiles_fwd_kernel(const T* __restrict__ pair, T* __restrict__ out,
                                                             int64_t QL, int64_t KL, int H, int64_t qlp,
                                                             int64_t klp, int causal) {
    extern __shared__ __align__(16) uint8_t sm_raw[];
    T* s = reinterpret_cast<T*>(sm_raw);   // [8][128][H]
    const int c = blockIdx.x;
    const int64_t g = blockIdx.y;
    const int b = blockIdx.z;
    if (causal && (g * 8) / kTile > c) return;   // never read by the forward
    const int64_t i0 = (int64_t)c * kTile;
    const int row = kTile * H;                     // elements of one key's run
    const bool full_q = i0 + kTile <= QL;
    for (int e = 0; e < 8; ++e) {
        const int64_t key = g * 8 + e;
        T* dst = s + e * row;
        const T* src = pair + ((b * KL + key) * QL + i0) * H;
        if (key < KL && full_q && vec_ok(src, QL * H)) {
            for (int v = threadIdx.x; v < row / 8; v += kTB)
                reinterpret_cast<uint4*>(dst)[v] = __ldcs(reinterpret_cast<const uint4*>(src) + v);
        } else {
            for (int x = threadIdx.x; x < row; x += kTB) {
                const int64_t i = i0 + x / H;
                dst[x] = (key < KL && i < QL) ? src[x] : from_f<T>(0.f);
            }
        }
    }
    __syncthreads();
    for (int x = threadIdx.x; x < H * kTile; x += kTB) {
        const int h = x / kTile, i = x % kTile;
        T v8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v8[e] = s[(e * kTile + i) * H + h];
        T* dst = out + ((((int64_t)b * H + h) * (klp / 8) + g) * qlp + i0 + i) * 8;
        __stcs(reinterpret_cast<uint4*>(dst), *reinterpret_cast<uint4*>(v8));
    }
}

// T[b][h][qg][k][e] = pair[b][k][qg*8+e][h]; block = (key chunk kc, query group qg, b)
template <typename T>
__global__ void __launch_bounds__(kTB) pair_tiles_bwd_kernel(const T* __restrict__ pair, T* __restrict__ out,
                                                             const int* __restrict__ kv_len, int64_t QL, int64_t KL,
                                                             int H, int64_t qlp, int64_t klp, int causal) {
    extern __shared__ __align__(16) uint8_t sm_raw[];
    T* s = reinterpret_cast<T*>(sm_raw);   // [128][8][H]
    const int kc = blockIdx.x;
    const int64_t qg = blockIdx.y;
    const int b = blockIdx.z;
    if (causal && kc > (qg * 8) / kTile) return;           // never read by the backward
    if (kv_len != nullptr && (int64_t)kc * kTile >= kv_len[b]) return;
    const int64_t k0 = (int64_t)kc * kTile;
    const int run = 8 * H;                                  // elements of one key's run
    const bool full_q = qg * 8 + 8 <= QL;
    if (full_q && vec_ok(pair, QL * H) && (QL * H) % 8 == 0) {
        // each key's run is 8·H contiguous elements = H 16-byte vectors
        for (int x = threadIdx.x; x < kTile * H; x += kTB) {
            const int k = x / H, v = x % H;
            const int64_t key = k0 + k;
            uint4 u = make_uint4(0, 0, 0, 0);
            if (key < KL) u = __ldcs(reinterpret_cast<const uint4*>(pair + ((b * KL + key) * QL + qg * 8) * H) + v);
            reinterpret_cast<uint4*>(s + k * run)[v] = u;
        }
    } else {
        for (int x = threadIdx.x; x < kTile * run; x += kTB) {
            const int k = x / run, r = x % run;
            const int64_t key = k0 + k, i = qg * 8 + r / H;
            T v = from_f<T>(0.f);
            if (key < KL && i < QL) v = pair[((b * KL + key) * QL + qg * 8) * H + r];
            s[x] = v;
        }
    }
    __syncthreads();
    for (int x = threadIdx.x; x < H * kTile; x += kTB) {
        const int h = x / kTile, k = x % kTile;
        T v8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v8[e] = s[(k * 8 + e) * H + h];
        T* dst = out + ((((int64_t)b * H + h) * (qlp / 8) + qg) * klp + k0 + k) * 8;
        __stcs(reinterpret_cast<uint4*>(dst), *reinterpret_cast<uint4*>(v8));
    }
}

// dpair[b][g*8+kk][i][h] = T[b][h][i/8][g*8+kk][i%8] on visited tiles, 0 elsewhere.
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
    const int64_t kt = (g * 8) / kTile;
    bool visited = !(causal && kt > c);
    if (kv_len != nullptr && kt * kTile >= kv_len[b]) visited = false;
    const int row = kTile * H;
    if (visited) {
        // 8 keys x 16 query groups x H heads of 16-byte pieces
        for (int x = threadIdx.x; x < H * 16 * 8; x += kTB) {
            const int kk = x % 8, qgl = (x / 8) % 16, h = x / 128;
            const T* src = tiles + ((((int64_t)b * H + h) * (qlp / 8) + (i0 / 8 + qgl)) * klp + g * 8 + kk) * 8;
            const uint4 u = __ldcs(reinterpret_cast<const uint4*>(src));
            const T* v8 = reinterpret_cast<const T*>(&u);
#pragma unroll
            for (int e = 0; e < 8; ++e) s[(kk * kTile + qgl * 8 + e) * H + h] = v8[e];
        }
        __syncthreads();
    }
    const bool full_q = i0 + kTile <= QL;
    for (int kk = 0; kk < 8; ++kk) {
        const int64_t key = g * 8 + kk;
        if (key >= KL) break;
        T* dst = dpair + ((b * KL + key) * QL + i0) * H;
        const int n = (int)((full_q ? kTile : QL - i0) * H);
        if (full_q && vec_ok(dst, QL * H)) {
            for (int v = threadIdx.x; v < row / 8; v += kTB) {
                const uint4 u = visited ? reinterpret_cast<const uint4*>(s + kk * row)[v] : make_uint4(0, 0, 0, 0);
                __stcs(reinterpret_cast<uint4*>(dst) + v, u);
            }
        } else {
            for (int x = threadIdx.x; x < n; x += kTB) dst[x] = visited ? s[kk * row + x] : from_f<T>(0.f);
        }
    }
}

}  // namespace

namespace fa_host {

int64_t pad_tile(int64_t n) { return (n + kTile - 1) / kTile * kTile; }

size_t pair_tiles_bytes(int64_t QL, int64_t KL, int64_t H, int64_t B) {
    return (size_t)B * H * pad_tile(QL) * pad_tile(KL) * 2;
}

template <typename T>
int launch_pair_tiles_fwd(const T* pair, T* out, int64_t QL, int64_t KL, int H, int B, bool causal, cudaStream_t s) {
    const int64_t qlp = pad_tile(QL), klp = pad_tile(KL);
    const size_t smem = (size_t)8 * kTile * H * sizeof(T);
    auto kern = pair_tiles_fwd_kernel<T>;
    if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return fail(NNOP_ERR_CUDA, "pair_tiles_fwd: cannot set shared memory size");
    dim3 grid((unsigned)(qlp / kTile), (unsigned)(klp / 8), B);
    kern<<<grid, kTB, smem, s>>>(pair, out, QL, KL, H, qlp, klp, causal ? 1 : 0);
    return check_launch("pair_tiles_fwd");
}

template <typename T>
int launch_pair_tiles_bwd(const T* pair, T* out, const int* kv_len, int64_t QL, int64_t KL, int H, int B, bool causal,
                          cudaStream_t s) {
    const int64_t qlp = pad_tile(QL), klp = pad_tile(KL);
    const size_t smem = (size_t)8 * kTile * H * sizeof(T);
    auto kern = pair_tiles_bwd_kernel<T>;
    if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return fail(NNOP_ERR_CUDA, "pair_tiles_bwd: cannot set shared memory size");
    dim3 grid((unsigned)(klp / kTile), (unsigned)(qlp / 8), B);
    kern<<<grid, kTB, smem, s>>>(pair, out, kv_len, QL, KL, H, qlp, klp, causal ? 1 : 0);
    return check_launch("pair_tiles_bwd");
}

template <typename T>
int launch_dpair_from_tiles(const T* tiles, T* dpair, const int* kv_len, int64_t QL, int64_t KL, int H, int B,
                            bool causal, cudaStream_t s) {
    const int64_t qlp = pad_tile(QL), klp = pad_tile(KL);
    const size_t smem = (size_t)8 * kTile * H * sizeof(T);
    auto kern = dpair_from_tiles_kernel<T>;
    if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return fail(NNOP_ERR_CUDA, "dpair_from_tiles: cannot set shared memory size");
    dim3 grid((unsigned)(qlp / kTile), (unsigned)(klp / 8), B);
    kern<<<grid, kTB, smem, s>>>(tiles, dpair, kv_len, QL, KL, H, qlp, klp, causal ? 1 : 0);
    return check_launch("dpair_from_tiles");
}

template int launch_pair_tiles_fwd<__half>(const __half*, __half*, int64_t, int64_t, int, int, bool, cudaStream_t);
template int launch_pair_tiles_fwd<__nv_bfloat16>(const __nv_bfloat16*, __nv_bfloat16*, int64_t, int64_t, int, int,
                                                  bool, cudaStream_t);
template int launch_pair_tiles_bwd<__half>(const __half*, __half*, const int*, int64_t, int64_t, int, int, bool,
                                           cudaStream_t);
template int launch_pair_tiles_bwd<__nv_bfloat16>(const __nv_bfloat16*, __nv_bfloat16*, const int*, int64_t, int64_t,
                                                  int, int, bool, cudaStream_t);
template int launch_dpair_from_tiles<__half>(const __half*, __half*, const int*, int64_t, int64_t, int, int, bool,
                                             cudaStream_t);
template int launch_dpair_from_tiles<__nv_bfloat16>(const __nv_bfloat16*, __nv_bfloat16*, const int*, int64_t,
                                                    int64_t, int, int, bool, cudaStream_t);

}  // namespace fa_host
}  // namespace nnop
