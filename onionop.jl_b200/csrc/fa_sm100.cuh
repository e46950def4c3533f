// Helpers shared by the tcgen05 flash-attention kernels (forward and
// backward): fast exp2, 16-bit packing, and TMA tensor-map construction
// through the driver entry point (no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "fa_common.cuh"
#include "sm100.cuh"

namespace nnop {
namespace fa {
namespace {   // internal linkage: one copy per translation unit

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}

template <typename T>
__device__ __forceinline__ uint32_t pack16(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack16<__nv_bfloat16>(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack16<__half>(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = to_f(h[i]);
}

// Shifted identity for the pair-bias UMMA (scores += c·I · pair tile): 192
// rows of a K-major 128-byte-swizzled operand (1024-byte aligned) holding c at
// (row 64+m, column m) for m < 64 and zeros elsewhere.  K16 step kk of a
// 128x128x128 product reads rows [64, 192) (kk < 4) or [0, 128) (kk >= 4) at
// column block kk%4: that is c times the 128x128 identity restricted to
// columns [16kk, 16kk+16).
constexpr int kEyeBytes = 192 * 128;

template <typename T>
__device__ __forceinline__ void build_eye(uint8_t* eye, float c, int tid, int nthreads) {
    const uint32_t cb = pack16<T>(c, 0.f) & 0xffffu;
    for (int u = tid; u < kEyeBytes / 16; u += nthreads) {
        const int row = u >> 3, chunk = (u & 7) ^ (row & 7);   // logical 8-column chunk
        const int m = row - 64;
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        if (m >= 0 && m < 64 && (m >> 3) == chunk) w[(m & 7) >> 1] = cb << (16 * (m & 1));
        reinterpret_cast<uint4*>(eye)[u] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// Start address of K16 step kk of the shifted identity.
__device__ __forceinline__ uint32_t eye_step(uint32_t eye, int kk) {
    return eye + (kk < 4 ? 64 * 128 : 0) + (kk & 3) * 32;
}

// Warp-uniform bounded wait: true only if every lane saw the phase complete
// (guards warp-wide tcgen05.ld/st, which must not run divergent).
__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t parity, volatile int* ab, int site) {
    const bool ok = sm100::wait(bar, parity, ab, site);
    return __all_sync(0xffffffffu, ok);
}

// Two packed 16-bit values -> float (exact)
template <typename T>
__device__ __forceinline__ float lo16(uint32_t w);
template <typename T>
__device__ __forceinline__ float hi16(uint32_t w);
template <>
__device__ __forceinline__ float lo16<__nv_bfloat16>(uint32_t w) { return __uint_as_float(w << 16); }
template <>
__device__ __forceinline__ float hi16<__nv_bfloat16>(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
template <>
__device__ __forceinline__ float lo16<__half>(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)w)); }
template <>
__device__ __forceinline__ float hi16<__half>(uint32_t w) {
    return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}

// Backward elementwise step on 16 score columns of one key row (keys on TMEM
// lanes): Pᵀ = exp2(Sᵀ·scale·log2e + pairᵀ·log2e − lse) and dSᵀ = Pᵀ∘(dPᵀ − δ),
// packed to 16 bits.  lse is in log2 units; columns t outside [lo, hi) are
// masked (probability 0).  `pw`: the 16 pair values (packed), when PAIR.
template <typename T, bool PAIR, bool MASKED>
__device__ __forceinline__ void elementwise16(const uint32_t (&sr)[16], const uint32_t (&dr)[16],
                                              const uint32_t (&pw)[8], const float4 (&l4)[4],
                                              const float4 (&d4)[4], float sl2, int lo, int hi, uint32_t (&pk)[8],
                                              uint32_t (&dk)[8]) {
    const float* lse = reinterpret_cast<const float*>(l4);
    const float* del = reinterpret_cast<const float*>(d4);
#pragma unroll
    for (int t = 0; t < 16; t += 2) {
        float pv[2], dv[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            float off = -lse[t + u];
            if (PAIR) off = fmaf(u ? hi16<T>(pw[t >> 1]) : lo16<T>(pw[t >> 1]), kLog2e, off);
            float pr = ex2(fmaf(__uint_as_float(sr[t + u]), sl2, off));
            if (MASKED) pr = (t + u >= lo && t + u < hi) ? pr : 0.f;
            pv[u] = pr;
            dv[u] = pr * (__uint_as_float(dr[t + u]) - del[t + u]);
        }
        pk[t >> 1] = pack16<T>(pv[0], pv[1]);
        dk[t >> 1] = pack16<T>(dv[0], dv[1]);
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

// 3-D map over a [BH][rows][E] 16-bit tensor, box (64, box_rows, 1), 128-byte swizzle.
bool make_map(CUtensorMap* m, const void* base, int E, int64_t rows, int64_t bh, int box_rows, bool bf16) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)E, (cuuint64_t)rows, (cuuint64_t)bh};
    cuuint64_t strides[2] = {(cuuint64_t)E * 2, (cuuint64_t)rows * E * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// 4-D map over the per-head pair / dS tiles [B·H][QLp/128][KLp][128]
// (pair_tiles.cu), box (64, 128, 1, 1): one 64-query half of a (128-query,
// 128-key) tile, 128-byte swizzle.
bool make_tiles_map(CUtensorMap* m, const void* base, int64_t qlp, int64_t klp, int64_t bh, bool bf16) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[4] = {128, (cuuint64_t)klp, (cuuint64_t)(qlp / 128), (cuuint64_t)bh};
    cuuint64_t strides[3] = {256, (cuuint64_t)klp * 256, (cuuint64_t)(qlp / 128) * klp * 256};
    cuuint32_t box[4] = {64, 128, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// 3-D map over a pair bias laid out per head, [B·H][KL][QL] 16-bit (Julia
// (QL, KL, H, B)), box (64 queries, 128 keys, 1), 128-byte swizzle: the same
// [key][64 queries] half tile the per-head tiles map yields, read (or, for
// dpair, written) in place.  Rows past KL / columns past QL are zero-filled
// on loads and clipped on stores.  The row stride QL·2 bytes must be a
// multiple of 16 (QL % 8 == 0).
bool make_per_head_map(CUtensorMap* m, const void* base, int64_t QL, int64_t KL, int64_t bh, bool bf16) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)QL, (cuuint64_t)KL, (cuuint64_t)bh};
    cuuint64_t strides[2] = {(cuuint64_t)QL * 2, (cuuint64_t)QL * KL * 2};
    cuuint32_t box[3] = {64, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace
}  // namespace fa
}  // namespace nnop
