// Shared helpers for the NNop B200 kernels: dtype conversion, 16-byte vector
// access, warp/block reductions, status reporting for the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>
#include <string>

#include "../../include/nnop_b200.h"

namespace nnop {

// ---------------------------------------------------------------------------
// Status reporting (thread-local message, like the reference's error() text)
// ---------------------------------------------------------------------------
void set_error(const std::string& msg);
int fail(int status, const std::string& msg);
int check_launch(const char* what);
int num_sms();              // SM count of the current device (cached per device)

// ---------------------------------------------------------------------------
// dtype helpers
// ---------------------------------------------------------------------------
template <typename T> struct DT;
template <> struct DT<float> { static constexpr int id = NNOP_F32; };
template <> struct DT<__half> { static constexpr int id = NNOP_F16; };
template <> struct DT<__nv_bfloat16> { static constexpr int id = NNOP_BF16; };

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
    return __float2bfloat16_rn(x);
}

// A 16-byte vector of VEC elements of T (VEC = 16 / sizeof(T)), or a single
// element when VEC == 1 (scalar path for unaligned rows).
template <typename T, int VEC> struct alignas(sizeof(T) * VEC) Vec {
    T v[VEC];
};

template <typename T, int VEC>
__device__ __forceinline__ void load_vec(float (&out)[VEC], const T* p) {
    Vec<T, VEC> r = *reinterpret_cast<const Vec<T, VEC>*>(p);
#pragma unroll
    for (int i = 0; i < VEC; ++i) out[i] = to_f(r.v[i]);
}

// Streaming load: data read exactly once, do not keep it in L1.
template <typename T, int VEC>
__device__ __forceinline__ Vec<T, VEC> ldg_stream(const T* p) {
    if constexpr (sizeof(Vec<T, VEC>) == 16) {
        uint4 u = __ldcs(reinterpret_cast<const uint4*>(p));
        return *reinterpret_cast<Vec<T, VEC>*>(&u);
    } else {
        return *reinterpret_cast<const Vec<T, VEC>*>(p);
    }
}

template <typename T, int VEC>
__device__ __forceinline__ void st_stream(T* p, const Vec<T, VEC>& v) {
    if constexpr (sizeof(Vec<T, VEC>) == 16) {
        __stcs(reinterpret_cast<uint4*>(p), *reinterpret_cast<const uint4*>(&v));
    } else {
        *reinterpret_cast<Vec<T, VEC>*>(p) = v;
    }
}

template <typename T, int VEC>
__device__ __forceinline__ void store_vec(T* p, const float (&in)[VEC]) {
    Vec<T, VEC> r;
#pragma unroll
    for (int i = 0; i < VEC; ++i) r.v[i] = from_f<T>(in[i]);
    st_stream<T, VEC>(p, r);
}

// ---------------------------------------------------------------------------
// Reductions: warp shuffles plus one shared-memory stage (replaces the
// reference's log2(groupsize)-barrier tree, src/groupreduce.jl:13-43).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum of NV values at once; every thread receives the totals.
// `red` must hold 32 * NV floats.  Ends with a __syncthreads so `red` can be
// reused immediately.
template <int NV>
__device__ __forceinline__ void block_sum(float (&v)[NV], float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nw = (blockDim.x + 31) >> 5;
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = warp_sum(v[i]);
    if (lane == 0) {
#pragma unroll
        for (int i = 0; i < NV; ++i) red[i * 32 + warp] = v[i];
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        float t = lane < nw ? red[i * 32 + lane] : 0.f;
        v[i] = warp_sum(t);
    }
    __syncthreads();
}

__device__ __forceinline__ float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nw = (blockDim.x + 31) >> 5;
    v = warp_max(v);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : -INFINITY;
    v = warp_max(t);
    __syncthreads();
    return v;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace nnop

#define NNOP_DISPATCH_DTYPE(dtype, T, ...)                                  \
    switch (dtype) {                                                        \
        case NNOP_F32: { using T = float; __VA_ARGS__; } break;             \
        case NNOP_F16: { using T = __half; __VA_ARGS__; } break;            \
        case NNOP_BF16: { using T = __nv_bfloat16; __VA_ARGS__; } break;    \
        default: return nnop::fail(NNOP_ERR_DTYPE, "unsupported dtype " + std::to_string(dtype)); \
    }
