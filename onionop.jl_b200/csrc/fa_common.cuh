// Shared definitions of the flash-attention kernels.
//
// Layouts (row-major buffers of the reference's column-major Julia arrays):
//   q, o, dO, dq   [B][QH][QL][E]
//   k, v, dk, dv   [B][KH][KL][E]
//   pair, dpair    [B][KL][QL][QH]      (Julia (QH, QL, KL, B), head innermost)
//   kpad_mask      [B][KL] uint8        (Julia (KL, B) Bool)
//   lse, delta     [B][QH][QL] float32
#pragma once

#include "common.cuh"

namespace nnop {
namespace fa {

constexpr float kLog2e = 1.4426950408889634f;

struct Params {
    const void* q;
    const void* k;
    const void* v;
    const void* pair;        // may be null
    const uint8_t* kmask;    // may be null
    void* o;
    float* lse;
    // backward
    const void* dO;
    const float* delta;      // rowsum(dO ∘ O), fp32
    float* dq_acc;           // fp32 accumulator [B][QH][QL][E] (bf16/f16 path)
    const int* kv_len;       // per-batch valid key count (last kept key + 1), or null
    void* dq;
    void* dk;
    void* dv;
    void* dpair;
    int64_t QL, KL;
    int E, QH, KH, B, n_rep;
    float scale;
    // pair / dpair laid out per head, [B][QH][KL][QL] (Julia (QL, KL, H, B)),
    // read and written by the tcgen05 kernels directly; 0: the reference's
    // head-innermost layout, which reaches them as per-head tiles (pair_tiles.cu)
    int pair_per_head;
    // Llama RoPE folded into the backward's outputs (the fused RoPE entry
    // points): when rope_cos is set, dq and dk leave the backward rotated by
    // the inverse rotation (sin → −sin), i.e. as gradients of the un-rotated
    // q and k.  Tables [rope_cb][L][E] fp32 (rope_cb = 1 or B), L = QL = KL;
    // pairs (e, e + E/2) use the cos/sin of index e (src/rope/llama_rope.jl:45-61).
    const float* rope_cos;
    const float* rope_sin;
    int64_t rope_cb;
};

// Index of the last kept key + 1 for one batch row of the key-padding mask
// (block-wide; every thread gets the result).  Key tiles at or beyond it are
// fully masked and contribute exp(−Inf) = 0, so skipping them is exact.
__device__ __forceinline__ int kv_valid_len_block(const uint8_t* __restrict__ m, int64_t KL) {
    __shared__ int s_len;
    if (threadIdx.x == 0) s_len = 0;
    __syncthreads();
    int best = 0;
    for (int64_t j = threadIdx.x; j < KL; j += blockDim.x)
        if (m[j]) best = (int)(j + 1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if ((threadIdx.x & 31) == 0 && best > 0) atomicMax(&s_len, best);
    __syncthreads();
    const int r = s_len;
    __syncthreads();
    return r;
}

}  // namespace fa

// Host-side helpers implemented in fa_common.cu.
namespace fa_host {
int launch_kv_len(const uint8_t* kmask, int* kv_len, int64_t KL, int B, cudaStream_t s);
template <typename T>
int launch_preprocess(const T* dO, const T* o, float* delta, int64_t rows, int E, cudaStream_t s);
template <typename T>
int launch_dpair_fill(T* dpair, const int* kv_len, int64_t QL, int64_t KL, int QH, int B, int tile,
                      bool causal, cudaStream_t s);
template <typename T>
int launch_convert(const float* src, T* dst, int64_t n, cudaStream_t s);
template <typename T>
int launch_convert_rope(const float* src, T* dst, const float* cos_t, const float* sin_t, int64_t cb, int64_t B,
                        int64_t QH, int64_t L, int E, cudaStream_t s);
}  // namespace fa_host

}  // namespace nnop
