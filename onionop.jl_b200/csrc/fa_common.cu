// Small memory-bound kernels around the flash-attention backward:
// * kv_len        : per-batch last kept key (+1) of the key-padding mask;
// * preprocess    : delta = rowsum(dO ∘ O) in fp32.  The reference computes
//                   Δs = Δ/l and δ = Σ Δs∘o (src/attention_bwd.jl:177-211); with
//                   the forward saving a normalised O and lse, δ = rowsum(dO∘O)
//                   is the same quantity and Δ needs no rescaled copy;
// * dpair_fill    : zeros of the dpair entries no backward CTA writes (tiles
//                   above the causal diagonal, fully masked key tiles), written
//                   head-innermost and coalesced.  The reference zero-fills the
//                   whole dpair first (`KA.zeros`, src/attention_bwd.jl:250-252);
//                   here every element is written exactly once;
// * convert       : fp32 dq accumulator -> dq dtype (convert_rope: with the
//                   inverse RoPE rotation, for the fused RoPE backward).
#include "fa_common.cuh"

namespace nnop {
namespace {

__global__ void kv_len_kernel(const uint8_t* __restrict__ kmask, int* __restrict__ kv_len, int64_t KL) {
    const int b = blockIdx.x;
    const int r = fa::kv_valid_len_block(kmask + (int64_t)b * KL, KL);
    if (threadIdx.x == 0) kv_len[b] = r;
}

// One thread per row of E elements; 16-byte vector loads.
template <typename T, int VEC>
__global__ void preprocess_kernel(const T* __restrict__ dO, const T* __restrict__ o, float* __restrict__ delta,
                                  int64_t rows, int E) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const T* a = dO + r * E;
    const T* c = o + r * E;
    float s = 0.f;
    for (int e = 0; e < E; e += VEC) {
        float av[VEC], cv[VEC];
        load_vec<T, VEC>(av, a + e);
        load_vec<T, VEC>(cv, c + e);
#pragma unroll
        for (int i = 0; i < VEC; ++i) s += av[i] * cv[i];
    }
    delta[r] = s;
}

// One CTA per (batch, key) row of dpair ([QL][QH] contiguous).  The backward
// kernels write query range [i_lo, QL) of key j; this kernel zeros [0, i_lo).
template <typename T>
__global__ void dpair_fill_kernel(T* __restrict__ dpair, const int* __restrict__ kv_len, int64_t QL, int64_t KL,
                                  int QH, int tile, int causal) {
    const int64_t row = blockIdx.x;
    const int64_t b = row / KL, j = row % KL;
    const int64_t jt = (j / tile) * tile;
    int64_t i_lo = causal ? jt : 0;
    if (kv_len != nullptr && jt >= kv_len[b]) i_lo = QL;
    if (i_lo > QL) i_lo = QL;
    T* base = dpair + row * QL * QH;
    const int64_t n = i_lo * QH;
    // 16-byte stores where the row start allows it.
    const int64_t head = ((16 - (reinterpret_cast<uintptr_t>(base) & 15)) & 15) / sizeof(T);
    const int64_t h = head < n ? head : n;
    for (int64_t x = threadIdx.x; x < h; x += blockDim.x) base[x] = from_f<T>(0.f);
    constexpr int V = 16 / sizeof(T);
    const int64_t nv = (n - h) / V;
    uint4 z = make_uint4(0, 0, 0, 0);
    uint4* vb = reinterpret_cast<uint4*>(base + h);
    for (int64_t x = threadIdx.x; x < nv; x += blockDim.x) __stcs(vb + x, z);
    for (int64_t x = h + nv * V + threadIdx.x; x < n; x += blockDim.x) base[x] = from_f<T>(0.f);
}

template <typename T>
__global__ void convert_kernel(const float* __restrict__ src, T* __restrict__ dst, int64_t n) {
    const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i + 3 < n) {
        float4 f = __ldcs(reinterpret_cast<const float4*>(src + i));
        dst[i] = from_f<T>(f.x);
        dst[i + 1] = from_f<T>(f.y);
        dst[i + 2] = from_f<T>(f.z);
        dst[i + 3] = from_f<T>(f.w);
    } else {
        for (int64_t k = i; k < n; ++k) dst[k] = from_f<T>(src[k]);
    }
}

// dq fp32 accumulator -> dq dtype with the inverse RoPE rotation (the fused
// RoPE backward): for the pair (e, e + E/2) of row (b, h, i),
//   dq[e] = a·cos + b·sin,   dq[e + E/2] = b·cos − a·sin,
// a, b the accumulator values, cos/sin of index e at position i (the
// reference's ∇llama_rope, src/rope/llama_rope.jl:86-92: sin → −sin).  One
// thread per 4 consecutive e of the first half.
template <typename T>
__global__ void convert_rope_kernel(const float* __restrict__ src, T* __restrict__ dst, const float* __restrict__ cos_t,
                                    const float* __restrict__ sin_t, int64_t cb, int64_t QH, int64_t L, int E,
                                    int64_t total) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= total) return;
    const int half = E / 2, q4 = half / 4;
    const int e = (int)(t % q4) * 4;
    const int64_t row = t / q4;                  // (b, h, i)
    const int64_t i = row % L, b = row / (L * QH);
    const int64_t tr = ((cb == 1 ? 0 : b) * L + i) * E + e;
    const float4 c = *reinterpret_cast<const float4*>(cos_t + tr);
    const float4 sn = *reinterpret_cast<const float4*>(sin_t + tr);
    const float4 a = __ldcs(reinterpret_cast<const float4*>(src + row * E + e));
    const float4 bb = __ldcs(reinterpret_cast<const float4*>(src + row * E + e + half));
    // 8-byte stores of the 4 results of each half
    Vec<T, 4> lo, hi;
    lo.v[0] = from_f<T>(a.x * c.x + bb.x * sn.x);
    lo.v[1] = from_f<T>(a.y * c.y + bb.y * sn.y);
    lo.v[2] = from_f<T>(a.z * c.z + bb.z * sn.z);
    lo.v[3] = from_f<T>(a.w * c.w + bb.w * sn.w);
    hi.v[0] = from_f<T>(bb.x * c.x - a.x * sn.x);
    hi.v[1] = from_f<T>(bb.y * c.y - a.y * sn.y);
    hi.v[2] = from_f<T>(bb.z * c.z - a.z * sn.z);
    hi.v[3] = from_f<T>(bb.w * c.w - a.w * sn.w);
    *reinterpret_cast<Vec<T, 4>*>(dst + row * E + e) = lo;
    *reinterpret_cast<Vec<T, 4>*>(dst + row * E + e + half) = hi;
}

}  // namespace

namespace fa_host {

int launch_kv_len(const uint8_t* kmask, int* kv_len, int64_t KL, int B, cudaStream_t s) {
    kv_len_kernel<<<B, 256, 0, s>>>(kmask, kv_len, KL);
    return check_launch("flash_attention kv_len");
}

template <typename T>
int launch_preprocess(const T* dO, const T* o, float* delta, int64_t rows, int E, cudaStream_t s) {
    const unsigned grid = (unsigned)((rows + 127) / 128);
    constexpr int V = 16 / sizeof(T);
    if (E % V == 0 && aligned16(dO) && aligned16(o))
        preprocess_kernel<T, V><<<grid, 128, 0, s>>>(dO, o, delta, rows, E);
    else
        preprocess_kernel<T, 1><<<grid, 128, 0, s>>>(dO, o, delta, rows, E);
    return check_launch("flash_attention_bwd preprocess");
}

template <typename T>
int launch_dpair_fill(T* dpair, const int* kv_len, int64_t QL, int64_t KL, int QH, int B, int tile, bool causal,
                      cudaStream_t s) {
    if (!causal && kv_len == nullptr) return NNOP_OK;
    const int64_t rows = (int64_t)B * KL;
    dpair_fill_kernel<T><<<(unsigned)rows, 256, 0, s>>>(dpair, kv_len, QL, KL, QH, tile, causal ? 1 : 0);
    return check_launch("flash_attention_bwd dpair fill");
}

template <typename T>
int launch_convert(const float* src, T* dst, int64_t n, cudaStream_t s) {
    const int64_t threads = (n + 3) / 4;
    convert_kernel<T><<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(src, dst, n);
    return check_launch("flash_attention_bwd dq convert");
}

template int launch_preprocess<float>(const float*, const float*, float*, int64_t, int, cudaStream_t);
template int launch_preprocess<__half>(const __half*, const __half*, float*, int64_t, int, cudaStream_t);
template int launch_preprocess<__nv_bfloat16>(const __nv_bfloat16*, const __nv_bfloat16*, float*, int64_t, int,
                                              cudaStream_t);
template int launch_dpair_fill<float>(float*, const int*, int64_t, int64_t, int, int, int, bool, cudaStream_t);
template int launch_dpair_fill<__half>(__half*, const int*, int64_t, int64_t, int, int, int, bool, cudaStream_t);
template int launch_dpair_fill<__nv_bfloat16>(__nv_bfloat16*, const int*, int64_t, int64_t, int, int, int, bool,
                                              cudaStream_t);
template <typename T>
int launch_convert_rope(const float* src, T* dst, const float* cos_t, const float* sin_t, int64_t cb, int64_t B,
                        int64_t QH, int64_t L, int E, cudaStream_t s) {
    const int64_t total = B * QH * L * (E / 8);
    if (total == 0) return NNOP_OK;
    convert_rope_kernel<T><<<(unsigned)((total + 255) / 256), 256, 0, s>>>(src, dst, cos_t, sin_t, cb, QH, L, E,
                                                                            total);
    return check_launch("flash_attention_bwd dq convert (rope)");
}

template int launch_convert_rope<__half>(const float*, __half*, const float*, const float*, int64_t, int64_t,
                                         int64_t, int64_t, int, cudaStream_t);
template int launch_convert_rope<__nv_bfloat16>(const float*, __nv_bfloat16*, const float*, const float*, int64_t,
                                                int64_t, int64_t, int64_t, int, cudaStream_t);
template int launch_convert<__half>(const float*, __half*, int64_t, cudaStream_t);
template int launch_convert<__nv_bfloat16>(const float*, __nv_bfloat16*, int64_t, cudaStream_t);

}  // namespace fa_host
}  // namespace nnop
