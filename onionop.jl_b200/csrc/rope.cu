// Llama RoPE (q and k in one launch) and the LlamaRotaryEmbedding cos/sin
// tables, for sm_100a.
//
// Reference: src/rope/llama_rope.jl -- `llama_rope!` (:24-65) gives each
// thread one sequence position of one head and walks E/2 element pairs with a
// thread stride of E (uncoalesced), on copies of q and k made first (:75-76).
//
// Here the launch is out of place (the copy is fused into the rotation: read q
// once, write q_out once).  A thread owns one 16-byte vector of the first half
// of a (batch, position) row and its partner vector E/2 further on for a group
// of kHeads heads: it loads the matching cos/sin values once, issues the loads
// of all its heads' q and k vectors before any arithmetic, then rotates and
// stores them.  Every q/k byte moves exactly once; the cos/sin rows are read
// once per head group (from L2 after the first): HBM bytes =
// 2·(|q| + |k|) + |cos| + |sin|.
#include "common.cuh"

namespace nnop {
namespace {

constexpr int kRopeBlock = 256;
constexpr int kHeads = 4;   // heads per thread

template <typename T, int VEC>
__global__ void __launch_bounds__(kRopeBlock)
rope_kernel(const T* __restrict__ q, const T* __restrict__ k, const float* __restrict__ cos_t,
            const float* __restrict__ sin_t, T* __restrict__ qo, T* __restrict__ ko, int E, int64_t L,
            int QH, int KH, int64_t B, int64_t cos_batch, float sign) {
    const int half = E / 2;
    const int nh = half / VEC;
    const int H = QH > KH ? QH : KH;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t per_group = B * L * nh;
    const int64_t total = per_group * ((H + kHeads - 1) / kHeads);
    if (t >= total) return;
    const int hg = (int)(t / per_group);   // head group: heads hg·kHeads ..
    const int64_t r = t % per_group;
    const int u = (int)(r % nh);
    const int64_t l = (r / nh) % L;
    const int64_t b = r / ((int64_t)nh * L);
    const int64_t cb = cos_batch == 1 ? 0 : b;
    const float* cr = cos_t + (cb * L + l) * E + u * VEC;
    const float* sr = sin_t + (cb * L + l) * E + u * VEC;
    float c[VEC], sn[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
        c[e] = __ldg(cr + e);
        sn[e] = __ldg(sr + e) * sign;
    }
    const int64_t head_stride = L * E;
    const int64_t qbase = (b * QH * L + l) * E + u * VEC;
    const int64_t kbase = (b * KH * L + l) * E + u * VEC;
    // all loads of the group first
    Vec<T, VEC> qa[kHeads], qb[kHeads], ka[kHeads], kb[kHeads];
#pragma unroll
    for (int j = 0; j < kHeads; ++j) {
        const int h = hg * kHeads + j;
        if (h < QH) {
            qa[j] = ldg_stream<T, VEC>(q + qbase + h * head_stride);
            qb[j] = ldg_stream<T, VEC>(q + qbase + h * head_stride + half);
        }
        if (h < KH) {
            ka[j] = ldg_stream<T, VEC>(k + kbase + h * head_stride);
            kb[j] = ldg_stream<T, VEC>(k + kbase + h * head_stride + half);
        }
    }
    auto rot = [&](const Vec<T, VEC>& a, const Vec<T, VEC>& bb, T* dst) {
        Vec<T, VEC> oa, ob;
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
            const float x1 = to_f(a.v[e]), x2 = to_f(bb.v[e]);
            oa.v[e] = from_f<T>(x1 * c[e] - x2 * sn[e]);
            ob.v[e] = from_f<T>(x2 * c[e] + x1 * sn[e]);
        }
        st_stream<T, VEC>(dst, oa);
        st_stream<T, VEC>(dst + half, ob);
    };
#pragma unroll
    for (int j = 0; j < kHeads; ++j) {
        const int h = hg * kHeads + j;
        if (h < QH) rot(qa[j], qb[j], qo + qbase + h * head_stride);
        if (h < KH) rot(ka[j], kb[j], ko + kbase + h * head_stride);
    }
}

// cos/sin of inv_freq[i mod dim/2] · position, inv_freq[i] = 1/base^(2i/dim),
// in float32 like `LlamaRotaryEmbedding` (src/rope/llama_rope.jl:7-22).
__global__ void rope_table_kernel(const float* __restrict__ pos, float* __restrict__ cos_t,
                                  float* __restrict__ sin_t, int dim, int64_t L, int64_t B, float base) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t total = B * L * dim;
    if (t >= total) return;
    const int i = (int)(t % dim);
    const int64_t bl = t / dim;
    const int half = dim / 2;
    const int j = i < half ? i : i - half;
    const float id = (float)(2 * j) / (float)dim;
    const float inv_freq = 1.0f / powf(base, id);
    const float f = inv_freq * pos[bl];
    cos_t[t] = cosf(f);
    sin_t[t] = sinf(f);
}

}  // namespace
}  // namespace nnop

using namespace nnop;

extern "C" {

int nnop_llama_rope(const void* q, const void* k, const float* cos_t, const float* sin_t, void* q_out,
                    void* k_out, int64_t E, int64_t L, int64_t QH, int64_t KH, int64_t B,
                    int64_t cos_batch, float sign, int dtype, void* stream) {
    if (E <= 0 || E % 2 != 0) return fail(NNOP_ERR_SHAPE, "llama_rope: embedding dim must be even and > 0");
    if (L < 0 || QH < 0 || KH < 0 || B < 0) return fail(NNOP_ERR_SHAPE, "llama_rope: negative dimension");
    if (cos_batch != B && cos_batch != 1)
        return fail(NNOP_ERR_SHAPE, "llama_rope: cos/sin batch must equal the q/k batch or be 1");
    if (E > (1 << 20) || QH > (1 << 20) || KH > (1 << 20)) return fail(NNOP_ERR_SHAPE, "llama_rope: dimension too large");
    if (L == 0 || B == 0 || (QH == 0 && KH == 0)) return NNOP_OK;
    if ((QH && (!q || !q_out)) || (KH && (!k || !k_out)) || !cos_t || !sin_t)
        return fail(NNOP_ERR_ARG, "llama_rope: NULL pointer");
    cudaStream_t s = (cudaStream_t)stream;
    const int half = (int)(E / 2);
    NNOP_DISPATCH_DTYPE(dtype, T, {
        constexpr int V = 16 / sizeof(T);
        bool vec = (half % V == 0) && aligned16(cos_t) && aligned16(sin_t) &&
                   (!QH || (aligned16(q) && aligned16(q_out))) && (!KH || (aligned16(k) && aligned16(k_out)));
        const int vw = vec ? V : 1;
        const int64_t H = QH > KH ? QH : KH;
        const int64_t total = B * L * (half / vw) * ((H + kHeads - 1) / kHeads);
        const unsigned grid = (unsigned)((total + kRopeBlock - 1) / kRopeBlock);
        if (vec) {
            rope_kernel<T, V><<<grid, kRopeBlock, 0, s>>>((const T*)q, (const T*)k, cos_t, sin_t, (T*)q_out,
                                                          (T*)k_out, (int)E, L, (int)QH, (int)KH, B,
                                                          cos_batch, sign);
        } else {
            rope_kernel<T, 1><<<grid, kRopeBlock, 0, s>>>((const T*)q, (const T*)k, cos_t, sin_t, (T*)q_out,
                                                          (T*)k_out, (int)E, L, (int)QH, (int)KH, B,
                                                          cos_batch, sign);
        }
    });
    return check_launch("llama_rope");
}

int nnop_llama_rope_cos_sin(const float* position_ids, float* cos_t, float* sin_t, int64_t dim, int64_t L,
                            int64_t B, int64_t base, void* stream) {
    if (dim <= 0 || dim % 2 != 0) return fail(NNOP_ERR_SHAPE, "llama_rope_cos_sin: dim must be even and > 0");
    if (L < 0 || B < 0) return fail(NNOP_ERR_SHAPE, "llama_rope_cos_sin: negative dimension");
    if (L == 0 || B == 0) return NNOP_OK;
    if (!position_ids || !cos_t || !sin_t) return fail(NNOP_ERR_ARG, "llama_rope_cos_sin: NULL pointer");
    const int64_t total = B * L * dim;
    rope_table_kernel<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        position_ids, cos_t, sin_t, (int)dim, L, B, (float)base);
    return check_launch("llama_rope_cos_sin");
}

}  // extern "C"
