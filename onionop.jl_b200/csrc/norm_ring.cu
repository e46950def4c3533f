// RMSNorm and LayerNorm, forward and backward, streamed through a ring of
// shared-memory row buffers (sm_100a).
//
// Reference: src/rms_norm.jl (kernels :3-115) and src/layer_norm.jl (kernels
// :8-148).  These ops move 2·N·s (forward) or 3·N·s (backward) bytes and do
// little arithmetic, so their speed is how many bytes each SM keeps in flight.
// A persistent CTA here walks rows blockIdx.x, +gridDim.x, ... with S row
// buffers in shared memory filled by bulk asynchronous copies
// (cp.async.bulk, completion counted on one mbarrier per buffer): while the
// CTA reduces and writes row r, rows r+1 .. r+S-1 are already on their way.
// Each thread reads its 16-byte vectors of the row from shared memory once,
// keeps them in registers for the reduction and the output, and the buffer is
// refilled (row r+S) right after the row's block reduction -- the point by
// which every thread has read it.  The arithmetic runs on packed fp32 pairs
// (FFMA2 / FADD2 / FMUL2): with 16-bit rows these kernels issue more
// instructions per byte than anything else limits them by.  Rows too long for
// S >= 3 buffers, or not 16-byte aligned, and the fp32 forward passes and
// RMSNorm backward (faster with the one-row-per-CTA / register-prefetch
// kernels, measured) take the kernels of norm.cu.
// Every mbarrier wait is bounded (sm100::wait) and its result made uniform
// over the block through the row's reduction, so a wait that gives up ends
// the CTA without a divergent __syncthreads; in-flight copies are waited for
// (bounded) before exit.
#include <cuda.h>

#include "common.cuh"
#include "sm100.cuh"

namespace nnop {
namespace {

using namespace sm100;

constexpr int kRingThreads = 256;
constexpr int kMaxStages = 8;
constexpr int kRingSmemBudget = 96 * 1024;   // two CTAs per SM

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__host__ __device__ constexpr uint32_t align128(uint32_t x) { return (x + 127u) & ~127u; }

// The ring: S buffers of NT row slots each (NT = tensors streamed per row).
template <int NT>
struct Ring {
    uint8_t* base;
    uint32_t slot;        // bytes of one row slot (128-byte aligned)
    uint32_t row_bytes;   // bytes of one row
    int S;
    uint64_t* full;
    __device__ uint8_t* at(int s, int t) const { return base + ((size_t)s * NT + t) * slot; }
    // thread 0: copy row `row` of the NT tensors into buffer it % S
    __device__ void issue(int64_t it, int64_t row, const void* const* src) const {
        const int s = (int)(it % S);
        mbar_expect_tx(&full[s], NT * row_bytes);
#pragma unroll
        for (int t = 0; t < NT; ++t)
            bulk_load(at(s, t), reinterpret_cast<const uint8_t*>(src[t]) + row * (int64_t)row_bytes, row_bytes,
                      &full[s]);
    }
};

// Shared preamble of the ring kernels: barriers, the row count of this CTA.
struct RingCtl {
    int64_t first, stride, rows;
};
__device__ __forceinline__ RingCtl ring_ctl(int64_t n) {
    RingCtl c;
    c.first = blockIdx.x;
    c.stride = gridDim.x;
    c.rows = c.first < n ? (n - 1 - c.first) / c.stride + 1 : 0;
    return c;
}

// Bounded wait for buffer it % S by this thread.  The kernels make the result
// uniform over the block through the row's block reduction (a count of the
// threads whose wait gave up travels with the sums), so a wait that gives up
// ends the CTA after that reduction, with no divergent barrier and no extra
// one; a thread whose wait gave up reads a stale buffer, whose values are
// never used.
template <int NT>
__device__ __forceinline__ float ring_wait(const Ring<NT>& r, int64_t it, volatile int* ab) {
    const int s = (int)(it % r.S);
    return wait(&r.full[s], (uint32_t)((it / r.S) & 1), ab, 0) ? 0.f : 1.f;
}
// The same wait made uniform by a barrier of its own (true: every thread saw
// the buffer land) -- cheaper where the row's reduction carries one value.
template <int NT>
__device__ __forceinline__ bool ring_wait_all(const Ring<NT>& r, int64_t it, volatile int* ab) {
    return __syncthreads_and(ring_wait(r, it, ab) == 0.f) != 0;
}

// After an abort: thread 0 waits (bounded, without the abort flag) for the
// copies it issued that nobody consumed, so none is in flight at exit.
template <int NT>
__device__ __forceinline__ void ring_drain(const Ring<NT>& r, int64_t it, int64_t issued) {
    if (threadIdx.x != 0) return;
    for (int64_t j = it; j < issued; ++j) wait(&r.full[j % r.S], (uint32_t)((j / r.S) & 1), nullptr, 1);
}

template <int NT>
__device__ __forceinline__ Ring<NT> ring_init(uint8_t* smem, uint64_t* full, int emb, int esize, int S) {
    Ring<NT> r;
    r.base = smem;
    r.row_bytes = (uint32_t)emb * (uint32_t)esize;
    r.slot = align128(r.row_bytes);
    r.S = S;
    r.full = full;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    return r;
}

template <typename T, int NV>
__device__ __forceinline__ void load_slot(Vec<T, 16 / sizeof(T)> (&v)[NV], const uint8_t* slot, int nvec) {
    constexpr int V = 16 / sizeof(T);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int idx = threadIdx.x + i * kRingThreads;
        if (idx < nvec) v[i] = *reinterpret_cast<const Vec<T, V>*>(slot + (size_t)idx * 16);
    }
}

// Packed fp32x2 arithmetic (sm_100 FFMA2 / FADD2 / FMUL2): two elements per
// instruction; these ops issue more instructions per byte than the memory
// system needs cycles, so halving the arithmetic matters.
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// Element pair j of a 16-byte vector, as float2 (exact conversion).
template <typename T>
__device__ __forceinline__ float2 pair_f2(const Vec<T, 16 / sizeof(T)>& v, int j);
template <>
__device__ __forceinline__ float2 pair_f2<float>(const Vec<float, 4>& v, int j) {
    return make_float2(v.v[2 * j], v.v[2 * j + 1]);
}
template <>
__device__ __forceinline__ float2 pair_f2<__nv_bfloat16>(const Vec<__nv_bfloat16, 8>& v, int j) {
    const uint32_t w = reinterpret_cast<const uint32_t*>(&v)[j];
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 pair_f2<__half>(const Vec<__half, 8>& v, int j) {
    return __half22float2(reinterpret_cast<const __half2*>(&v)[j]);
}

// A 16-byte vector of T from V/2 float2 pairs (round to nearest).
template <typename T>
__device__ __forceinline__ void store_pairs(T* dst, const float2* pr);
template <>
__device__ __forceinline__ void store_pairs<float>(float* dst, const float2* pr) {
    __stcs(reinterpret_cast<float4*>(dst), make_float4(pr[0].x, pr[0].y, pr[1].x, pr[1].y));
}
template <>
__device__ __forceinline__ void store_pairs<__nv_bfloat16>(__nv_bfloat16* dst, const float2* pr) {
    uint32_t u[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 h = __float22bfloat162_rn(pr[j]);
        u[j] = *reinterpret_cast<uint32_t*>(&h);
    }
    __stcs(reinterpret_cast<uint4*>(dst), make_uint4(u[0], u[1], u[2], u[3]));
}
template <>
__device__ __forceinline__ void store_pairs<__half>(__half* dst, const float2* pr) {
    uint32_t u[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        __half2 h = __float22half2_rn(pr[j]);
        u[j] = *reinterpret_cast<uint32_t*>(&h);
    }
    __stcs(reinterpret_cast<uint4*>(dst), make_uint4(u[0], u[1], u[2], u[3]));
}

// A pair rounded to T and widened back (the values a T tensor stores).
template <typename T>
__device__ __forceinline__ float2 round_pair(float2 v);
template <>
__device__ __forceinline__ float2 round_pair<float>(float2 v) { return v; }
template <>
__device__ __forceinline__ float2 round_pair<__nv_bfloat16>(float2 v) { return __bfloat1622float2(__float22bfloat162_rn(v)); }
template <>
__device__ __forceinline__ float2 round_pair<__half>(float2 v) { return __half22float2(__float22half2_rn(v)); }

// The thread's NV vectors of a row-length array in global memory (w, b), as float2 pairs.
template <typename T, int NV>
__device__ __forceinline__ void load_pairs(float2 (&out)[NV][8 / sizeof(T)], const T* src, int nvec, float add) {
    constexpr int V = 16 / sizeof(T), P = V / 2;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int idx = threadIdx.x + i * kRingThreads;
        Vec<T, V> v;
        if (idx < nvec) v = *reinterpret_cast<const Vec<T, V>*>(src + (size_t)idx * V);
#pragma unroll
        for (int j = 0; j < P; ++j) out[i][j] = idx < nvec ? add2(pair_f2<T>(v, j), f2(add)) : f2(0.f);
    }
}

// ---------------------------------------------------------------- RMSNorm fwd
template <typename T, int NV>
__global__ void __launch_bounds__(kRingThreads, NV * 16 / sizeof(T) <= 16 ? 2 : 1)
rms_fwd_ring_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y, float* __restrict__ rstd_out,
                    int emb, int64_t n, float eps, float offset, float inv_emb, int S) {
    constexpr int V = 16 / sizeof(T), P = V / 2;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[kMaxStages];
    __shared__ float red[64];
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = 0;
    const int nvec = emb / V, tid = threadIdx.x;
    const RingCtl c = ring_ctl(n);
    const Ring<1> r = ring_init<1>(smem, full, emb, sizeof(T), S);
    const void* const src[1] = {x};
    int64_t issued = 0;
    if (tid == 0)
        for (; issued < c.rows && issued < S; ++issued) r.issue(issued, c.first + issued * c.stride, src);
    float2 wo[NV][P];
    load_pairs<T, NV>(wo, w, nvec, offset);
    int64_t it = 0;
    for (; it < c.rows; ++it) {
        const int64_t row = c.first + it * c.stride;
        if (!ring_wait_all(r, it, &s_abort)) break;
        Vec<T, V> xv[NV];
        load_slot<T, NV>(xv, r.at((int)(it % S), 0), nvec);
        float2 acc = f2(0.f);
#pragma unroll
        for (int i = 0; i < NV; ++i)
            if (tid + i * kRingThreads < nvec)
#pragma unroll
                for (int j = 0; j < P; ++j) {
                    const float2 x2 = pair_f2<T>(xv[i], j);
                    acc = fma2(x2, x2, acc);
                }
        float ss[1] = {acc.x + acc.y};
        block_sum<1>(ss, red);
        if (tid == 0 && it + S < c.rows) {   // every thread has read buffer it % S
            fence_proxy_async_smem();
            r.issue(it + S, c.first + (it + S) * c.stride, src);
            issued = it + S + 1;
        }
        const float rs = 1.0f / sqrtf(ss[0] * inv_emb + eps);
        if (tid == 0) rstd_out[row] = rs;
        const float2 rs2 = f2(rs);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int idx = tid + i * kRingThreads;
            if (idx < nvec) {
                float2 o[P];
#pragma unroll
                for (int j = 0; j < P; ++j) o[j] = mul2(mul2(pair_f2<T>(xv[i], j), rs2), wo[i][j]);
                store_pairs<T>(y + row * (int64_t)emb + idx * V, o);
            }
        }
    }
    if (it < c.rows) ring_drain(r, it, issued);
}

// ---------------------------------------------------------------- residual add + RMSNorm fwd
// h = x + residual, stored in T (the values a separate add would store), and
// y = (w + offset)·h·rstd(h): one pass over x and residual instead of an add
// pass and a norm pass that reads h back.
template <typename T, int NV>
__global__ void __launch_bounds__(kRingThreads, NV * 16 / sizeof(T) <= 16 ? 2 : 1)
add_rms_fwd_ring_kernel(const T* __restrict__ x, const T* __restrict__ res, const T* __restrict__ w,
                        T* __restrict__ h, T* __restrict__ y, float* __restrict__ rstd_out, int emb, int64_t n,
                        float eps, float offset, float inv_emb, int S) {
    constexpr int V = 16 / sizeof(T), P = V / 2;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[kMaxStages];
    __shared__ float red[32];
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = 0;
    const int nvec = emb / V, tid = threadIdx.x;
    const RingCtl c = ring_ctl(n);
    const Ring<2> r = ring_init<2>(smem, full, emb, sizeof(T), S);
    const void* const src[2] = {x, res};
    int64_t issued = 0;
    if (tid == 0)
        for (; issued < c.rows && issued < S; ++issued) r.issue(issued, c.first + issued * c.stride, src);
    float2 wo[NV][P];
    load_pairs<T, NV>(wo, w, nvec, offset);
    int64_t it = 0;
    for (; it < c.rows; ++it) {
        const int64_t row = c.first + it * c.stride;
        if (!ring_wait_all(r, it, &s_abort)) break;
        const int s = (int)(it % S);
        Vec<T, V> xv[NV], rv[NV];
        load_slot<T, NV>(xv, r.at(s, 0), nvec);
        load_slot<T, NV>(rv, r.at(s, 1), nvec);
        float2 hv[NV][P];
        float2 acc = f2(0.f);
#pragma unroll
        for (int i = 0; i < NV; ++i)
#pragma unroll
            for (int j = 0; j < P; ++j) {
                hv[i][j] = round_pair<T>(add2(pair_f2<T>(xv[i], j), pair_f2<T>(rv[i], j)));
                if (tid + i * kRingThreads < nvec) acc = fma2(hv[i][j], hv[i][j], acc);
            }
        float ss[1] = {acc.x + acc.y};
        block_sum<1>(ss, red);
        if (tid == 0 && it + S < c.rows) {
            fence_proxy_async_smem();
            r.issue(it + S, c.first + (it + S) * c.stride, src);
            issued = it + S + 1;
        }
        const float rs = 1.0f / sqrtf(ss[0] * inv_emb + eps);
        if (tid == 0) rstd_out[row] = rs;
        const float2 rs2 = f2(rs);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int idx = tid + i * kRingThreads;
            if (idx < nvec) {
                float2 o[P];
#pragma unroll
                for (int j = 0; j < P; ++j) o[j] = mul2(mul2(hv[i][j], rs2), wo[i][j]);
                store_pairs<T>(h + row * (int64_t)emb + idx * V, hv[i]);
                store_pairs<T>(y + row * (int64_t)emb + idx * V, o);
            }
        }
    }
    if (it < c.rows) ring_drain(r, it, issued);
}

// ---------------------------------------------------------------- RMSNorm bwd
// dx = rstd·m − rstd³/N·(Σ m∘x)·x with m = dy∘(w+offset); dw partial += dy∘x·rstd.
// ADD: dx += dh, a third streamed tensor (the residual stream's gradient of
// the fused residual add + RMSNorm).
template <typename T, int NV, bool ADD = false>
__global__ void __launch_bounds__(kRingThreads, NV * 16 / sizeof(T) <= 16 ? 2 : 1)
rms_bwd_ring_kernel(const T* __restrict__ dy, const T* __restrict__ x, const T* __restrict__ w,
                    const float* __restrict__ rstd, T* __restrict__ dx, float* __restrict__ partial, int emb,
                    int64_t n, float offset, float inv_emb, int S, const T* __restrict__ dh) {
    constexpr int V = 16 / sizeof(T), P = V / 2;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[kMaxStages];
    __shared__ float red[64];
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = 0;
    const int nvec = emb / V, tid = threadIdx.x;
    const RingCtl c = ring_ctl(n);
    constexpr int NT = ADD ? 3 : 2;
    const Ring<NT> r = ring_init<NT>(smem, full, emb, sizeof(T), S);
    const void* const src[3] = {x, dy, dh};
    int64_t issued = 0;
    if (tid == 0)
        for (; issued < c.rows && issued < S; ++issued) r.issue(issued, c.first + issued * c.stride, src);
    float2 wo[NV][P], dwa[NV][P];
    load_pairs<T, NV>(wo, w, nvec, offset);
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int j = 0; j < P; ++j) dwa[i][j] = f2(0.f);
    int64_t it = 0;
    for (; it < c.rows; ++it) {
        const int64_t row = c.first + it * c.stride;
        const float rs = rstd[row];
        if (!ring_wait_all(r, it, &s_abort)) break;
        const int s = (int)(it % S);
        Vec<T, V> xv[NV], dv[NV], hv[ADD ? NV : 1];
        load_slot<T, NV>(xv, r.at(s, 0), nvec);
        load_slot<T, NV>(dv, r.at(s, 1), nvec);
        if constexpr (ADD) load_slot<T, NV>(hv, r.at(s, NT - 1), nvec);   // before the buffer is refilled
        float2 acc = f2(0.f);
#pragma unroll
        for (int i = 0; i < NV; ++i)
            if (tid + i * kRingThreads < nvec)
#pragma unroll
                for (int j = 0; j < P; ++j)
                    acc = fma2(mul2(pair_f2<T>(dv[i], j), wo[i][j]), pair_f2<T>(xv[i], j), acc);
        float dd[1] = {acc.x + acc.y};
        block_sum<1>(dd, red);
        if (tid == 0 && it + S < c.rows) {
            fence_proxy_async_smem();
            r.issue(it + S, c.first + (it + S) * c.stride, src);
            issued = it + S + 1;
        }
        const float2 rs2 = f2(rs), crs2 = f2(-inv_emb * rs * rs * dd[0] * rs);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int idx = tid + i * kRingThreads;
            if (idx < nvec) {
                float2 o[P];
#pragma unroll
#pragma unroll
                for (int j = 0; j < P; ++j) {
                    const float2 d2 = pair_f2<T>(dv[i], j), x2 = pair_f2<T>(xv[i], j);
                    o[j] = fma2(crs2, x2, mul2(rs2, mul2(d2, wo[i][j])));
                    if constexpr (ADD) o[j] = add2(o[j], pair_f2<T>(hv[i], j));
                    dwa[i][j] = fma2(d2, mul2(x2, rs2), dwa[i][j]);
                }
                store_pairs<T>(dx + row * (int64_t)emb + idx * V, o);
            }
        }
    }
    if (it < c.rows) ring_drain(r, it, issued);
    float* prow = partial + (int64_t)blockIdx.x * emb;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int idx = tid + i * kRingThreads;
        if (idx < nvec)
#pragma unroll
            for (int j = 0; j < P; ++j) reinterpret_cast<float2*>(prow + idx * V)[j] = dwa[i][j];
    }
}

// ---------------------------------------------------------------- LayerNorm fwd
// Mean and biased variance (src/layer_norm.jl:21-62) from ONE block reduction
// of the shifted sums s1 = Σ(x−K), s2 = Σ(x−K)² with K = the row's first
// element (read from the row buffer): mean = K + s1/N, var = s2/N − (s1/N)².
// Shifting by a sample of the row keeps (mean − K)² of the order of the
// variance, so the subtraction loses no more than a few ulps (the shifted-data
// algorithm); it saves the second reduction's two block barriers per row.
template <typename T, int NV>
__global__ void __launch_bounds__(kRingThreads, NV * 16 / sizeof(T) <= 16 ? 2 : 1)
ln_fwd_ring_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ b, T* __restrict__ y,
                   float* __restrict__ mean_out, float* __restrict__ rstd_out, int emb, int64_t n, float eps,
                   float inv_emb, int S) {
    constexpr int V = 16 / sizeof(T), P = V / 2;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[kMaxStages];
    __shared__ float red[96];
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = 0;
    const int nvec = emb / V, tid = threadIdx.x;
    const RingCtl c = ring_ctl(n);
    const Ring<1> r = ring_init<1>(smem, full, emb, sizeof(T), S);
    const void* const src[1] = {x};
    int64_t issued = 0;
    if (tid == 0)
        for (; issued < c.rows && issued < S; ++issued) r.issue(issued, c.first + issued * c.stride, src);
    float2 wv[NV][P], bv[NV][P];
    load_pairs<T, NV>(wv, w, nvec, 0.f);
    load_pairs<T, NV>(bv, b, nvec, 0.f);
    int64_t it = 0;
    for (; it < c.rows; ++it) {
        const int64_t row = c.first + it * c.stride;
        if (!ring_wait_all(r, it, &s_abort)) break;
        Vec<T, V> xv[NV];
        load_slot<T, NV>(xv, r.at((int)(it % S), 0), nvec);
        const float K = to_f(*reinterpret_cast<const T*>(r.at((int)(it % S), 0)));
        const float2 nk2 = f2(-K);
        float2 a1 = f2(0.f), a2 = f2(0.f);
#pragma unroll
        for (int i = 0; i < NV; ++i)
            if (tid + i * kRingThreads < nvec)
#pragma unroll
                for (int j = 0; j < P; ++j) {
                    const float2 d = add2(pair_f2<T>(xv[i], j), nk2);
                    a1 = add2(a1, d);
                    a2 = fma2(d, d, a2);
                }
        float sm[2] = {a1.x + a1.y, a2.x + a2.y};
        block_sum<2>(sm, red);
        if (tid == 0 && it + S < c.rows) {
            fence_proxy_async_smem();
            r.issue(it + S, c.first + (it + S) * c.stride, src);
            issued = it + S + 1;
        }
        const float m1 = sm[0] * inv_emb;
        const float mu = K + m1;
        const float var = fmaxf(sm[1] * inv_emb - m1 * m1, 0.f);
        const float rs = 1.0f / sqrtf(var + eps);
        if (tid == 0) { mean_out[row] = mu; rstd_out[row] = rs; }
        const float2 rs2 = f2(rs), nmr2 = f2(-mu * rs);   // (x − mu)·rs = x·rs − mu·rs
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int idx = tid + i * kRingThreads;
            if (idx < nvec) {
                float2 o[P];
#pragma unroll
                for (int j = 0; j < P; ++j) o[j] = fma2(fma2(pair_f2<T>(xv[i], j), rs2, nmr2), wv[i][j], bv[i][j]);
                store_pairs<T>(y + row * (int64_t)emb + idx * V, o);
            }
        }
    }
    if (it < c.rows) ring_drain(r, it, issued);
}

// ---------------------------------------------------------------- LayerNorm bwd
// c1 = mean(w·dy·xn), c2 = mean(w·dy); dx = (w·dy − (xn·c1 + c2))·rstd;
// dw partial += dy·xn; db partial += dy      (src/layer_norm.jl:94-137)
template <typename T, int NV>
__global__ void __launch_bounds__(kRingThreads, NV * 16 / sizeof(T) <= 16 ? 2 : 1)
ln_bwd_ring_kernel(const T* __restrict__ dy, const T* __restrict__ x, const T* __restrict__ w,
                   const float* __restrict__ mean, const float* __restrict__ rstd, T* __restrict__ dx,
                   float* __restrict__ partial, int emb, int64_t n, float inv_emb, int S) {
    constexpr int V = 16 / sizeof(T), P = V / 2;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[kMaxStages];
    __shared__ float red[96];
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = 0;
    const int nvec = emb / V, tid = threadIdx.x;
    const RingCtl c = ring_ctl(n);
    const Ring<2> r = ring_init<2>(smem, full, emb, sizeof(T), S);
    const void* const src[2] = {x, dy};
    int64_t issued = 0;
    if (tid == 0)
        for (; issued < c.rows && issued < S; ++issued) r.issue(issued, c.first + issued * c.stride, src);
    float2 wv[NV][P], dwa[NV][P], dba[NV][P];
    load_pairs<T, NV>(wv, w, nvec, 0.f);
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int j = 0; j < P; ++j) { dwa[i][j] = f2(0.f); dba[i][j] = f2(0.f); }
    int64_t it = 0;
    for (; it < c.rows; ++it) {
        const int64_t row = c.first + it * c.stride;
        const float mu = mean[row], rs = rstd[row];
        const float gave_up = ring_wait(r, it, &s_abort);
        const int s = (int)(it % S);
        Vec<T, V> xv[NV], dv[NV];
        load_slot<T, NV>(xv, r.at(s, 0), nvec);
        load_slot<T, NV>(dv, r.at(s, 1), nvec);
        const float2 rs2 = f2(rs), nmr2 = f2(-mu * rs);
        // 16-bit rows keep xn = (x − mu)·rs and dy as float2 for the output
        // (their conversion is the costly part); fp32 rows recompute them,
        // which needs fewer registers
        constexpr bool kKeep = sizeof(T) == 2;
        float2 xn[kKeep ? NV : 1][P], d2[kKeep ? NV : 1][P];
        float2 a1 = f2(0.f), a2 = f2(0.f);
#pragma unroll
        for (int i = 0; i < NV; ++i)
#pragma unroll
            for (int j = 0; j < P; ++j) {
                const float2 xnv = fma2(pair_f2<T>(xv[i], j), rs2, nmr2);
                const float2 dyv = pair_f2<T>(dv[i], j);
                if constexpr (kKeep) { xn[i][j] = xnv; d2[i][j] = dyv; }
                if (tid + i * kRingThreads < nvec) {
                    const float2 wdy = mul2(wv[i][j], dyv);
                    a1 = fma2(wdy, xnv, a1);
                    a2 = add2(a2, wdy);
                }
            }
        float cs[3] = {a1.x + a1.y, a2.x + a2.y, gave_up};
        block_sum<3>(cs, red);
        if (cs[2] != 0.f) break;
        if (tid == 0 && it + S < c.rows) {
            fence_proxy_async_smem();
            r.issue(it + S, c.first + (it + S) * c.stride, src);
            issued = it + S + 1;
        }
        // dx = (wdy − xn·c1 − c2)·rstd = wdy·rstd + xn·(−c1·rstd) + (−c2·rstd)
        const float2 nc1 = f2(-cs[0] * inv_emb * rs), nc2 = f2(-cs[1] * inv_emb * rs);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int idx = tid + i * kRingThreads;
            if (idx < nvec) {
                float2 o[P];
#pragma unroll
                for (int j = 0; j < P; ++j) {
                    float2 xnv, dyv;
                    if constexpr (kKeep) {
                        xnv = xn[i][j];
                        dyv = d2[i][j];
                    } else {
                        xnv = fma2(pair_f2<T>(xv[i], j), rs2, nmr2);
                        dyv = pair_f2<T>(dv[i], j);
                    }
                    o[j] = fma2(mul2(wv[i][j], dyv), rs2, fma2(xnv, nc1, nc2));
                    dwa[i][j] = fma2(dyv, xnv, dwa[i][j]);
                    dba[i][j] = add2(dba[i][j], dyv);
                }
                store_pairs<T>(dx + row * (int64_t)emb + idx * V, o);
            }
        }
    }
    if (it < c.rows) ring_drain(r, it, issued);
    float* pw = partial + (int64_t)blockIdx.x * 2 * emb;
    float* pb = pw + emb;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int idx = tid + i * kRingThreads;
        if (idx < nvec)
#pragma unroll
            for (int j = 0; j < P; ++j) {
                reinterpret_cast<float2*>(pw + idx * V)[j] = dwa[i][j];
                reinterpret_cast<float2*>(pb + idx * V)[j] = dba[i][j];
            }
    }
}

// ---------------------------------------------------------------- planning
struct RingPlan {
    bool ok;
    int nv;      // 16-byte vectors per thread: 1, 2, 4 or 8
    int S;       // buffers
    int smem;    // dynamic shared memory bytes
};

// The ring applies when the rows are 16-byte vectors (emb·s % 16 == 0, every
// base 16-byte aligned), a thread holds at most 8 vectors and `max_elems`
// elements of a row (the backward kernels also keep dw/db accumulators per
// element, which spill beyond 32), and at least 3 buffers of NT row slots fit
// in the per-CTA budget.
template <typename T>
RingPlan plan_ring(int emb, int NT, std::initializer_list<const void*> ptrs, int max_elems = 1 << 30) {
    RingPlan p{false, 0, 0, 0};
    const int row_bytes = emb * (int)sizeof(T);
    if (row_bytes % 16 != 0) return p;
    for (const void* q : ptrs)
        if (q != nullptr && !aligned16(q)) return p;
    const int nvec = row_bytes / 16;
    const int per = (nvec + kRingThreads - 1) / kRingThreads;
    int nv = 1;
    while (nv < per) nv *= 2;
    if (nv > 8 || nv * (16 / (int)sizeof(T)) > max_elems) return p;
    const int stage = NT * (int)align128((uint32_t)row_bytes);
    int S = kRingSmemBudget / stage;
    if (S > kMaxStages) S = kMaxStages;
    if (S < 3) return p;
    return {true, nv, S, S * stage};
}

#define NNOP_RING_NV_SWITCH(nv, NVC, ...)                      \
    switch (nv) {                                              \
        case 1: { constexpr int NVC = 1; __VA_ARGS__; } break; \
        case 2: { constexpr int NVC = 2; __VA_ARGS__; } break; \
        case 4: { constexpr int NVC = 4; __VA_ARGS__; } break; \
        default: { constexpr int NVC = 8; __VA_ARGS__; } break; \
    }

// Persistent grid: SM count × resident CTAs (for the given shared memory),
// at most `cap_per_sm` per SM and at most one CTA per row.
template <typename KernelT>
int ring_grid(KernelT kern, int smem, int64_t n, int cap_per_sm) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return 0;
    int occ = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kRingThreads, smem) != cudaSuccess || occ < 1)
        occ = 1;
    if (occ > cap_per_sm) occ = cap_per_sm;
    int64_t g = (int64_t)num_sms() * occ;
    if (g > n) g = n;
    return (int)(g < 1 ? 1 : g);
}

}  // namespace

// Host entry points used by norm.cu: each returns true when the ring path
// applies and was launched (*st holds the launch status), false otherwise.
namespace ring {

template <typename T>
bool rms_fwd(const T* x, const T* w, T* y, float* rstd, int emb, int64_t n, float eps, float offset, cudaStream_t s,
             int* st) {
    if (sizeof(T) == 4) return false;   // fp32 rows: the one-row-per-CTA kernel is faster (measured)
    const RingPlan p = plan_ring<T>(emb, 1, {x, w, y});
    if (!p.ok) return false;
    NNOP_RING_NV_SWITCH(p.nv, NVC, {
        auto kern = rms_fwd_ring_kernel<T, NVC>;
        const int g = ring_grid(kern, p.smem, n, 8);
        if (g == 0) return false;
        kern<<<g, kRingThreads, p.smem, s>>>(x, w, y, rstd, emb, n, eps, offset, 1.0f / (float)emb, p.S);
    });
    *st = check_launch("rms_norm_fwd (ring)");
    return true;
}

template <typename T>
bool rms_bwd(const T* dy, const T* x, const T* w, const float* rstd, T* dx, float* partial, int emb, int64_t n,
             float offset, int max_parts, cudaStream_t s, int* parts, int* st) {
    if (sizeof(T) == 4) return false;   // fp32 rows: the register-prefetch kernel is faster (measured)
    const RingPlan p = plan_ring<T>(emb, 2, {dy, x, w, dx}, 32);
    if (!p.ok) return false;
    NNOP_RING_NV_SWITCH(p.nv, NVC, {
        auto kern = rms_bwd_ring_kernel<T, NVC>;
        int g = ring_grid(kern, p.smem, n, 8);
        if (g == 0) return false;
        if (g > max_parts) g = max_parts;
        *parts = g;
        kern<<<g, kRingThreads, p.smem, s>>>(dy, x, w, rstd, dx, partial, emb, n, offset, 1.0f / (float)emb, p.S,
                                              nullptr);
    });
    *st = check_launch("rms_norm_bwd (ring)");
    return true;
}

template <typename T>
bool add_rms_fwd(const T* x, const T* res, const T* w, T* h, T* y, float* rstd, int emb, int64_t n, float eps,
                 float offset, cudaStream_t s, int* st) {
    const RingPlan p = plan_ring<T>(emb, 2, {x, res, w, h, y});
    if (!p.ok) return false;
    NNOP_RING_NV_SWITCH(p.nv, NVC, {
        auto kern = add_rms_fwd_ring_kernel<T, NVC>;
        const int g = ring_grid(kern, p.smem, n, 8);
        if (g == 0) return false;
        kern<<<g, kRingThreads, p.smem, s>>>(x, res, w, h, y, rstd, emb, n, eps, offset, 1.0f / (float)emb, p.S);
    });
    *st = check_launch("add_rms_norm_fwd (ring)");
    return true;
}

// RMSNorm backward plus dh (the fused residual add's gradient): every dtype
// through the ring when it applies.
template <typename T>
bool rms_bwd_add(const T* dy, const T* dh, const T* x, const T* w, const float* rstd, T* dx, float* partial, int emb,
                 int64_t n, float offset, int max_parts, cudaStream_t s, int* parts, int* st) {
    const RingPlan p = plan_ring<T>(emb, 3, {dy, dh, x, w, dx}, 32);
    if (!p.ok) return false;
    NNOP_RING_NV_SWITCH(p.nv, NVC, {
        auto kern = rms_bwd_ring_kernel<T, NVC, true>;
        int g = ring_grid(kern, p.smem, n, 8);
        if (g == 0) return false;
        if (g > max_parts) g = max_parts;
        *parts = g;
        kern<<<g, kRingThreads, p.smem, s>>>(dy, x, w, rstd, dx, partial, emb, n, offset, 1.0f / (float)emb, p.S,
                                              dh);
    });
    *st = check_launch("add_rms_norm_bwd (ring)");
    return true;
}

template <typename T>
bool ln_fwd(const T* x, const T* w, const T* b, T* y, float* mean, float* rstd, int emb, int64_t n, float eps,
            cudaStream_t s, int* st) {
    if (sizeof(T) == 4) return false;   // fp32 rows: the one-row-per-CTA kernel is as fast or faster (measured)
    const RingPlan p = plan_ring<T>(emb, 1, {x, w, b, y});
    if (!p.ok) return false;
    NNOP_RING_NV_SWITCH(p.nv, NVC, {
        auto kern = ln_fwd_ring_kernel<T, NVC>;
        const int g = ring_grid(kern, p.smem, n, 8);
        if (g == 0) return false;
        kern<<<g, kRingThreads, p.smem, s>>>(x, w, b, y, mean, rstd, emb, n, eps, 1.0f / (float)emb, p.S);
    });
    *st = check_launch("layer_norm_fwd (ring)");
    return true;
}

template <typename T>
bool ln_bwd(const T* dy, const T* x, const T* w, const float* mean, const float* rstd, T* dx, float* partial,
            int emb, int64_t n, int max_parts, cudaStream_t s, int* parts, int* st) {
    const RingPlan p = plan_ring<T>(emb, 2, {dy, x, w, dx}, 32);
    if (!p.ok) return false;
    NNOP_RING_NV_SWITCH(p.nv, NVC, {
        auto kern = ln_bwd_ring_kernel<T, NVC>;
        int g = ring_grid(kern, p.smem, n, 8);
        if (g == 0) return false;
        if (g > max_parts) g = max_parts;
        *parts = g;
        kern<<<g, kRingThreads, p.smem, s>>>(dy, x, w, mean, rstd, dx, partial, emb, n, 1.0f / (float)emb, p.S);
    });
    *st = check_launch("layer_norm_bwd (ring)");
    return true;
}

#define NNOP_RING_INST(T)                                                                                          \
    template bool rms_fwd<T>(const T*, const T*, T*, float*, int, int64_t, float, float, cudaStream_t, int*);    \
    template bool rms_bwd<T>(const T*, const T*, const T*, const float*, T*, float*, int, int64_t, float, int,   \
                             cudaStream_t, int*, int*);                                                          \
    template bool ln_fwd<T>(const T*, const T*, const T*, T*, float*, float*, int, int64_t, float, cudaStream_t, \
                            int*);                                                                               \
    template bool ln_bwd<T>(const T*, const T*, const T*, const float*, const float*, T*, float*, int, int64_t,  \
                            int, cudaStream_t, int*, int*);                                                      \
    template bool add_rms_fwd<T>(const T*, const T*, const T*, T*, T*, float*, int, int64_t, float, float,        \
                                 cudaStream_t, int*);                                                            \
    template bool rms_bwd_add<T>(const T*, const T*, const T*, const T*, const float*, T*, float*, int, int64_t,  \
                                 float, int, cudaStream_t, int*, int*);
NNOP_RING_INST(float)
NNOP_RING_INST(__half)
NNOP_RING_INST(__nv_bfloat16)

}  // namespace ring
}  // namespace nnop
