// Online softmax over the contiguous axis, forward and backward, for sm_100a.
//
// Reference: src/softmax.jl -- `online_softmax!` (:19-58) reads x twice (an
// online (max, denominator) pass and a write pass); its backward (:70-80) is
// three unfused broadcast/reduction launches.
//
// Here one CTA owns one row (a Julia column of length n) at a time and keeps
// it in registers as 16-byte vectors, so the forward reads x once and writes y
// once (2·n·s bytes per row) and the backward reads dy and y once and writes dx
// once (3·n·s).  Rows too long to cache fall back to re-reading (the second
// read mostly hits L2).  Semantics follow the reference: an all −Inf row gives
// NaN (exp(−Inf − (−Inf))).
#include "common.cuh"

namespace nnop {
namespace {

constexpr int kSmBlock = 256;
constexpr int kSmMaxNV = 16;

template <typename T, int VEC, int NV>
__global__ void __launch_bounds__(kSmBlock)
softmax_fwd_kernel(const T* __restrict__ x, T* __restrict__ y, int n, int64_t rows) {
    __shared__ float red[32];
    const int nvec = n / VEC;
    const int tid = threadIdx.x, nt = blockDim.x;
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const T* xr = x + row * (int64_t)n;
        T* yr = y + row * (int64_t)n;
        if constexpr (NV > 0) {
            Vec<T, VEC> xc[NV];
            float m = -INFINITY;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
                    xc[i] = ldg_stream<T, VEC>(xr + idx * VEC);
#pragma unroll
                    for (int e = 0; e < VEC; ++e) m = fmaxf(m, to_f(xc[i].v[e]));
                }
            }
            m = block_max(m, red);
            float d[1] = {0.f};
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
#pragma unroll
                    for (int e = 0; e < VEC; ++e) d[0] += expf(to_f(xc[i].v[e]) - m);
                }
            }
            block_sum<1>(d, red);
            const float inv = 1.0f / d[0];
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
                    float o[VEC];
#pragma unroll
                    for (int e = 0; e < VEC; ++e) o[e] = expf(to_f(xc[i].v[e]) - m) * inv;
                    store_vec<T, VEC>(yr + idx * VEC, o);
                }
            }
        } else {
            float m = -INFINITY;
            for (int idx = tid; idx < nvec; idx += nt) {
                float xv[VEC];
                load_vec<T, VEC>(xv, xr + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) m = fmaxf(m, xv[e]);
            }
            m = block_max(m, red);
            float d[1] = {0.f};
            for (int idx = tid; idx < nvec; idx += nt) {
                float xv[VEC];
                load_vec<T, VEC>(xv, xr + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) d[0] += expf(xv[e] - m);
            }
            block_sum<1>(d, red);
            const float inv = 1.0f / d[0];
            for (int idx = tid; idx < nvec; idx += nt) {
                float xv[VEC], o[VEC];
                load_vec<T, VEC>(xv, xr + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) o[e] = expf(xv[e] - m) * inv;
                store_vec<T, VEC>(yr + idx * VEC, o);
            }
        }
    }
}

// dx = dy∘y − y∘Σ(dy∘y)
template <typename T, int VEC, int NV>
__global__ void __launch_bounds__(kSmBlock)
softmax_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ y, T* __restrict__ dx, int n,
                   int64_t rows) {
    __shared__ float red[32];
    const int nvec = n / VEC;
    const int tid = threadIdx.x, nt = blockDim.x;
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const T* dr = dy + row * (int64_t)n;
        const T* yr = y + row * (int64_t)n;
        T* xr = dx + row * (int64_t)n;
        float s[1] = {0.f};
        if constexpr (NV > 0) {
            Vec<T, VEC> dc[NV], yc[NV];
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
                    dc[i] = ldg_stream<T, VEC>(dr + idx * VEC);
                    yc[i] = ldg_stream<T, VEC>(yr + idx * VEC);
#pragma unroll
                    for (int e = 0; e < VEC; ++e) s[0] += to_f(dc[i].v[e]) * to_f(yc[i].v[e]);
                }
            }
            block_sum<1>(s, red);
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
                    float o[VEC];
#pragma unroll
                    for (int e = 0; e < VEC; ++e) {
                        const float yv = to_f(yc[i].v[e]);
                        o[e] = to_f(dc[i].v[e]) * yv - yv * s[0];
                    }
                    store_vec<T, VEC>(xr + idx * VEC, o);
                }
            }
        } else {
            for (int idx = tid; idx < nvec; idx += nt) {
                float dv[VEC], yv[VEC];
                load_vec<T, VEC>(dv, dr + idx * VEC);
                load_vec<T, VEC>(yv, yr + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) s[0] += dv[e] * yv[e];
            }
            block_sum<1>(s, red);
            for (int idx = tid; idx < nvec; idx += nt) {
                float dv[VEC], yv[VEC], o[VEC];
                load_vec<T, VEC>(dv, dr + idx * VEC);
                load_vec<T, VEC>(yv, yr + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) o[e] = dv[e] * yv[e] - yv[e] * s[0];
                store_vec<T, VEC>(xr + idx * VEC, o);
            }
        }
    }
}

struct SmPlan {
    bool vec;
    int block;
    int nv;
};

template <typename T>
SmPlan plan(int n, std::initializer_list<const void*> ptrs) {
    constexpr int V = 16 / sizeof(T);
    bool vec = (n % V == 0);
    for (const void* p : ptrs) vec = vec && aligned16(p);
    const int nvec = vec ? n / V : n;
    int block = ((nvec + 31) / 32) * 32;
    if (block > kSmBlock) block = kSmBlock;
    if (block < 32) block = 32;
    const int per = (nvec + block - 1) / block;
    int nv = 1;
    while (nv < per) nv *= 2;
    if (nv > kSmMaxNV) nv = 0;
    return {vec, block, nv};
}

#define NNOP_SM_NV_SWITCH(nv, NVC, ...)                          \
    switch (nv) {                                                \
        case 1: { constexpr int NVC = 1; __VA_ARGS__; } break;   \
        case 2: { constexpr int NVC = 2; __VA_ARGS__; } break;   \
        case 4: { constexpr int NVC = 4; __VA_ARGS__; } break;   \
        case 8: { constexpr int NVC = 8; __VA_ARGS__; } break;   \
        case 16: { constexpr int NVC = 16; __VA_ARGS__; } break; \
        default: { constexpr int NVC = 0; __VA_ARGS__; } break;  \
    }

int check_args(int64_t n, int64_t cols) {
    if (n <= 0 || cols < 0) return fail(NNOP_ERR_SHAPE, "online_softmax: n must be > 0 and cols >= 0");
    if (n > (int64_t)1 << 28) return fail(NNOP_ERR_SHAPE, "online_softmax: n too large (max 2^28)");
    return NNOP_OK;
}

}  // namespace
}  // namespace nnop

using namespace nnop;

extern "C" {

int nnop_online_softmax_fwd(const void* x, void* y, int64_t n, int64_t cols, int dtype, void* stream) {
    int st = check_args(n, cols);
    if (st) return st;
    if (cols == 0) return NNOP_OK;
    if (!x || !y) return fail(NNOP_ERR_ARG, "online_softmax_fwd: NULL pointer");
    cudaStream_t s = (cudaStream_t)stream;
    const unsigned grid = (unsigned)(cols < (1 << 30) ? cols : (1 << 30));
    NNOP_DISPATCH_DTYPE(dtype, T, {
        SmPlan p = plan<T>((int)n, {x, y});
        if (p.vec) {
            constexpr int VC = 16 / sizeof(T);
            NNOP_SM_NV_SWITCH(p.nv, NVC, {
                softmax_fwd_kernel<T, VC, NVC><<<grid, p.block, 0, s>>>((const T*)x, (T*)y, (int)n, cols);
            });
        } else {
            NNOP_SM_NV_SWITCH(p.nv, NVC, {
                softmax_fwd_kernel<T, 1, NVC><<<grid, p.block, 0, s>>>((const T*)x, (T*)y, (int)n, cols);
            });
        }
    });
    return check_launch("online_softmax_fwd");
}

int nnop_online_softmax_bwd(const void* dy, const void* y, void* dx, int64_t n, int64_t cols, int dtype,
                            void* stream) {
    int st = check_args(n, cols);
    if (st) return st;
    if (cols == 0) return NNOP_OK;
    if (!dy || !y || !dx) return fail(NNOP_ERR_ARG, "online_softmax_bwd: NULL pointer");
    cudaStream_t s = (cudaStream_t)stream;
    const unsigned grid = (unsigned)(cols < (1 << 30) ? cols : (1 << 30));
    NNOP_DISPATCH_DTYPE(dtype, T, {
        SmPlan p = plan<T>((int)n, {dy, y, dx});
        if (p.vec) {
            constexpr int VC = 16 / sizeof(T);
            NNOP_SM_NV_SWITCH(p.nv, NVC, {
                softmax_bwd_kernel<T, VC, NVC><<<grid, p.block, 0, s>>>((const T*)dy, (const T*)y, (T*)dx,
                                                                        (int)n, cols);
            });
        } else {
            NNOP_SM_NV_SWITCH(p.nv, NVC, {
                softmax_bwd_kernel<T, 1, NVC><<<grid, p.block, 0, s>>>((const T*)dy, (const T*)y, (T*)dx,
                                                                       (int)n, cols);
            });
        }
    });
    return check_launch("online_softmax_bwd");
}

}  // extern "C"
