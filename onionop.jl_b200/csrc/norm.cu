// RMSNorm and LayerNorm, forward and backward, for sm_100a.
//
// Reference: src/rms_norm.jl (kernels :3-115, launchers :117-169) and
// src/layer_norm.jl (kernels :8-148, launchers :150-204).
//
// Design (HBM-bound, 2·N·s bytes forward, 3·N·s backward):
// * one CTA normalises one row (a Julia column of length emb) at a time; each
//   thread holds its slice of the row in registers as raw 16-byte vectors, so x
//   (and dy) are read from HBM exactly once; CTAs that walk several rows load
//   the next row's vectors while the current row is reduced and written (the
//   backward, and the 16-bit forward, which runs persistent CTAs);
// * reductions are warp shuffles plus one shared-memory stage;
// * the backward runs a persistent grid (SM count x resident CTAs); a thread
//   owns the same columns for every row it visits, so dw/db accumulate in
//   registers, and each CTA writes one fp32 partial row to the workspace.  A
//   second, deterministic kernel sums the partials over CTAs (the reference
//   sums a (n/4, emb) partial with `sum(dw; dims=1)`, src/rms_norm.jl:162-167).
// * rows whose length is not a multiple of the 16-byte vector, or unaligned
//   base pointers, take the same kernels with a vector width of one element.
#include <cuda.h>

#include "common.cuh"

#include <mutex>

namespace nnop {
namespace {

constexpr int kNormBlock = 256;
constexpr int kMaxNV = 16;  // register-cached vectors per thread

// ---------------------------------------------------------------- RMSNorm fwd
template <typename T, int VEC, int NV>
__global__ void __launch_bounds__(kNormBlock)
rms_fwd_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y,
               float* __restrict__ rstd_out, int emb, int64_t n, float eps, float offset,
               float inv_emb) {
    __shared__ float red[32];
    const int nvec = emb / VEC;
    const int tid = threadIdx.x, nt = blockDim.x;
    if constexpr (NV > 0) {
        // persistent CTAs; the next row is loaded while this one is reduced and written
        Vec<T, VEC> xn_[NV];
        auto load_row = [&](int64_t row) {
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (row < n && idx < nvec) xn_[i] = ldg_stream<T, VEC>(x + row * (int64_t)emb + idx * VEC);
            }
        };
        load_row(blockIdx.x);
        for (int64_t row = blockIdx.x; row < n; row += gridDim.x) {
            T* yr = y + row * (int64_t)emb;
            Vec<T, VEC> xc[NV];
#pragma unroll
            for (int i = 0; i < NV; ++i) xc[i] = xn_[i];
            load_row(row + gridDim.x);
            float ss[1] = {0.f};
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
#pragma unroll
                    for (int e = 0; e < VEC; ++e) {
                        const float f = to_f(xc[i].v[e]);
                        ss[0] += f * f;
                    }
                }
            }
            block_sum<1>(ss, red);
            const float r = 1.0f / sqrtf(ss[0] * inv_emb + eps);
            if (tid == 0) rstd_out[row] = r;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
                    float wv[VEC], o[VEC];
                    load_vec<T, VEC>(wv, w + idx * VEC);
#pragma unroll
                    for (int e = 0; e < VEC; ++e) o[e] = (offset + wv[e]) * to_f(xc[i].v[e]) * r;
                    store_vec<T, VEC>(yr + idx * VEC, o);
                }
            }
        }
    } else {
        for (int64_t row = blockIdx.x; row < n; row += gridDim.x) {
            const T* xr = x + row * (int64_t)emb;
            T* yr = y + row * (int64_t)emb;
            float ss[1] = {0.f};
            for (int idx = tid; idx < nvec; idx += nt) {
                float xv[VEC];
                load_vec<T, VEC>(xv, xr + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) ss[0] += xv[e] * xv[e];
            }
            block_sum<1>(ss, red);
            const float r = 1.0f / sqrtf(ss[0] * inv_emb + eps);
            if (tid == 0) rstd_out[row] = r;
            for (int idx = tid; idx < nvec; idx += nt) {
                float xv[VEC], wv[VEC], o[VEC];
                load_vec<T, VEC>(xv, xr + idx * VEC);
                load_vec<T, VEC>(wv, w + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) o[e] = (offset + wv[e]) * xv[e] * r;
                store_vec<T, VEC>(yr + idx * VEC, o);
            }
        }
    }
}

// RMSNorm fwd, one row per CTA (no prefetch): the faster form for fp32 rows
template <typename T, int VEC, int NV>
__global__ void __launch_bounds__(kNormBlock)
rms_fwd_rowwise_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y,
               float* __restrict__ rstd_out, int emb, int64_t n, float eps, float offset,
               float inv_emb) {
    __shared__ float red[32];
    const int nvec = emb / VEC;
    const int tid = threadIdx.x, nt = blockDim.x;
    for (int64_t row = blockIdx.x; row < n; row += gridDim.x) {
        const T* xr = x + row * (int64_t)emb;
        T* yr = y + row * (int64_t)emb;
        float ss[1] = {0.f};
        if constexpr (NV > 0) {
            Vec<T, VEC> xc[NV];
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
                    xc[i] = ldg_stream<T, VEC>(xr + idx * VEC);
#pragma unroll
                    for (int e = 0; e < VEC; ++e) {
                        float f = to_f(xc[i].v[e]);
                        ss[0] += f * f;
                    }
                }
            }
            block_sum<1>(ss, red);
            const float r = 1.0f / sqrtf(ss[0] * inv_emb + eps);
            if (tid == 0) rstd_out[row] = r;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
                    float wv[VEC], o[VEC];
                    load_vec<T, VEC>(wv, w + idx * VEC);
#pragma unroll
                    for (int e = 0; e < VEC; ++e) o[e] = (offset + wv[e]) * to_f(xc[i].v[e]) * r;
                    store_vec<T, VEC>(yr + idx * VEC, o);
                }
            }
        } else {
            for (int idx = tid; idx < nvec; idx += nt) {
                float xv[VEC];
                load_vec<T, VEC>(xv, xr + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) ss[0] += xv[e] * xv[e];
            }
            block_sum<1>(ss, red);
            const float r = 1.0f / sqrtf(ss[0] * inv_emb + eps);
            if (tid == 0) rstd_out[row] = r;
            for (int idx = tid; idx < nvec; idx += nt) {
                float xv[VEC], wv[VEC], o[VEC];
                load_vec<T, VEC>(xv, xr + idx * VEC);
                load_vec<T, VEC>(wv, w + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) o[e] = (offset + wv[e]) * xv[e] * r;
                store_vec<T, VEC>(yr + idx * VEC, o);
            }
        }
    }
}

// ---------------------------------------------------------------- RMSNorm bwd
// dx = rstd·m + rstd·(−rstd²/N·dd·x), m = dy∘(w+offset), dd = Σ m∘x
// dw partial += dy∘x·rstd      (src/rms_norm.jl:97-101)
template <typename T, int VEC, int NV>
__global__ void __launch_bounds__(kNormBlock)
rms_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ x, const T* __restrict__ w,
               const float* __restrict__ rstd, T* __restrict__ dx, float* __restrict__ partial,
               int emb, int64_t n, float offset, float inv_emb) {
    __shared__ float red[32];
    const int nvec = emb / VEC;
    const int tid = threadIdx.x, nt = blockDim.x;
    float* prow = partial + (int64_t)blockIdx.x * emb;
    if constexpr (NV > 0) {
        float wo[NV][VEC], dwa[NV][VEC];
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int idx = tid + i * nt;
#pragma unroll
            for (int e = 0; e < VEC; ++e) { wo[i][e] = 0.f; dwa[i][e] = 0.f; }
            if (idx < nvec) {
                float wv[VEC];
                load_vec<T, VEC>(wv, w + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) wo[i][e] = wv[e] + offset;
            }
        }
        // the next row's x and dy are loaded while this row is reduced and written
        Vec<T, VEC> xn_[NV], dn_[NV];
        auto load_row = [&](int64_t row) {
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (row < n && idx < nvec) {
                    xn_[i] = ldg_stream<T, VEC>(x + row * (int64_t)emb + idx * VEC);
                    dn_[i] = ldg_stream<T, VEC>(dy + row * (int64_t)emb + idx * VEC);
                }
            }
        };
        load_row(blockIdx.x);
        for (int64_t row = blockIdx.x; row < n; row += gridDim.x) {
            Vec<T, VEC> xc[NV], dc[NV];
#pragma unroll
            for (int i = 0; i < NV; ++i) { xc[i] = xn_[i]; dc[i] = dn_[i]; }
            load_row(row + gridDim.x);
            float dd[1] = {0.f};
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
#pragma unroll
                    for (int e = 0; e < VEC; ++e) dd[0] += to_f(dc[i].v[e]) * wo[i][e] * to_f(xc[i].v[e]);
                }
            }
            block_sum<1>(dd, red);
            const float r = rstd[row];
            const float c = -inv_emb * r * r * dd[0];
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
                    float o[VEC];
#pragma unroll
                    for (int e = 0; e < VEC; ++e) {
                        const float d = to_f(dc[i].v[e]), xv = to_f(xc[i].v[e]);
                        o[e] = r * (d * wo[i][e]) + r * (c * xv);
                        dwa[i][e] += d * (xv * r);
                    }
                    store_vec<T, VEC>(dx + row * (int64_t)emb + idx * VEC, o);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int idx = tid + i * nt;
            if (idx < nvec) {
#pragma unroll
                for (int e = 0; e < VEC; ++e) prow[idx * VEC + e] = dwa[i][e];
            }
        }
    } else {
        for (int idx = tid; idx < nvec * VEC; idx += nt) prow[idx] = 0.f;
        for (int64_t row = blockIdx.x; row < n; row += gridDim.x) {
            const T* xr = x + row * (int64_t)emb;
            const T* dr = dy + row * (int64_t)emb;
            float dd[1] = {0.f};
            for (int idx = tid; idx < nvec; idx += nt) {
                float xv[VEC], dv[VEC], wv[VEC];
                load_vec<T, VEC>(xv, xr + idx * VEC);
                load_vec<T, VEC>(dv, dr + idx * VEC);
                load_vec<T, VEC>(wv, w + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) dd[0] += dv[e] * (wv[e] + offset) * xv[e];
            }
            block_sum<1>(dd, red);
            const float r = rstd[row];
            const float c = -inv_emb * r * r * dd[0];
            for (int idx = tid; idx < nvec; idx += nt) {
                float xv[VEC], dv[VEC], wv[VEC], o[VEC];
                load_vec<T, VEC>(xv, xr + idx * VEC);
                load_vec<T, VEC>(dv, dr + idx * VEC);
                load_vec<T, VEC>(wv, w + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) {
                    o[e] = r * (dv[e] * (wv[e] + offset)) + r * (c * xv[e]);
                    prow[idx * VEC + e] += dv[e] * (xv[e] * r);
                }
                store_vec<T, VEC>(dx + row * (int64_t)emb + idx * VEC, o);
            }
        }
    }
}

// ---------------------------------------------------------------- LayerNorm fwd
// Two passes over the register-cached row: mean, then biased variance
// (src/layer_norm.jl:21-62).
template <typename T, int VEC, int NV>
__global__ void __launch_bounds__(kNormBlock)
ln_fwd_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ b,
              T* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out,
              int emb, int64_t n, float eps, float inv_emb) {
    __shared__ float red[32];
    const int nvec = emb / VEC;
    const int tid = threadIdx.x, nt = blockDim.x;
    if constexpr (NV > 0) {
        // persistent CTAs; the next row is loaded while this one is reduced and written
        Vec<T, VEC> xn_[NV];
        auto load_row = [&](int64_t row) {
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (row < n && idx < nvec) xn_[i] = ldg_stream<T, VEC>(x + row * (int64_t)emb + idx * VEC);
            }
        };
        load_row(blockIdx.x);
        for (int64_t row = blockIdx.x; row < n; row += gridDim.x) {
            T* yr = y + row * (int64_t)emb;
            Vec<T, VEC> xc[NV];
#pragma unroll
            for (int i = 0; i < NV; ++i) xc[i] = xn_[i];
            load_row(row + gridDim.x);
            float s[1] = {0.f};
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
#pragma unroll
                    for (int e = 0; e < VEC; ++e) s[0] += to_f(xc[i].v[e]);
                }
            }
            block_sum<1>(s, red);
            const float mu = s[0] * inv_emb;
            float v[1] = {0.f};
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
#pragma unroll
                    for (int e = 0; e < VEC; ++e) {
                        const float c = to_f(xc[i].v[e]) - mu;
                        v[0] += c * c;
                    }
                }
            }
            block_sum<1>(v, red);
            const float r = 1.0f / sqrtf(v[0] * inv_emb + eps);
            if (tid == 0) { mean_out[row] = mu; rstd_out[row] = r; }
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
                    float wv[VEC], bv[VEC], o[VEC];
                    load_vec<T, VEC>(wv, w + idx * VEC);
                    load_vec<T, VEC>(bv, b + idx * VEC);
#pragma unroll
                    for (int e = 0; e < VEC; ++e) o[e] = (to_f(xc[i].v[e]) - mu) * r * wv[e] + bv[e];
                    store_vec<T, VEC>(yr + idx * VEC, o);
                }
            }
        }
    } else {
        for (int64_t row = blockIdx.x; row < n; row += gridDim.x) {
            const T* xr = x + row * (int64_t)emb;
            T* yr = y + row * (int64_t)emb;
            float s[1] = {0.f};
            for (int idx = tid; idx < nvec; idx += nt) {
                float xv[VEC];
                load_vec<T, VEC>(xv, xr + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) s[0] += xv[e];
            }
            block_sum<1>(s, red);
            const float mu = s[0] * inv_emb;
            float v[1] = {0.f};
            for (int idx = tid; idx < nvec; idx += nt) {
                float xv[VEC];
                load_vec<T, VEC>(xv, xr + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) { const float c = xv[e] - mu; v[0] += c * c; }
            }
            block_sum<1>(v, red);
            const float r = 1.0f / sqrtf(v[0] * inv_emb + eps);
            if (tid == 0) { mean_out[row] = mu; rstd_out[row] = r; }
            for (int idx = tid; idx < nvec; idx += nt) {
                float xv[VEC], wv[VEC], bv[VEC], o[VEC];
                load_vec<T, VEC>(xv, xr + idx * VEC);
                load_vec<T, VEC>(wv, w + idx * VEC);
                load_vec<T, VEC>(bv, b + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) o[e] = (xv[e] - mu) * r * wv[e] + bv[e];
                store_vec<T, VEC>(yr + idx * VEC, o);
            }
        }
    }
}

// LayerNorm fwd, one row per CTA (no prefetch): the faster form for fp32 rows
template <typename T, int VEC, int NV>
__global__ void __launch_bounds__(kNormBlock)
ln_fwd_rowwise_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ b,
              T* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out,
              int emb, int64_t n, float eps, float inv_emb) {
    __shared__ float red[32];
    const int nvec = emb / VEC;
    const int tid = threadIdx.x, nt = blockDim.x;
    for (int64_t row = blockIdx.x; row < n; row += gridDim.x) {
        const T* xr = x + row * (int64_t)emb;
        T* yr = y + row * (int64_t)emb;
        float s[1] = {0.f};
        if constexpr (NV > 0) {
            Vec<T, VEC> xc[NV];
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
                    xc[i] = ldg_stream<T, VEC>(xr + idx * VEC);
#pragma unroll
                    for (int e = 0; e < VEC; ++e) s[0] += to_f(xc[i].v[e]);
                }
            }
            block_sum<1>(s, red);
            const float mu = s[0] * inv_emb;
            float v[1] = {0.f};
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
#pragma unroll
                    for (int e = 0; e < VEC; ++e) {
                        const float c = to_f(xc[i].v[e]) - mu;
                        v[0] += c * c;
                    }
                }
            }
            block_sum<1>(v, red);
            const float r = 1.0f / sqrtf(v[0] * inv_emb + eps);
            if (tid == 0) { mean_out[row] = mu; rstd_out[row] = r; }
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
                    float wv[VEC], bv[VEC], o[VEC];
                    load_vec<T, VEC>(wv, w + idx * VEC);
                    load_vec<T, VEC>(bv, b + idx * VEC);
#pragma unroll
                    for (int e = 0; e < VEC; ++e) o[e] = (to_f(xc[i].v[e]) - mu) * r * wv[e] + bv[e];
                    store_vec<T, VEC>(yr + idx * VEC, o);
                }
            }
        } else {
            for (int idx = tid; idx < nvec; idx += nt) {
                float xv[VEC];
                load_vec<T, VEC>(xv, xr + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) s[0] += xv[e];
            }
            block_sum<1>(s, red);
            const float mu = s[0] * inv_emb;
            float v[1] = {0.f};
            for (int idx = tid; idx < nvec; idx += nt) {
                float xv[VEC];
                load_vec<T, VEC>(xv, xr + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) { const float c = xv[e] - mu; v[0] += c * c; }
            }
            block_sum<1>(v, red);
            const float r = 1.0f / sqrtf(v[0] * inv_emb + eps);
            if (tid == 0) { mean_out[row] = mu; rstd_out[row] = r; }
            for (int idx = tid; idx < nvec; idx += nt) {
                float xv[VEC], wv[VEC], bv[VEC], o[VEC];
                load_vec<T, VEC>(xv, xr + idx * VEC);
                load_vec<T, VEC>(wv, w + idx * VEC);
                load_vec<T, VEC>(bv, b + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) o[e] = (xv[e] - mu) * r * wv[e] + bv[e];
                store_vec<T, VEC>(yr + idx * VEC, o);
            }
        }
    }
}

// ---------------------------------------------------------------- LayerNorm bwd
// c1 = mean(w·dy·xn), c2 = mean(w·dy); dx = (w·dy − (xn·c1 + c2))·rstd;
// dw += dy·xn; db += dy      (src/layer_norm.jl:94-137)
template <typename T, int VEC, int NV>
__global__ void __launch_bounds__(kNormBlock)
ln_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ x, const T* __restrict__ w,
              const float* __restrict__ mean, const float* __restrict__ rstd,
              T* __restrict__ dx, float* __restrict__ partial, int emb, int64_t n, float inv_emb) {
    __shared__ float red[64];
    const int nvec = emb / VEC;
    const int tid = threadIdx.x, nt = blockDim.x;
    float* pw = partial + (int64_t)blockIdx.x * 2 * emb;
    float* pb = pw + emb;
    if constexpr (NV > 0) {
        float wv[NV][VEC], dwa[NV][VEC], dba[NV][VEC];
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int idx = tid + i * nt;
#pragma unroll
            for (int e = 0; e < VEC; ++e) { wv[i][e] = 0.f; dwa[i][e] = 0.f; dba[i][e] = 0.f; }
            if (idx < nvec) load_vec<T, VEC>(wv[i], w + idx * VEC);
        }
        // the next row's x and dy are loaded while this row is reduced and written
        Vec<T, VEC> xn_[NV], dn_[NV];
        auto load_row = [&](int64_t row) {
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (row < n && idx < nvec) {
                    xn_[i] = ldg_stream<T, VEC>(x + row * (int64_t)emb + idx * VEC);
                    dn_[i] = ldg_stream<T, VEC>(dy + row * (int64_t)emb + idx * VEC);
                }
            }
        };
        load_row(blockIdx.x);
        for (int64_t row = blockIdx.x; row < n; row += gridDim.x) {
            const float mu = mean[row], r = rstd[row];
            Vec<T, VEC> xc[NV], dc[NV];
#pragma unroll
            for (int i = 0; i < NV; ++i) { xc[i] = xn_[i]; dc[i] = dn_[i]; }
            load_row(row + gridDim.x);
            float c[2] = {0.f, 0.f};
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
#pragma unroll
                    for (int e = 0; e < VEC; ++e) {
                        const float xn = (to_f(xc[i].v[e]) - mu) * r;
                        const float wdy = wv[i][e] * to_f(dc[i].v[e]);
                        c[0] += wdy * xn;
                        c[1] += wdy;
                    }
                }
            }
            block_sum<2>(c, red);
            const float c1 = c[0] * inv_emb, c2 = c[1] * inv_emb;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int idx = tid + i * nt;
                if (idx < nvec) {
                    float o[VEC];
#pragma unroll
                    for (int e = 0; e < VEC; ++e) {
                        const float d = to_f(dc[i].v[e]);
                        const float xn = (to_f(xc[i].v[e]) - mu) * r;
                        const float wdy = wv[i][e] * d;
                        o[e] = (wdy - (xn * c1 + c2)) * r;
                        dwa[i][e] += d * xn;
                        dba[i][e] += d;
                    }
                    store_vec<T, VEC>(dx + row * (int64_t)emb + idx * VEC, o);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int idx = tid + i * nt;
            if (idx < nvec) {
#pragma unroll
                for (int e = 0; e < VEC; ++e) {
                    pw[idx * VEC + e] = dwa[i][e];
                    pb[idx * VEC + e] = dba[i][e];
                }
            }
        }
    } else {
        for (int idx = tid; idx < nvec * VEC; idx += nt) { pw[idx] = 0.f; pb[idx] = 0.f; }
        for (int64_t row = blockIdx.x; row < n; row += gridDim.x) {
            const T* xr = x + row * (int64_t)emb;
            const T* dr = dy + row * (int64_t)emb;
            const float mu = mean[row], r = rstd[row];
            float c[2] = {0.f, 0.f};
            for (int idx = tid; idx < nvec; idx += nt) {
                float xv[VEC], dv[VEC], wl[VEC];
                load_vec<T, VEC>(xv, xr + idx * VEC);
                load_vec<T, VEC>(dv, dr + idx * VEC);
                load_vec<T, VEC>(wl, w + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) {
                    const float xn = (xv[e] - mu) * r;
                    const float wdy = wl[e] * dv[e];
                    c[0] += wdy * xn;
                    c[1] += wdy;
                }
            }
            block_sum<2>(c, red);
            const float c1 = c[0] * inv_emb, c2 = c[1] * inv_emb;
            for (int idx = tid; idx < nvec; idx += nt) {
                float xv[VEC], dv[VEC], wl[VEC], o[VEC];
                load_vec<T, VEC>(xv, xr + idx * VEC);
                load_vec<T, VEC>(dv, dr + idx * VEC);
                load_vec<T, VEC>(wl, w + idx * VEC);
#pragma unroll
                for (int e = 0; e < VEC; ++e) {
                    const float xn = (xv[e] - mu) * r;
                    o[e] = (wl[e] * dv[e] - (xn * c1 + c2)) * r;
                    pw[idx * VEC + e] += dv[e] * xn;
                    pb[idx * VEC + e] += dv[e];
                }
                store_vec<T, VEC>(dx + row * (int64_t)emb + idx * VEC, o);
            }
        }
    }
}

// Column sums of `nparts` fp32 partial rows, each `stride` floats apart; one
// thread per column, fixed summation order (deterministic).
template <typename TO>
__global__ void reduce_partials_kernel(const float* __restrict__ partial, TO* __restrict__ out,
                                       int emb, int64_t stride, int nparts) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= emb) return;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    int g = 0;
    for (; g + 3 < nparts; g += 4) {
        s0 += partial[(int64_t)g * stride + c];
        s1 += partial[(int64_t)(g + 1) * stride + c];
        s2 += partial[(int64_t)(g + 2) * stride + c];
        s3 += partial[(int64_t)(g + 3) * stride + c];
    }
    for (; g < nparts; ++g) s0 += partial[(int64_t)g * stride + c];
    out[c] = from_f<TO>((s0 + s1) + (s2 + s3));
}

// ---------------------------------------------------------------- dispatch
// Picks the 16-byte vector path when every row starts 16-byte aligned, and the
// number of cached vectors per thread from the row length.  `max_elems`
// bounds the elements a thread caches: the backward kernels also keep per-thread
// dw/db accumulators for their columns, and beyond 32 elements those spill, so
// longer rows take the uncached path (x, dy re-read, mostly from L2).
struct RowPlan {
    bool vec;
    int block;
    int nv;  // 0 = uncached
};

template <typename T>
RowPlan plan_rows(int emb, std::initializer_list<const void*> ptrs, int max_elems = 1 << 30) {
    constexpr int V = 16 / sizeof(T);
    bool vec = (emb % V == 0);
    for (const void* p : ptrs) vec = vec && (p == nullptr || aligned16(p));
    const int nvec = vec ? emb / V : emb;
    int block = ((nvec + 31) / 32) * 32;
    if (block > kNormBlock) block = kNormBlock;
    if (block < 32) block = 32;
    const int per = (nvec + block - 1) / block;
    int nv = 1;
    while (nv < per) nv *= 2;
    if (nv > kMaxNV || nv * (vec ? V : 1) > max_elems) nv = 0;
    return {vec, block, nv};
}

#define NNOP_NV_SWITCH(nv, NVC, ...)                         \
    switch (nv) {                                            \
        case 1: { constexpr int NVC = 1; __VA_ARGS__; } break;   \
        case 2: { constexpr int NVC = 2; __VA_ARGS__; } break;   \
        case 4: { constexpr int NVC = 4; __VA_ARGS__; } break;   \
        case 8: { constexpr int NVC = 8; __VA_ARGS__; } break;   \
        case 16: { constexpr int NVC = 16; __VA_ARGS__; } break; \
        default: { constexpr int NVC = 0; __VA_ARGS__; } break;  \
    }

#define NNOP_VEC_SWITCH(vec, T, VC, ...)                                      \
    if (vec) { constexpr int VC = 16 / sizeof(T); __VA_ARGS__; }             \
    else { constexpr int VC = 1; __VA_ARGS__; }

int64_t rows_grid(int64_t n) { return n < (int64_t)1 << 30 ? n : (int64_t)1 << 30; }

// Persistent backward grid: at most kBwdBlocksPerSm CTAs per SM; the workspace
// is sized for that bound so its size does not depend on occupancy.
constexpr int kBwdBlocksPerSm = 8;

template <typename KernelT>
int bwd_grid(KernelT kernel, int block, int64_t n) {
    int occ = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, block, 0) != cudaSuccess || occ < 1) occ = 1;
    if (occ > kBwdBlocksPerSm) occ = kBwdBlocksPerSm;
    int64_t g = (int64_t)num_sms() * occ;
    if (g > n) g = n;
    if (g < 1) g = 1;
    return (int)g;
}

// Grid of the prefetching forward: persistent CTAs (SM count × resident CTAs)
// walking rows with a one-row prefetch; one CTA per row without register
// caching.  (16-bit rows only: for fp32 rows the one-row-per-CTA kernels are
// faster, measured.)
template <typename KernelT>
int64_t fwd_grid(KernelT kernel, int block, int nv, int64_t n) {
    if (nv == 0) return rows_grid(n);
    int occ = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, block, 0) != cudaSuccess || occ < 1) occ = 1;
    const int64_t g = (int64_t)num_sms() * occ;
    return g < n ? g : n;
}

// Forward launches: the prefetching persistent kernels for 16-bit rows, the
// one-row-per-CTA kernels for fp32 rows (measured faster there).
template <typename T, int VC, int NVC>
void launch_rms_fwd(const T* x, const T* w, T* y, float* rstd, int emb, int64_t n, float eps, float offset,
                    int block, cudaStream_t s) {
    if constexpr (sizeof(T) <= 2) {
        auto kern = rms_fwd_kernel<T, VC, NVC>;
        kern<<<(unsigned)fwd_grid(kern, block, NVC, n), block, 0, s>>>(x, w, y, rstd, emb, n, eps, offset,
                                                                        1.0f / (float)emb);
    } else {
        rms_fwd_rowwise_kernel<T, VC, NVC><<<(unsigned)rows_grid(n), block, 0, s>>>(x, w, y, rstd, emb, n, eps,
                                                                                     offset, 1.0f / (float)emb);
    }
}

template <typename T, int VC, int NVC>
void launch_ln_fwd(const T* x, const T* w, const T* b, T* y, float* mean, float* rstd, int emb, int64_t n,
                   float eps, int block, cudaStream_t s) {
    if constexpr (sizeof(T) <= 2) {
        auto kern = ln_fwd_kernel<T, VC, NVC>;
        kern<<<(unsigned)fwd_grid(kern, block, NVC, n), block, 0, s>>>(x, w, b, y, mean, rstd, emb, n, eps,
                                                                        1.0f / (float)emb);
    } else {
        ln_fwd_rowwise_kernel<T, VC, NVC><<<(unsigned)rows_grid(n), block, 0, s>>>(x, w, b, y, mean, rstd, emb, n,
                                                                                    eps, 1.0f / (float)emb);
    }
}

int64_t bwd_max_parts(int64_t n) {
    int64_t g = (int64_t)num_sms() * kBwdBlocksPerSm;
    return g < n ? g : (n < 1 ? 1 : n);
}

int check_norm_args(int64_t emb, int64_t n) {
    if (emb <= 0 || n < 0) return fail(NNOP_ERR_SHAPE, "norm: emb must be > 0 and n >= 0");
    if (emb > (int64_t)1 << 24) return fail(NNOP_ERR_SHAPE, "norm: emb too large (max 2^24)");
    return NNOP_OK;
}

}  // namespace

// The shared-memory ring kernels (norm_ring.cu): launched when they apply.
namespace ring {
template <typename T>
bool rms_fwd(const T* x, const T* w, T* y, float* rstd, int emb, int64_t n, float eps, float offset, cudaStream_t s,
             int* st);
template <typename T>
bool rms_bwd(const T* dy, const T* x, const T* w, const float* rstd, T* dx, float* partial, int emb, int64_t n,
             float offset, int max_parts, cudaStream_t s, int* parts, int* st);
template <typename T>
bool ln_fwd(const T* x, const T* w, const T* b, T* y, float* mean, float* rstd, int emb, int64_t n, float eps,
            cudaStream_t s, int* st);
template <typename T>
bool ln_bwd(const T* dy, const T* x, const T* w, const float* mean, const float* rstd, T* dx, float* partial,
            int emb, int64_t n, int max_parts, cudaStream_t s, int* parts, int* st);
template <typename T>
bool add_rms_fwd(const T* x, const T* res, const T* w, T* h, T* y, float* rstd, int emb, int64_t n, float eps,
                 float offset, cudaStream_t s, int* st);
template <typename T>
bool rms_bwd_add(const T* dy, const T* dh, const T* x, const T* w, const float* rstd, T* dx, float* partial, int emb,
                 int64_t n, float offset, int max_parts, cudaStream_t s, int* parts, int* st);
}  // namespace ring

namespace {
// out = a + b elementwise, rounded to T (the fused entry points' fallback for
// rows the ring kernels do not take)
template <typename T>
__global__ void add_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ out, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = from_f<T>(to_f(a[i]) + to_f(b[i]));
}
template <typename T>
int launch_add(const T* a, const T* b, T* out, int64_t n, cudaStream_t s) {
    if (n == 0) return NNOP_OK;
    const int64_t g = (n + 255) / 256;
    add_kernel<T><<<(unsigned)(g < 65536 ? g : 65536), 256, 0, s>>>(a, b, out, n);
    return check_launch("residual add");
}
}  // namespace
}  // namespace nnop

using namespace nnop;

extern "C" {

int nnop_rms_norm_fwd(const void* x, const void* w, void* y, float* rstd, int64_t emb, int64_t n,
                      float eps, float offset, int dtype, void* stream) {
    int st = check_norm_args(emb, n);
    if (st) return st;
    if (n == 0) return NNOP_OK;
    if (!x || !w || !y || !rstd) return fail(NNOP_ERR_ARG, "rms_norm_fwd: NULL pointer");
    cudaStream_t s = (cudaStream_t)stream;
    NNOP_DISPATCH_DTYPE(dtype, T, {
        int rst = NNOP_OK;
        if (ring::rms_fwd<T>((const T*)x, (const T*)w, (T*)y, rstd, (int)emb, n, eps, offset, s, &rst)) return rst;
        RowPlan p = plan_rows<T>((int)emb, {x, w, y});
        NNOP_VEC_SWITCH(p.vec, T, VC, {
            NNOP_NV_SWITCH(p.nv, NVC, {
                launch_rms_fwd<T, VC, NVC>((const T*)x, (const T*)w, (T*)y, rstd, (int)emb, n, eps, offset,
                                           p.block, s);
            });
        });
    });
    return check_launch("rms_norm_fwd");
}

size_t nnop_rms_norm_bwd_workspace_size(int64_t emb, int64_t n) {
    return (size_t)bwd_max_parts(n) * (size_t)emb * sizeof(float);
}

int nnop_rms_norm_bwd(const void* dy, const void* x, const void* w, const float* rstd, void* dx,
                      float* dw, void* workspace, size_t workspace_bytes, int64_t emb, int64_t n,
                      float offset, int dtype, void* stream) {
    int st = check_norm_args(emb, n);
    if (st) return st;
    if (!dy || !x || !w || !rstd || !dx || !dw) return fail(NNOP_ERR_ARG, "rms_norm_bwd: NULL pointer");
    cudaStream_t s = (cudaStream_t)stream;
    if (n == 0) {
        if (cudaMemsetAsync(dw, 0, emb * sizeof(float), s) != cudaSuccess)
            return fail(NNOP_ERR_CUDA, "rms_norm_bwd: memset failed");
        return NNOP_OK;
    }
    if (!workspace || workspace_bytes < nnop_rms_norm_bwd_workspace_size(emb, n))
        return fail(NNOP_ERR_WORKSPACE, "rms_norm_bwd: workspace too small");
    float* partial = (float*)workspace;
    int parts = 0;
    NNOP_DISPATCH_DTYPE(dtype, T, {
        if (!ring::rms_bwd<T>((const T*)dy, (const T*)x, (const T*)w, rstd, (T*)dx, partial, (int)emb, n, offset,
                              (int)bwd_max_parts(n), s, &parts, &st)) {
            RowPlan p = plan_rows<T>((int)emb, {dy, x, w, dx}, 32);
            NNOP_VEC_SWITCH(p.vec, T, VC, {
                NNOP_NV_SWITCH(p.nv, NVC, {
                    auto kern = rms_bwd_kernel<T, VC, NVC>;
                    parts = bwd_grid(kern, p.block, n);
                    kern<<<parts, p.block, 0, s>>>((const T*)dy, (const T*)x, (const T*)w, rstd, (T*)dx,
                                                    partial, (int)emb, n, offset, 1.0f / (float)emb);
                });
            });
            st = check_launch("rms_norm_bwd");
        }
    });
    if (st) return st;
    reduce_partials_kernel<float><<<(unsigned)((emb + 255) / 256), 256, 0, s>>>(partial, dw, (int)emb, emb, parts);
    return check_launch("rms_norm_bwd reduce");
}

int nnop_layer_norm_fwd(const void* x, const void* w, const void* b, void* y, float* mean, float* rstd,
                        int64_t emb, int64_t n, float eps, int dtype, void* stream) {
    int st = check_norm_args(emb, n);
    if (st) return st;
    if (n == 0) return NNOP_OK;
    if (!x || !w || !b || !y || !mean || !rstd) return fail(NNOP_ERR_ARG, "layer_norm_fwd: NULL pointer");
    cudaStream_t s = (cudaStream_t)stream;
    NNOP_DISPATCH_DTYPE(dtype, T, {
        int rst = NNOP_OK;
        if (ring::ln_fwd<T>((const T*)x, (const T*)w, (const T*)b, (T*)y, mean, rstd, (int)emb, n, eps, s, &rst))
            return rst;
        RowPlan p = plan_rows<T>((int)emb, {x, w, b, y});
        NNOP_VEC_SWITCH(p.vec, T, VC, {
            NNOP_NV_SWITCH(p.nv, NVC, {
                launch_ln_fwd<T, VC, NVC>((const T*)x, (const T*)w, (const T*)b, (T*)y, mean, rstd, (int)emb, n,
                                          eps, p.block, s);
            });
        });
    });
    return check_launch("layer_norm_fwd");
}

size_t nnop_layer_norm_bwd_workspace_size(int64_t emb, int64_t n) {
    return (size_t)bwd_max_parts(n) * 2 * (size_t)emb * sizeof(float);
}

int nnop_layer_norm_bwd(const void* dy, const void* x, const void* w, const float* mean,
                        const float* rstd, void* dx, void* dw, void* db, void* workspace,
                        size_t workspace_bytes, int64_t emb, int64_t n, int dtype, void* stream) {
    int st = check_norm_args(emb, n);
    if (st) return st;
    if (!dy || !x || !w || !mean || !rstd || !dx || !dw || !db)
        return fail(NNOP_ERR_ARG, "layer_norm_bwd: NULL pointer");
    cudaStream_t s = (cudaStream_t)stream;
    if (n == 0) {
        NNOP_DISPATCH_DTYPE(dtype, T, {
            if (cudaMemsetAsync(dw, 0, emb * sizeof(T), s) != cudaSuccess ||
                cudaMemsetAsync(db, 0, emb * sizeof(T), s) != cudaSuccess)
                return fail(NNOP_ERR_CUDA, "layer_norm_bwd: memset failed");
        });
        return NNOP_OK;
    }
    if (!workspace || workspace_bytes < nnop_layer_norm_bwd_workspace_size(emb, n))
        return fail(NNOP_ERR_WORKSPACE, "layer_norm_bwd: workspace too small");
    float* partial = (float*)workspace;
    int parts = 0;
    NNOP_DISPATCH_DTYPE(dtype, T, {
        if (!ring::ln_bwd<T>((const T*)dy, (const T*)x, (const T*)w, mean, rstd, (T*)dx, partial, (int)emb, n,
                             (int)bwd_max_parts(n), s, &parts, &st)) {
            RowPlan p = plan_rows<T>((int)emb, {dy, x, w, dx}, 32);
            NNOP_VEC_SWITCH(p.vec, T, VC, {
                NNOP_NV_SWITCH(p.nv, NVC, {
                    auto kern = ln_bwd_kernel<T, VC, NVC>;
                    parts = bwd_grid(kern, p.block, n);
                    kern<<<parts, p.block, 0, s>>>((const T*)dy, (const T*)x, (const T*)w, mean, rstd,
                                                    (T*)dx, partial, (int)emb, n, 1.0f / (float)emb);
                });
            });
            st = check_launch("layer_norm_bwd");
        }
        if (st) return st;
        const unsigned g = (unsigned)((emb + 255) / 256);
        reduce_partials_kernel<T><<<g, 256, 0, s>>>(partial, (T*)dw, (int)emb, 2 * emb, parts);
        reduce_partials_kernel<T><<<g, 256, 0, s>>>(partial + emb, (T*)db, (int)emb, 2 * emb, parts);
    });
    return check_launch("layer_norm_bwd reduce");
}

// ---------------------------------------------------------------------------
// Residual add fused into RMSNorm (no counterpart in the reference's API; the
// composition of a transformer block's residual add with `rms_norm`,
// src/rms_norm.jl:117-169).
// ---------------------------------------------------------------------------

int nnop_add_rms_norm_fwd(const void* x, const void* residual, const void* w, void* h, void* y, float* rstd,
                          int64_t emb, int64_t n, float eps, float offset, int dtype, void* stream) {
    int st = check_norm_args(emb, n);
    if (st) return st;
    if (n == 0) return NNOP_OK;
    if (!x || !residual || !w || !h || !y || !rstd) return fail(NNOP_ERR_ARG, "add_rms_norm_fwd: NULL pointer");
    cudaStream_t s = (cudaStream_t)stream;
    NNOP_DISPATCH_DTYPE(dtype, T, {
        int rst = NNOP_OK;
        if (ring::add_rms_fwd<T>((const T*)x, (const T*)residual, (const T*)w, (T*)h, (T*)y, rstd, (int)emb, n, eps,
                                 offset, s, &rst))
            return rst;
        if ((st = launch_add<T>((const T*)x, (const T*)residual, (T*)h, emb * n, s))) return st;
    });
    return nnop_rms_norm_fwd(h, w, y, rstd, emb, n, eps, offset, dtype, stream);
}

size_t nnop_add_rms_norm_bwd_workspace_size(int64_t emb, int64_t n) { return nnop_rms_norm_bwd_workspace_size(emb, n); }

int nnop_add_rms_norm_bwd(const void* dy, const void* dh, const void* h, const void* w, const float* rstd, void* dx,
                          float* dw, void* workspace, size_t workspace_bytes, int64_t emb, int64_t n, float offset,
                          int dtype, void* stream) {
    if (dh == nullptr)
        return nnop_rms_norm_bwd(dy, h, w, rstd, dx, dw, workspace, workspace_bytes, emb, n, offset, dtype, stream);
    int st = check_norm_args(emb, n);
    if (st) return st;
    if (!dy || !h || !w || !rstd || !dx || !dw) return fail(NNOP_ERR_ARG, "add_rms_norm_bwd: NULL pointer");
    cudaStream_t s = (cudaStream_t)stream;
    if (n == 0) {
        if (cudaMemsetAsync(dw, 0, emb * sizeof(float), s) != cudaSuccess)
            return fail(NNOP_ERR_CUDA, "add_rms_norm_bwd: memset failed");
        return NNOP_OK;
    }
    if (!workspace || workspace_bytes < nnop_rms_norm_bwd_workspace_size(emb, n))
        return fail(NNOP_ERR_WORKSPACE, "add_rms_norm_bwd: workspace too small");
    float* partial = (float*)workspace;
    int parts = 0;
    bool fused = false;
    NNOP_DISPATCH_DTYPE(dtype, T, {
        fused = ring::rms_bwd_add<T>((const T*)dy, (const T*)dh, (const T*)h, (const T*)w, rstd, (T*)dx, partial,
                                     (int)emb, n, offset, (int)bwd_max_parts(n), s, &parts, &st);
    });
    if (!fused) {
        st = nnop_rms_norm_bwd(dy, h, w, rstd, dx, dw, workspace, workspace_bytes, emb, n, offset, dtype, stream);
        if (st) return st;
        NNOP_DISPATCH_DTYPE(dtype, T, { return launch_add<T>((const T*)dx, (const T*)dh, (T*)dx, emb * n, s); });
    }
    if (st) return st;
    reduce_partials_kernel<float><<<(unsigned)((emb + 255) / 256), 256, 0, s>>>(partial, dw, (int)emb, emb, parts);
    return check_launch("add_rms_norm_bwd reduce");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// RMSNorm backward without any allocation.
//
// Some callers cannot allocate device memory at the moment they need the
// gradient: code that runs inside a memory pool's own callbacks, runtimes that
// plan every byte of device memory ahead of time, or embedded hosts whose
// allocator is not reachable from the call site.  They cannot provide the
// workspace that nnop_rms_norm_bwd needs, so this variant keeps its scratch
// (the per-CTA fp32 dw partial rows) in a fixed-size array that lives in the
// library itself.  The array occupies kNoAllocScratchBytes on every GPU that
// loads the library, for the life of the process.
// ---------------------------------------------------------------------------
namespace nnop {
namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;   // 8 MiB: 2^21 fp32 partials
constexpr int64_t kNoAllocScratchFloats = (int64_t)(kNoAllocScratchBytes / sizeof(float));
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// The current context of the calling thread (driver call reached through the
// runtime's entry-point query, so the library needs no libcuda link).
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
CUcontext current_context() {
    static CtxGetCurrentFn fn = [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (CtxGetCurrentFn) nullptr;
        return reinterpret_cast<CtxGetCurrentFn>(ptr);
    }();
    CUcontext c = nullptr;
    if (fn == nullptr || fn(&c) != CUDA_SUCCESS) return nullptr;
    return c;
}

// Device address of g_noalloc_scratch for the current device, looked up once
// per device and context (the host-side symbol is only a stand-in, never a
// device pointer).  A device reset gives the device a new primary context, in
// which the module -- and the array -- is loaded again at another address;
// the context recorded beside each cached address makes the next call look
// the address up again instead of writing through the stale one.
int noalloc_scratch(float** out) {
    static std::mutex mu;
    static float* addr[64] = {nullptr};
    static CUcontext ctx[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return fail(NNOP_ERR_CUDA, "rms_norm_bwd_noalloc: no current CUDA device");
    std::lock_guard<std::mutex> lock(mu);
    const CUcontext cur = current_context();
    if (addr[dev] == nullptr || cur == nullptr || cur != ctx[dev]) {
        // the lookup also makes the device's primary context current
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr)
            return fail(NNOP_ERR_CUDA, std::string("rms_norm_bwd_noalloc: cudaGetSymbolAddress failed: ") +
                                           cudaGetErrorString(e));
        addr[dev] = static_cast<float*>(p);
        ctx[dev] = current_context();
    }
    *out = addr[dev];
    return NNOP_OK;
}

}  // namespace
}  // namespace nnop

extern "C" {

int nnop_rms_norm_bwd_noalloc(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw,
                              int64_t emb, int64_t n, float offset, int dtype, void* stream) {
    int st = check_norm_args(emb, n);
    if (st) return st;
    if (emb > kNoAllocScratchFloats)
        return fail(NNOP_ERR_SHAPE, "rms_norm_bwd_noalloc: emb " + std::to_string(emb) + " exceeds the maximum " +
                                        std::to_string(kNoAllocScratchFloats) + " of the built-in scratch");
    if (!dy || !x || !w || !rstd || !dx || !dw) return fail(NNOP_ERR_ARG, "rms_norm_bwd_noalloc: NULL pointer");
    cudaStream_t s = (cudaStream_t)stream;
    if (n == 0) {
        if (cudaMemsetAsync(dw, 0, emb * sizeof(float), s) != cudaSuccess)
            return fail(NNOP_ERR_CUDA, "rms_norm_bwd_noalloc: memset failed");
        return NNOP_OK;
    }
    float* partial = nullptr;
    st = noalloc_scratch(&partial);
    if (st) return st;
    // Every partial row the reduction reads is fully written by its CTA first,
    // so the scratch left over from an earlier call needs no clearing.
    const int64_t max_parts = kNoAllocScratchFloats / emb;
    int parts = 0;
    NNOP_DISPATCH_DTYPE(dtype, T, {
        RowPlan p = plan_rows<T>((int)emb, {dy, x, w, dx}, 32);
        NNOP_VEC_SWITCH(p.vec, T, VC, {
            NNOP_NV_SWITCH(p.nv, NVC, {
                auto kern = rms_bwd_kernel<T, VC, NVC>;
                parts = bwd_grid(kern, p.block, n);
                if (parts > max_parts) parts = (int)max_parts;
                kern<<<parts, p.block, 0, s>>>((const T*)dy, (const T*)x, (const T*)w, rstd, (T*)dx, partial,
                                                (int)emb, n, offset, 1.0f / (float)emb);
            });
        });
    });
    st = check_launch("rms_norm_bwd_noalloc");
    if (st) return st;
    reduce_partials_kernel<float><<<(unsigned)((emb + 255) / 256), 256, 0, s>>>(partial, dw, (int)emb, emb, parts);
    return check_launch("rms_norm_bwd_noalloc reduce");
}

}  // extern "C"
