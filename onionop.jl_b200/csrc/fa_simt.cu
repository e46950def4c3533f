// Flash attention forward/backward in full fp32 on the CUDA cores.
//
// The reference runs fp32 attention through its SIMT register-tiled GEMM
// (`mma!`, src/mma.jl:6-48) and keeps the backward's Q/K tiles in Float16 even
// for fp32 inputs (src/attention_bwd.jl:20-21).  Tensor-core TF32 would lose
// the same precision, so this path multiplies in fp32 FMA throughout; it is the
// path of the fp32 parity configuration (E=64, L=512), not of the bf16/f16
// throughput configurations.
//
// Tiles: 32 queries x 32 keys, 128 threads; thread (r = tid/4, c = tid%4) owns
// row r and columns c, c+4, ..., c+28 of the score tile and embedding columns
// c, c+4, ... of its output row.
#include "fa_common.cuh"

namespace nnop {
namespace fa {
namespace {

constexpr int kT = 128;
constexpr int kB = 32;   // query tile = key tile

template <int E>
__device__ __forceinline__ void load_rows_f32(float* s, int ld, const float* g, int64_t row0, int64_t nrows) {
    for (int x = threadIdx.x; x < kB * E; x += kT) {
        const int r = x / E, e = x % E;
        const int64_t gr = row0 + r;
        s[r * ld + e] = gr < nrows ? g[gr * E + e] : 0.f;
    }
}

template <int E, bool CAUSAL>
__global__ void __launch_bounds__(kT) fa_fwd_f32_kernel(const Params p) {
    constexpr int LD = E + 1;
    constexpr int EW = E / 4;
    extern __shared__ float smem_f[];
    float* sQ = smem_f;              // [kB][LD]
    float* sK = sQ + kB * LD;        // [kB][LD]
    float* sV = sK + kB * LD;        // [kB][E]
    float* sP = sV + kB * E;         // [kB][kB+1]

    const int64_t QL = p.QL, KL = p.KL;
    const int n_qt = (int)((QL + kB - 1) / kB);
    const int qt = CAUSAL ? n_qt - 1 - (int)blockIdx.x : (int)blockIdx.x;
    const int h = blockIdx.y, b = blockIdx.z, kvh = h / p.n_rep;
    const int r = threadIdx.x >> 2, cg = threadIdx.x & 3;
    const int64_t q0 = (int64_t)qt * kB;
    const int64_t i = q0 + r;

    const float* qg = reinterpret_cast<const float*>(p.q) + ((int64_t)b * p.QH + h) * QL * E;
    const float* kg = reinterpret_cast<const float*>(p.k) + ((int64_t)b * p.KH + kvh) * KL * E;
    const float* vg = reinterpret_cast<const float*>(p.v) + ((int64_t)b * p.KH + kvh) * KL * E;
    const float* pg = p.pair ? reinterpret_cast<const float*>(p.pair) + (int64_t)b * KL * QL * p.QH + h : nullptr;
    const uint8_t* mg = p.kmask ? p.kmask + (int64_t)b * KL : nullptr;

    int64_t kv_len = KL;
    if (mg) kv_len = kv_valid_len_block(mg, KL);
    int n_kt = (int)((kv_len + kB - 1) / kB);
    if (CAUSAL) {
        const int64_t i_end = q0 + kB < QL ? q0 + kB : QL;
        const int lim = (int)((i_end + kB - 1) / kB);
        n_kt = n_kt < lim ? n_kt : lim;
    }

    load_rows_f32<E>(sQ, LD, qg, q0, QL);
    float o[EW];
#pragma unroll
    for (int w = 0; w < EW; ++w) o[w] = 0.f;
    float m = -INFINITY, l = 0.f;

    for (int kt = 0; kt < n_kt; ++kt) {
        const int64_t k0 = (int64_t)kt * kB;
        __syncthreads();
        load_rows_f32<E>(sK, LD, kg, k0, KL);
        load_rows_f32<E>(sV, E, vg, k0, KL);
        __syncthreads();
        float s[8];
        float mx = -INFINITY;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int c = cg + 4 * u;
            float acc = 0.f;
#pragma unroll 16
            for (int e = 0; e < E; ++e) acc = fmaf(sQ[r * LD + e], sK[c * LD + e], acc);
            const int64_t j = k0 + c;
            float x = acc * p.scale;
            if (pg && i < QL && j < KL) x += pg[(j * QL + i) * p.QH];
            bool valid = j < KL;
            if (CAUSAL) valid = valid && j <= i;
            if (mg) valid = valid && (j < KL ? mg[j] != 0 : false);
            s[u] = valid ? x : -INFINITY;
            mx = fmaxf(mx, s[u]);
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m, mx);
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const float alpha = expf(m - m_use);
        m = m_new;
        float ls = 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const float pe = expf(s[u] - m_use);
            ls += pe;
            sP[r * (kB + 1) + cg + 4 * u] = pe;
        }
        l = l * alpha + ls;
        __syncthreads();
#pragma unroll
        for (int w = 0; w < EW; ++w) {
            float acc = o[w] * alpha;
            const int e = cg + 4 * w;
#pragma unroll 8
            for (int c = 0; c < kB; ++c) acc = fmaf(sP[r * (kB + 1) + c], sV[c * E + e], acc);
            o[w] = acc;
        }
    }
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (i < QL) {
        const float inv = 1.0f / l;
        float* og = reinterpret_cast<float*>(p.o) + ((int64_t)b * p.QH + h) * QL * E + i * E;
#pragma unroll
        for (int w = 0; w < EW; ++w) og[cg + 4 * w] = o[w] * inv;
        if (cg == 0) p.lse[((int64_t)b * p.QH + h) * QL + i] = m + logf(l);
    }
}

template <int E, bool CAUSAL>
__global__ void __launch_bounds__(kT) fa_bwd_f32_kernel(const Params p) {
    constexpr int LD = E + 1;
    constexpr int EW = E / 4;
    constexpr int LP = kB + 1;
    extern __shared__ float smem_f[];
    float* sK = smem_f;              // [kB][LD]
    float* sV = sK + kB * LD;        // [kB][LD]
    float* sQ = sV + kB * LD;        // [kB][LD]
    float* sdO = sQ + kB * LD;       // [kB][LD]
    float* sP = sdO + kB * LD;       // [kB][LP]
    float* sdS = sP + kB * LP;       // [kB][LP]
    float* sLse = sdS + kB * LP;     // [kB]
    float* sDel = sLse + kB;         // [kB]

    const int64_t QL = p.QL, KL = p.KL;
    const int kt = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int QH = p.QH;
    const int r = threadIdx.x >> 2, cg = threadIdx.x & 3;
    const int64_t k0 = (int64_t)kt * kB;
    const int64_t j = k0 + r;

    const float* kg = reinterpret_cast<const float*>(p.k) + ((int64_t)b * p.KH + kvh) * KL * E;
    const float* vg = reinterpret_cast<const float*>(p.v) + ((int64_t)b * p.KH + kvh) * KL * E;
    const uint8_t* mg = p.kmask ? p.kmask + (int64_t)b * KL : nullptr;
    const int64_t kv_len = p.kv_len ? p.kv_len[b] : KL;
    const int n_qt = (int)((QL + kB - 1) / kB);
    const int qt0 = CAUSAL ? (int)(k0 / kB) : 0;
    const int nq = (k0 < kv_len && qt0 < n_qt) ? n_qt - qt0 : 0;
    const int steps = nq * p.n_rep;

    bool jok = j < KL;
    if (mg) jok = jok && mg[jok ? j : 0] != 0;

    load_rows_f32<E>(sK, LD, kg, k0, KL);
    load_rows_f32<E>(sV, LD, vg, k0, KL);
    float dk[EW], dv[EW];
#pragma unroll
    for (int w = 0; w < EW; ++w) { dk[w] = 0.f; dv[w] = 0.f; }

    for (int step = 0; step < steps; ++step) {
        const int hh = step / nq, qt = qt0 + step % nq;
        const int h = kvh * p.n_rep + hh;
        const int64_t q0 = (int64_t)qt * kB;
        const float* qg = reinterpret_cast<const float*>(p.q) + ((int64_t)b * QH + h) * QL * E;
        const float* dg = reinterpret_cast<const float*>(p.dO) + ((int64_t)b * QH + h) * QL * E;
        const float* pg = p.pair ? reinterpret_cast<const float*>(p.pair) + (int64_t)b * KL * QL * QH + h : nullptr;
        float* dpg = p.dpair ? reinterpret_cast<float*>(p.dpair) + (int64_t)b * KL * QL * QH + h : nullptr;
        __syncthreads();
        load_rows_f32<E>(sQ, LD, qg, q0, QL);
        load_rows_f32<E>(sdO, LD, dg, q0, QL);
        if (threadIdx.x < kB) {
            const int64_t ii = q0 + threadIdx.x;
            const int64_t ro = ((int64_t)b * QH + h) * QL;
            sLse[threadIdx.x] = ii < QL ? p.lse[ro + ii] : 0.f;
            sDel[threadIdx.x] = ii < QL ? p.delta[ro + ii] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int c = cg + 4 * u;
            const int64_t i = q0 + c;
            float s = 0.f, dp = 0.f;
#pragma unroll 16
            for (int e = 0; e < E; ++e) {
                s = fmaf(sK[r * LD + e], sQ[c * LD + e], s);
                dp = fmaf(sV[r * LD + e], sdO[c * LD + e], dp);
            }
            bool valid = jok && i < QL;
            if (CAUSAL) valid = valid && j <= i;
            float x = s * p.scale;
            if (pg && i < QL && j < KL) x += pg[(j * QL + i) * QH];
            const float pr = valid ? expf(x - sLse[c]) : 0.f;
            const float d = pr * (dp - sDel[c]);
            sP[r * LP + c] = pr;
            sdS[r * LP + c] = d;
            if (dpg && i < QL && j < KL) dpg[(j * QL + i) * QH] = d;
        }
        __syncthreads();
#pragma unroll
        for (int w = 0; w < EW; ++w) {
            const int e = cg + 4 * w;
            float av = dv[w], ak = dk[w];
#pragma unroll 8
            for (int c = 0; c < kB; ++c) {
                av = fmaf(sP[r * LP + c], sdO[c * LD + e], av);
                ak = fmaf(sdS[r * LP + c], sQ[c * LD + e], ak);
            }
            dv[w] = av;
            dk[w] = ak;
        }
        // dQ for query row r of this tile: Σ_j dS[j][r] K[j][e]
        const int64_t iq = q0 + r;
        if (iq < QL) {
            float* dqg = p.dq_acc + (((int64_t)b * QH + h) * QL + iq) * E;
#pragma unroll
            for (int w = 0; w < EW; ++w) {
                const int e = cg + 4 * w;
                float acc = 0.f;
#pragma unroll 8
                for (int c = 0; c < kB; ++c) acc = fmaf(sdS[c * LP + r], sK[c * LD + e], acc);
                atomicAdd(dqg + e, acc * p.scale);
            }
        }
    }
    if (j < KL) {
        float* dkg = reinterpret_cast<float*>(p.dk) + (((int64_t)b * p.KH + kvh) * KL + j) * E;
        float* dvg = reinterpret_cast<float*>(p.dv) + (((int64_t)b * p.KH + kvh) * KL + j) * E;
#pragma unroll
        for (int w = 0; w < EW; ++w) {
            dkg[cg + 4 * w] = dk[w] * p.scale;
            dvg[cg + 4 * w] = dv[w];
        }
    }
}

template <int E, bool CAUSAL>
int launch(const Params& p, cudaStream_t s, bool bwd) {
    constexpr int LD = E + 1;
    if (bwd) {
        const size_t smem = (size_t)(4 * kB * LD + 2 * kB * (kB + 1) + 2 * kB) * sizeof(float);
        auto kern = fa_bwd_f32_kernel<E, CAUSAL>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return fail(NNOP_ERR_CUDA, "flash_attention_bwd (f32): cannot set shared memory size");
        dim3 grid((unsigned)((p.KL + kB - 1) / kB), p.KH, p.B);
        kern<<<grid, kT, smem, s>>>(p);
        return check_launch("flash_attention_bwd (f32)");
    }
    const size_t smem = (size_t)(2 * kB * LD + kB * E + kB * (kB + 1)) * sizeof(float);
    auto kern = fa_fwd_f32_kernel<E, CAUSAL>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return fail(NNOP_ERR_CUDA, "flash_attention_fwd (f32): cannot set shared memory size");
    dim3 grid((unsigned)((p.QL + kB - 1) / kB), p.QH, p.B);
    kern<<<grid, kT, smem, s>>>(p);
    return check_launch("flash_attention_fwd (f32)");
}

template <bool CAUSAL>
int dispatch(const Params& p, cudaStream_t s, bool bwd) {
    switch (p.E) {
        case 16: return launch<16, CAUSAL>(p, s, bwd);
        case 32: return launch<32, CAUSAL>(p, s, bwd);
        case 64: return launch<64, CAUSAL>(p, s, bwd);
        case 128: return launch<128, CAUSAL>(p, s, bwd);
        default: return fail(NNOP_ERR_SHAPE, "flash_attention: unsupported embedding dim");
    }
}

}  // namespace

int simt_fwd(const Params& p, bool causal, cudaStream_t s) {
    return causal ? dispatch<true>(p, s, false) : dispatch<false>(p, s, false);
}
int simt_bwd(const Params& p, bool causal, cudaStream_t s) {
    return causal ? dispatch<true>(p, s, true) : dispatch<false>(p, s, true);
}
int simt_tile() { return kB; }

}  // namespace fa
}  // namespace nnop
