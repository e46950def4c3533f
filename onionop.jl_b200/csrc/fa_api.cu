// C-ABI entry points of flash attention: argument checks (the reference's
// `_flash_attention` / `∇flash_attention` error()s, src/attention.jl:185-188 and
// src/attention_bwd.jl:224-227), workspace layout and kernel dispatch.
#include "fa_common.cuh"

#include <cstdlib>

namespace nnop {
namespace fa {
template <typename T> int mma_fwd(const Params& p, bool causal, cudaStream_t s);
template <typename T> int mma_bwd(const Params& p, bool causal, cudaStream_t s);
int mma_tile();
int simt_fwd(const Params& p, bool causal, cudaStream_t s);
int simt_bwd(const Params& p, bool causal, cudaStream_t s);
int simt_tile();
bool sm100_fwd_supported(const Params& p, int dtype);
int sm100_fwd(const Params& p, int dtype, bool causal, cudaStream_t s);
bool sm100_bwd_supported(const Params& p, int dtype);
int sm100_bwd(const Params& p, int dtype, bool causal, cudaStream_t s);
int sm100_bwd_tile();
int sm100_fwd_timeouts();
int sm100_bwd_timeouts();
}  // namespace fa

namespace {

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// NNOP_B200_FA=mma selects the mma.sync kernels for every shape (used by the
// tests to check both kernel families); the default picks the tcgen05 kernels
// where they apply.
bool force_mma() {
    const char* e = getenv("NNOP_B200_FA");
    return e != nullptr && e[0] == 'm';
}

int check_dims(int64_t E, int64_t QL, int64_t KL, int64_t QH, int64_t KH, int64_t B, int dtype) {
    if (dtype != NNOP_F32 && dtype != NNOP_F16 && dtype != NNOP_BF16)
        return fail(NNOP_ERR_DTYPE, "flash_attention: unsupported dtype " + std::to_string(dtype));
    if (E <= 0 || QL < 0 || KL < 0 || QH <= 0 || KH <= 0 || B < 0)
        return fail(NNOP_ERR_SHAPE, "flash_attention: invalid dimensions");
    if ((E & (E - 1)) != 0) return fail(NNOP_ERR_SHAPE, "Only power-of-2 embedding dims are supported.");
    if (QH % KH != 0)
        return fail(NNOP_ERR_SHAPE, "Number of query heads `" + std::to_string(QH) +
                                        "` must be divisible by number of KV heads `" + std::to_string(KH) + "`.");
    if (E < 16 || E > 128)
        return fail(NNOP_ERR_SHAPE, "flash_attention: embedding dim " + std::to_string(E) +
                                        " not supported (16, 32, 64, 128)");
    if (KL == 0 && QL > 0) return fail(NNOP_ERR_SHAPE, "flash_attention: key length must be > 0");
    if (QH > 65535 || B > 65535 || KH > 65535) return fail(NNOP_ERR_SHAPE, "flash_attention: too many heads or batches");
    if (QL > ((int64_t)1 << 31) - 128 || KL > ((int64_t)1 << 31) - 128)
        return fail(NNOP_ERR_SHAPE, "flash_attention: sequence too long");
    return NNOP_OK;
}

struct BwdWorkspace {
    int* kv_len;
    float* delta;
    float* dq_acc;
    size_t bytes;
};

BwdWorkspace bwd_layout(void* base, int64_t E, int64_t QL, int64_t QH, int64_t B, int dtype) {
    BwdWorkspace w{};
    size_t off = 0;
    char* p = static_cast<char*>(base);
    w.kv_len = reinterpret_cast<int*>(p ? p + off : nullptr);
    off += align256((size_t)B * sizeof(int));
    w.delta = reinterpret_cast<float*>(p ? p + off : nullptr);
    off += align256((size_t)B * QH * QL * sizeof(float));
    if (dtype != NNOP_F32) {
        w.dq_acc = reinterpret_cast<float*>(p ? p + off : nullptr);
        off += align256((size_t)B * QH * QL * E * sizeof(float));
    } else {
        w.dq_acc = nullptr;
    }
    w.bytes = off;
    return w;
}

}  // namespace
}  // namespace nnop

using namespace nnop;

extern "C" {

int nnop_device_wait_timeouts(void) {
    const int f = fa::sm100_fwd_timeouts();
    const int b = fa::sm100_bwd_timeouts();
    return (f & 0xffff) | ((b & 0x7fff) << 16);
}

int nnop_flash_attention_fwd(const void* q, const void* k, const void* v, const void* pair,
                             const uint8_t* kpad_mask, void* o, float* lse, int64_t E, int64_t QL, int64_t KL,
                             int64_t QH, int64_t KH, int64_t B, int causal, int dtype, void* stream) {
    int st = check_dims(E, QL, KL, QH, KH, B, dtype);
    if (st) return st;
    if (QL == 0 || B == 0) return NNOP_OK;
    if (!q || !k || !v || !o || !lse) return fail(NNOP_ERR_ARG, "flash_attention_fwd: NULL pointer");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
        return fail(NNOP_ERR_ALIGN, "flash_attention_fwd: q, k, v, o must be 16-byte aligned");
    fa::Params p{};
    p.q = q; p.k = k; p.v = v; p.pair = pair; p.kmask = kpad_mask; p.o = o; p.lse = lse;
    p.QL = QL; p.KL = KL; p.E = (int)E; p.QH = (int)QH; p.KH = (int)KH; p.B = (int)B;
    p.n_rep = (int)(QH / KH);
    cudaStream_t s = (cudaStream_t)stream;
    switch (dtype) {
        case NNOP_F32:
            p.scale = (float)(1.0 / sqrt((double)E));
            return fa::simt_fwd(p, causal != 0, s);
        case NNOP_F16:
            p.scale = __half2float(__float2half_rn((float)(1.0 / sqrt((double)E))));
            if (!force_mma() && fa::sm100_fwd_supported(p, dtype)) return fa::sm100_fwd(p, dtype, causal != 0, s);
            return fa::mma_fwd<__half>(p, causal != 0, s);
        case NNOP_BF16:
            p.scale = __bfloat162float(__float2bfloat16_rn((float)(1.0 / sqrt((double)E))));
            if (!force_mma() && fa::sm100_fwd_supported(p, dtype)) return fa::sm100_fwd(p, dtype, causal != 0, s);
            return fa::mma_fwd<__nv_bfloat16>(p, causal != 0, s);
    }
    return fail(NNOP_ERR_DTYPE, "flash_attention_fwd: unsupported dtype");
}

size_t nnop_flash_attention_bwd_workspace_size(int64_t E, int64_t QL, int64_t KL, int64_t QH, int64_t KH, int64_t B,
                                               int dtype) {
    (void)KL; (void)KH;
    if (E <= 0 || QL < 0 || QH <= 0 || B < 0) return 0;
    return bwd_layout(nullptr, E, QL, QH, B, dtype).bytes;
}

int nnop_flash_attention_bwd(const void* dO, const void* o, const float* lse, const void* q, const void* k,
                             const void* v, const void* pair, const uint8_t* kpad_mask, void* dq, void* dk,
                             void* dv, void* dpair, void* workspace, size_t workspace_bytes, int64_t E, int64_t QL,
                             int64_t KL, int64_t QH, int64_t KH, int64_t B, int causal, int dtype, void* stream) {
    int st = check_dims(E, QL, KL, QH, KH, B, dtype);
    if (st) return st;
    if ((pair == nullptr) != (dpair == nullptr))
        return fail(NNOP_ERR_ARG, "flash_attention_bwd: dpair must be given exactly when pair is given");
    if (QL == 0 || B == 0) {
        // no queries: dk = dv = 0
        if (B > 0 && KL > 0) {
            const size_t esz = dtype == NNOP_F32 ? 4 : 2;
            cudaStream_t s = (cudaStream_t)stream;
            if (cudaMemsetAsync(dk, 0, (size_t)B * KH * KL * E * esz, s) != cudaSuccess ||
                cudaMemsetAsync(dv, 0, (size_t)B * KH * KL * E * esz, s) != cudaSuccess)
                return fail(NNOP_ERR_CUDA, "flash_attention_bwd: memset failed");
        }
        return NNOP_OK;
    }
    if (!dO || !o || !lse || !q || !k || !v || !dq || !dk || !dv)
        return fail(NNOP_ERR_ARG, "flash_attention_bwd: NULL pointer");
    if (!aligned16(dO) || !aligned16(o) || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(dq) ||
        !aligned16(dk) || !aligned16(dv))
        return fail(NNOP_ERR_ALIGN, "flash_attention_bwd: dense tensors must be 16-byte aligned");
    BwdWorkspace ws = bwd_layout(workspace, E, QL, QH, B, dtype);
    if (!workspace || workspace_bytes < ws.bytes)
        return fail(NNOP_ERR_WORKSPACE, "flash_attention_bwd: workspace too small (need " + std::to_string(ws.bytes) +
                                            " bytes)");
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
        return fail(NNOP_ERR_ALIGN, "flash_attention_bwd: workspace must be 256-byte aligned");
    cudaStream_t s = (cudaStream_t)stream;

    fa::Params p{};
    p.q = q; p.k = k; p.v = v; p.pair = pair; p.kmask = kpad_mask; p.o = const_cast<void*>(o);
    p.lse = const_cast<float*>(lse); p.dO = dO; p.delta = ws.delta;
    p.kv_len = kpad_mask ? ws.kv_len : nullptr;
    p.dq = dq; p.dk = dk; p.dv = dv; p.dpair = dpair;
    p.QL = QL; p.KL = KL; p.E = (int)E; p.QH = (int)QH; p.KH = (int)KH; p.B = (int)B;
    p.n_rep = (int)(QH / KH);
    const int64_t rows = B * QH * QL;

    if (kpad_mask) {
        st = fa_host::launch_kv_len(kpad_mask, ws.kv_len, KL, (int)B, s);
        if (st) return st;
    }
    const bool c = causal != 0;
    switch (dtype) {
        case NNOP_F32: {
            p.scale = (float)(1.0 / sqrt((double)E));
            st = fa_host::launch_preprocess<float>((const float*)dO, (const float*)o, ws.delta, rows, (int)E, s);
            if (st) return st;
            if (cudaMemsetAsync(dq, 0, (size_t)rows * E * sizeof(float), s) != cudaSuccess)
                return fail(NNOP_ERR_CUDA, "flash_attention_bwd: memset failed");
            p.dq_acc = (float*)dq;
            st = fa::simt_bwd(p, c, s);
            if (st) return st;
            if (pair) st = fa_host::launch_dpair_fill<float>((float*)dpair, p.kv_len, QL, KL, (int)QH, (int)B,
                                                             fa::simt_tile(), c, s);
            return st;
        }
        case NNOP_F16:
        case NNOP_BF16: {
            if (cudaMemsetAsync(ws.dq_acc, 0, (size_t)rows * E * sizeof(float), s) != cudaSuccess)
                return fail(NNOP_ERR_CUDA, "flash_attention_bwd: memset failed");
            p.dq_acc = ws.dq_acc;
            const bool tc = !force_mma() && fa::sm100_bwd_supported(p, dtype);
            const int tile = tc ? fa::sm100_bwd_tile() : fa::mma_tile();
            if (dtype == NNOP_F16) {
                p.scale = __half2float(__float2half_rn((float)(1.0 / sqrt((double)E))));
                st = fa_host::launch_preprocess<__half>((const __half*)dO, (const __half*)o, ws.delta, rows, (int)E, s);
                if (!st) st = tc ? fa::sm100_bwd(p, dtype, c, s) : fa::mma_bwd<__half>(p, c, s);
                if (!st) st = fa_host::launch_convert<__half>(ws.dq_acc, (__half*)dq, rows * E, s);
                if (!st && pair)
                    st = fa_host::launch_dpair_fill<__half>((__half*)dpair, p.kv_len, QL, KL, (int)QH, (int)B,
                                                            tile, c, s);
            } else {
                p.scale = __bfloat162float(__float2bfloat16_rn((float)(1.0 / sqrt((double)E))));
                st = fa_host::launch_preprocess<__nv_bfloat16>((const __nv_bfloat16*)dO, (const __nv_bfloat16*)o,
                                                               ws.delta, rows, (int)E, s);
                if (!st) st = tc ? fa::sm100_bwd(p, dtype, c, s) : fa::mma_bwd<__nv_bfloat16>(p, c, s);
                if (!st) st = fa_host::launch_convert<__nv_bfloat16>(ws.dq_acc, (__nv_bfloat16*)dq, rows * E, s);
                if (!st && pair)
                    st = fa_host::launch_dpair_fill<__nv_bfloat16>((__nv_bfloat16*)dpair, p.kv_len, QL, KL, (int)QH,
                                                                   (int)B, tile, c, s);
            }
            return st;
        }
    }
    return fail(NNOP_ERR_DTYPE, "flash_attention_bwd: unsupported dtype");
}

}  // extern "C"
