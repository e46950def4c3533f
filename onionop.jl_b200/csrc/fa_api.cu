// C-ABI entry points of flash attention: argument checks (the reference's
// `_flash_attention` / `∇flash_attention` error()s, src/attention.jl:153-156 and
// src/attention_bwd.jl:224-227), workspace layout and kernel dispatch.
#include "fa_common.cuh"

#include <cstdlib>
#include <mutex>
#include <type_traits>

namespace nnop {
namespace fa {
template <typename T> int mma_fwd(const Params& p, bool causal, cudaStream_t s);
template <typename T> int mma_bwd(const Params& p, bool causal, cudaStream_t s);
int mma_tile();
int simt_fwd(const Params& p, bool causal, cudaStream_t s);
int simt_bwd(const Params& p, bool causal, cudaStream_t s);
int simt_tile();
bool sm100_fwd_supported(const Params& p, int dtype, bool have_pair_tiles);
int sm100_fwd(const Params& p, const void* pair_tiles, int dtype, bool causal, cudaStream_t s);
bool sm100_bwd_supported(const Params& p, int dtype);
int sm100_bwd(const Params& p, const void* pair_tiles, void* ds_tiles, int dtype, bool causal, cudaStream_t s);
int sm100_bwd_tile();
int sm100_fwd_timeouts();
int sm100_bwd_timeouts();
int sm100_bwd128_timeouts();
int sm100_fwd2_timeouts();
}  // namespace fa

namespace fa_host {
size_t pair_tiles_bytes(int64_t QL, int64_t KL, int64_t H, int64_t B);
template <typename T>
int launch_pair_tiles(const T* pair, T* out, const int* kv_len, int64_t QL, int64_t KL, int H, int B, bool causal,
                      cudaStream_t s);
template <typename T>
int launch_dpair_from_tiles(const T* tiles, T* dpair, const int* kv_len, int64_t QL, int64_t KL, int H, int B,
                            bool causal, cudaStream_t s);
}  // namespace fa_host

namespace {

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// NNOP_B200_FA=mma selects the mma.sync kernels for every shape (used by the
// tests to check both kernel families; NNOP_B200_FA=one_tile selects the
// one-tile tcgen05 forward, fa_fwd_sm100.cu); the default picks the tcgen05
// kernels where they apply.
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

// The tcgen05 kernels take the pair bias as per-head tiles (pair_tiles.cu):
// bf16/f16, E = 64, at most 64 heads (the re-layout stages [8][128][H] blocks).
bool pair_tiles_path(int64_t E, int64_t QH, int dtype) {
    return !force_mma() && (dtype == NNOP_BF16 || dtype == NNOP_F16) && E == 64 && QH <= 64;
}

// Optional CUDA-event timing of the attention kernels (nnop_kernel_timing).
struct KernelTimer {
    static constexpr int kMax = 256;
    std::mutex mu;
    bool on = false;
    int dev[2][kMax];
    int n[2] = {0, 0};
    cudaEvent_t ev[2][kMax][2];
    bool made = false;
};
KernelTimer& timer() {
    static KernelTimer t;
    return t;
}
// Records the start event of a timed launch; returns the slot or -1.
int timer_begin(int which, cudaStream_t s) {
    KernelTimer& t = timer();
    std::lock_guard<std::mutex> lock(t.mu);
    if (!t.on || t.n[which] >= KernelTimer::kMax) return -1;
    if (!t.made) {
        for (int w = 0; w < 2; ++w)
            for (int i = 0; i < KernelTimer::kMax; ++i)
                for (int e = 0; e < 2; ++e)
                    if (cudaEventCreate(&t.ev[w][i][e]) != cudaSuccess) return -1;
        t.made = true;
    }
    const int slot = t.n[which]++;
    cudaGetDevice(&t.dev[which][slot]);
    cudaEventRecord(t.ev[which][slot][0], s);
    return slot;
}
void timer_end(int which, int slot, cudaStream_t s) {
    if (slot < 0) return;
    cudaEventRecord(timer().ev[which][slot][1], s);
}

struct BwdWorkspace {
    int* kv_len;
    float* delta;
    float* dq_acc;
    void* ds_tiles;     // tcgen05 path with a pair bias: the per-head dS tiles
    void* pair_tiles;   // ... and the per-head pair tiles (unless the forward's are reused)
    size_t bytes;
};

// Size the forward's workspace needs for the pair tiles (0: no tiles).
size_t fwd_tiles_bytes(int64_t E, int64_t QL, int64_t KL, int64_t QH, int64_t B, bool has_pair, int dtype) {
    if (!has_pair || !pair_tiles_path(E, QH, dtype)) return 0;
    return align256(fa_host::pair_tiles_bytes(QL, KL, QH, B));
}

// True when nnop_flash_attention_fwd, called with this workspace, wrote the
// per-head pair tiles into it (the tcgen05 forward ran with a pair bias).
bool fwd_keeps_tiles(const fa::Params& p, int dtype, const void* ws, size_t ws_bytes) {
    const size_t need = fwd_tiles_bytes(p.E, p.QL, p.KL, p.QH, p.B, p.pair != nullptr, dtype);
    const bool tiles = need > 0 && ws != nullptr && ws_bytes >= need && (reinterpret_cast<uintptr_t>(ws) & 255u) == 0;
    return tiles && !force_mma() && fa::sm100_fwd_supported(p, dtype, true);
}

BwdWorkspace bwd_layout(void* base, int64_t E, int64_t QL, int64_t KL, int64_t QH, int64_t B, bool has_pair,
                        bool own_pair_tiles, int dtype) {
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
    w.pair_tiles = w.ds_tiles = nullptr;
    if (has_pair && pair_tiles_path(E, QH, dtype)) {
        const size_t tb = align256(fa_host::pair_tiles_bytes(QL, KL, QH, B));
        w.ds_tiles = p ? p + off : nullptr;
        off += tb;
        if (own_pair_tiles) {
            w.pair_tiles = p ? p + off : nullptr;
            off += tb;
        }
    }
    w.bytes = off;
    return w;
}

// f16/bf16 backward: delta, dq accumulator, the tcgen05 (or mma.sync) kernel,
// dq conversion, and dpair (from the per-head dS tiles, or the zero fill of the
// tiles the mma.sync kernel does not visit).  `fwd_tiles`: the forward's pair
// tiles when they are reused, else nullptr (the tiles are built here).
template <typename T>
int bwd_16bit(fa::Params& p, const BwdWorkspace& ws, const void* fwd_tiles, int64_t rows, bool causal, int dtype,
              cudaStream_t s) {
    const int64_t E = p.E, QL = p.QL, KL = p.KL;
    const float sc = (float)(1.0 / sqrt((double)E));
    p.scale = std::is_same<T, __nv_bfloat16>::value ? __bfloat162float(__float2bfloat16_rn(sc))
                                                    : __half2float(__float2half_rn(sc));
    if (cudaMemsetAsync(ws.dq_acc, 0, (size_t)rows * E * sizeof(float), s) != cudaSuccess)
        return fail(NNOP_ERR_CUDA, "flash_attention_bwd: memset failed");
    p.dq_acc = ws.dq_acc;
    const void* tiles = fwd_tiles ? fwd_tiles : ws.pair_tiles;
    const bool tc = !force_mma() && fa::sm100_bwd_supported(p, dtype) && (p.pair == nullptr || (tiles && ws.ds_tiles));
    int st = fa_host::launch_preprocess<T>((const T*)p.dO, (const T*)p.o, ws.delta, rows, (int)E, s);
    if (st) return st;
    if (tc) {
        if (p.pair && !fwd_tiles) {
            st = fa_host::launch_pair_tiles<T>((const T*)p.pair, (T*)ws.pair_tiles, p.kv_len, QL, KL, p.QH, p.B,
                                               causal, s);
            if (st) return st;
        }
        const int slot = timer_begin(1, s);
        st = fa::sm100_bwd(p, tiles, ws.ds_tiles, dtype, causal, s);
        timer_end(1, slot, s);
    } else {
        st = fa::mma_bwd<T>(p, causal, s);
    }
    if (st) return st;
    st = fa_host::launch_convert<T>(ws.dq_acc, (T*)p.dq, rows * E, s);
    if (st || !p.pair) return st;
    if (tc)
        return fa_host::launch_dpair_from_tiles<T>((const T*)ws.ds_tiles, (T*)p.dpair, p.kv_len, QL, KL, p.QH, p.B,
                                                   causal, s);
    return fa_host::launch_dpair_fill<T>((T*)p.dpair, p.kv_len, QL, KL, p.QH, p.B, fa::mma_tile(), causal, s);
}

}  // namespace
}  // namespace nnop

using namespace nnop;

extern "C" {

void nnop_kernel_timing(int enable) {
    KernelTimer& t = timer();
    std::lock_guard<std::mutex> lock(t.mu);
    t.on = enable != 0;
}

int nnop_kernel_timing_read(int which, double* total_ms, int* count) {
    if ((which != 0 && which != 1) || !total_ms || !count)
        return fail(NNOP_ERR_ARG, "kernel_timing_read: which must be 0 or 1, outputs non-NULL");
    KernelTimer& t = timer();
    std::lock_guard<std::mutex> lock(t.mu);
    int dev = 0;
    cudaGetDevice(&dev);
    double sum = 0;
    int c = 0;
    for (int i = 0; i < t.n[which]; ++i) {
        if (t.dev[which][i] != dev) continue;
        float ms = 0.f;
        if (cudaEventSynchronize(t.ev[which][i][1]) != cudaSuccess ||
            cudaEventElapsedTime(&ms, t.ev[which][i][0], t.ev[which][i][1]) != cudaSuccess)
            return fail(NNOP_ERR_CUDA, "kernel_timing_read: event query failed");
        sum += ms;
        ++c;
    }
    t.n[which] = 0;
    *total_ms = sum;
    *count = c;
    return NNOP_OK;
}

int nnop_device_wait_timeouts(void) {
    const int f = fa::sm100_fwd_timeouts() | fa::sm100_fwd2_timeouts();
    const int b = fa::sm100_bwd_timeouts() | fa::sm100_bwd128_timeouts();
    return (f & 0xffff) | ((b & 0x7fff) << 16);
}

size_t nnop_flash_attention_fwd_workspace_size(int64_t E, int64_t QL, int64_t KL, int64_t QH, int64_t KH, int64_t B,
                                               int has_pair, int dtype) {
    (void)KH;
    if (E <= 0 || QL < 0 || KL < 0 || QH <= 0 || B < 0) return 0;
    return fwd_tiles_bytes(E, QL, KL, QH, B, has_pair != 0, dtype);
}

int nnop_flash_attention_fwd(const void* q, const void* k, const void* v, const void* pair,
                             const uint8_t* kpad_mask, void* o, float* lse, void* workspace, size_t workspace_bytes,
                             int64_t E, int64_t QL, int64_t KL, int64_t QH, int64_t KH, int64_t B, int causal,
                             int dtype, void* stream) {
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
        case NNOP_BF16: {
            const bool bf = dtype == NNOP_BF16;
            const float sc = (float)(1.0 / sqrt((double)E));
            p.scale = bf ? __bfloat162float(__float2bfloat16_rn(sc)) : __half2float(__float2half_rn(sc));
            // The pair bias reaches the tcgen05 kernel as per-head tiles written
            // into the workspace; without (enough) workspace the mma.sync
            // kernel, which reads the pair directly, runs instead.
            const size_t need = nnop_flash_attention_fwd_workspace_size(E, QL, KL, QH, KH, B, pair != nullptr, dtype);
            const bool tiles = pair != nullptr && need > 0 && workspace != nullptr && workspace_bytes >= need &&
                               (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0;
            if (!force_mma() && fa::sm100_fwd_supported(p, dtype, tiles)) {
                if (tiles) {
                    st = bf ? fa_host::launch_pair_tiles<__nv_bfloat16>((const __nv_bfloat16*)pair,
                                                                         (__nv_bfloat16*)workspace, nullptr, QL, KL,
                                                                         (int)QH, (int)B, causal != 0, s)
                            : fa_host::launch_pair_tiles<__half>((const __half*)pair, (__half*)workspace, nullptr, QL,
                                                                 KL, (int)QH, (int)B, causal != 0, s);
                    if (st) return st;
                }
                const int slot = timer_begin(0, s);
                st = fa::sm100_fwd(p, workspace, dtype, causal != 0, s);
                timer_end(0, slot, s);
                return st;
            }
            return bf ? fa::mma_fwd<__nv_bfloat16>(p, causal != 0, s) : fa::mma_fwd<__half>(p, causal != 0, s);
        }
    }
    return fail(NNOP_ERR_DTYPE, "flash_attention_fwd: unsupported dtype");
}

size_t nnop_flash_attention_bwd_workspace_size(int64_t E, int64_t QL, int64_t KL, int64_t QH, int64_t KH, int64_t B,
                                               int has_pair, int dtype) {
    (void)KH;
    if (E <= 0 || QL < 0 || KL < 0 || QH <= 0 || B < 0) return 0;
    return bwd_layout(nullptr, E, QL, KL, QH, B, has_pair != 0, true, dtype).bytes;
}

size_t nnop_flash_attention_bwd_workspace_size_reuse(int64_t E, int64_t QL, int64_t KL, int64_t QH, int64_t KH,
                                                     int64_t B, int has_pair, size_t fwd_workspace_bytes, int dtype) {
    (void)KH;
    if (E <= 0 || QL < 0 || KL < 0 || QH <= 0 || B < 0) return 0;
    const size_t need = fwd_tiles_bytes(E, QL, KL, QH, B, has_pair != 0, dtype);
    const bool reuse = need > 0 && fwd_workspace_bytes >= need && (KL + 31) / 32 <= 2048;
    return bwd_layout(nullptr, E, QL, KL, QH, B, has_pair != 0, !reuse, dtype).bytes;
}

int nnop_flash_attention_bwd_reuse(const void* dO, const void* o, const float* lse, const void* q, const void* k,
                                   const void* v, const void* pair, const uint8_t* kpad_mask, void* dq, void* dk,
                                   void* dv, void* dpair, const void* fwd_workspace, size_t fwd_workspace_bytes,
                                   void* workspace, size_t workspace_bytes, int64_t E, int64_t QL, int64_t KL,
                                   int64_t QH, int64_t KH, int64_t B, int causal, int dtype, void* stream) {
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
    fa::Params p{};
    p.q = q; p.k = k; p.v = v; p.pair = pair; p.kmask = kpad_mask; p.o = const_cast<void*>(o);
    p.lse = const_cast<float*>(lse); p.dO = dO;
    p.dq = dq; p.dk = dk; p.dv = dv; p.dpair = dpair;
    p.QL = QL; p.KL = KL; p.E = (int)E; p.QH = (int)QH; p.KH = (int)KH; p.B = (int)B;
    p.n_rep = (int)(QH / KH);
    const bool reuse = pair != nullptr && dtype != NNOP_F32 && fwd_keeps_tiles(p, dtype, fwd_workspace, fwd_workspace_bytes);
    BwdWorkspace ws = bwd_layout(workspace, E, QL, KL, QH, B, pair != nullptr, !reuse, dtype);
    if (!workspace || workspace_bytes < ws.bytes)
        return fail(NNOP_ERR_WORKSPACE, "flash_attention_bwd: workspace too small (need " + std::to_string(ws.bytes) +
                                            " bytes)");
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
        return fail(NNOP_ERR_ALIGN, "flash_attention_bwd: workspace must be 256-byte aligned");
    cudaStream_t s = (cudaStream_t)stream;
    p.delta = ws.delta;
    p.kv_len = kpad_mask ? ws.kv_len : nullptr;
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
            return bwd_16bit<__half>(p, ws, reuse ? fwd_workspace : nullptr, rows, c, dtype, s);
        case NNOP_BF16:
            return bwd_16bit<__nv_bfloat16>(p, ws, reuse ? fwd_workspace : nullptr, rows, c, dtype, s);
    }
    return fail(NNOP_ERR_DTYPE, "flash_attention_bwd: unsupported dtype");
}

int nnop_flash_attention_bwd(const void* dO, const void* o, const float* lse, const void* q, const void* k,
                             const void* v, const void* pair, const uint8_t* kpad_mask, void* dq, void* dk,
                             void* dv, void* dpair, void* workspace, size_t workspace_bytes, int64_t E, int64_t QL,
                             int64_t KL, int64_t QH, int64_t KH, int64_t B, int causal, int dtype, void* stream) {
    return nnop_flash_attention_bwd_reuse(dO, o, lse, q, k, v, pair, kpad_mask, dq, dk, dv, dpair, nullptr, 0,
                                          workspace, workspace_bytes, E, QL, KL, QH, KH, B, causal, dtype, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Pair bias laid out per head.
//
// The reference takes the pair bias head-innermost, Julia (H, QL, KL, B)
// (src/attention.jl:72), and returns dpair the same way, zero-filled first
// (src/attention_bwd.jl:247-252).  The tcgen05 kernels read and write it per
// head and key-major, so the drop-in entry points above move it through
// re-layout passes (pair_tiles.cu).  A caller that can keep the bias per head,
// Julia (QL, KL, H, B) = row-major [B][QH][KL][QL], uses these entry points
// instead: the forward reads the bias with a 3-D tensor map, the backward
// stores dS straight into dpair, and each CTA also zeroes the parts of its key
// rows that no tile covers (above the causal diagonal, every query of a key
// tile past the last kept key), so every element is written once.
// bf16 / f16, E = 64, QL a multiple of 8 (16-byte rows).  The forward adds
// the bias on the tensor cores (an identity UMMA), where 0·(−Inf) would turn
// the 16 queries of a UMMA K block into NaN, so −Inf entries are allowed only
// at keys the key-padding mask removes (their scores are discarded); express
// other −Inf entries with the mask.  There is no mma.sync fallback:
// NNOP_B200_FA does not apply here.
// ---------------------------------------------------------------------------
namespace nnop {
namespace {

int check_per_head(const char* what, int64_t E, int64_t QL, int64_t KL, int64_t QH, int64_t KH, int64_t B,
                   int dtype) {
    int st = check_dims(E, QL, KL, QH, KH, B, dtype);
    if (st) return st;
    if (dtype != NNOP_BF16 && dtype != NNOP_F16)
        return fail(NNOP_ERR_DTYPE, std::string(what) + ": a per-head pair bias takes bf16 or f16");
    if (E != 64) return fail(NNOP_ERR_SHAPE, std::string(what) + ": a per-head pair bias takes E = 64");
    if (QL % 8 != 0)
        return fail(NNOP_ERR_SHAPE, std::string(what) + ": a per-head pair bias needs QL a multiple of 8 (got " +
                                        std::to_string(QL) + ")");
    if ((KL + 31) / 32 > 2048) return fail(NNOP_ERR_SHAPE, std::string(what) + ": key length above 65536");
    return NNOP_OK;
}

}  // namespace
}  // namespace nnop

extern "C" {

int nnop_flash_attention_fwd_pair_per_head(const void* q, const void* k, const void* v, const void* pair,
                                           const uint8_t* kpad_mask, void* o, float* lse, int64_t E, int64_t QL,
                                           int64_t KL, int64_t QH, int64_t KH, int64_t B, int causal, int dtype,
                                           void* stream) {
    int st = check_per_head("flash_attention_fwd", E, QL, KL, QH, KH, B, dtype);
    if (st) return st;
    if (QL == 0 || B == 0) return NNOP_OK;
    if (!q || !k || !v || !pair || !o || !lse) return fail(NNOP_ERR_ARG, "flash_attention_fwd: NULL pointer");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(pair))
        return fail(NNOP_ERR_ALIGN, "flash_attention_fwd: q, k, v, pair, o must be 16-byte aligned");
    fa::Params p{};
    p.q = q; p.k = k; p.v = v; p.pair = pair; p.kmask = kpad_mask; p.o = o; p.lse = lse;
    p.QL = QL; p.KL = KL; p.E = (int)E; p.QH = (int)QH; p.KH = (int)KH; p.B = (int)B;
    p.n_rep = (int)(QH / KH);
    p.pair_per_head = 1;
    const float sc = (float)(1.0 / sqrt((double)E));
    p.scale = dtype == NNOP_BF16 ? __bfloat162float(__float2bfloat16_rn(sc)) : __half2float(__float2half_rn(sc));
    cudaStream_t s = (cudaStream_t)stream;
    const int slot = timer_begin(0, s);
    st = fa::sm100_fwd(p, nullptr, dtype, causal != 0, s);
    timer_end(0, slot, s);
    return st;
}

size_t nnop_flash_attention_bwd_pair_per_head_workspace_size(int64_t E, int64_t QL, int64_t KL, int64_t QH,
                                                             int64_t KH, int64_t B, int dtype) {
    (void)KH;
    if (E <= 0 || QL < 0 || KL < 0 || QH <= 0 || B < 0) return 0;
    return bwd_layout(nullptr, E, QL, KL, QH, B, false, false, dtype).bytes;
}

int nnop_flash_attention_bwd_pair_per_head(const void* dO, const void* o, const float* lse, const void* q,
                                           const void* k, const void* v, const void* pair, const uint8_t* kpad_mask,
                                           void* dq, void* dk, void* dv, void* dpair, void* workspace,
                                           size_t workspace_bytes, int64_t E, int64_t QL, int64_t KL, int64_t QH,
                                           int64_t KH, int64_t B, int causal, int dtype, void* stream) {
    int st = check_per_head("flash_attention_bwd", E, QL, KL, QH, KH, B, dtype);
    if (st) return st;
    cudaStream_t s = (cudaStream_t)stream;
    if (QL == 0 || B == 0) {
        // no queries: dk = dv = 0 (dpair is empty)
        if (B > 0 && KL > 0 &&
            (cudaMemsetAsync(dk, 0, (size_t)B * KH * KL * E * 2, s) != cudaSuccess ||
             cudaMemsetAsync(dv, 0, (size_t)B * KH * KL * E * 2, s) != cudaSuccess))
            return fail(NNOP_ERR_CUDA, "flash_attention_bwd: memset failed");
        return NNOP_OK;
    }
    if (!dO || !o || !lse || !q || !k || !v || !pair || !dq || !dk || !dv || !dpair)
        return fail(NNOP_ERR_ARG, "flash_attention_bwd: NULL pointer");
    if (!aligned16(dO) || !aligned16(o) || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(dq) ||
        !aligned16(dk) || !aligned16(dv) || !aligned16(pair) || !aligned16(dpair))
        return fail(NNOP_ERR_ALIGN, "flash_attention_bwd: dense tensors must be 16-byte aligned");
    BwdWorkspace ws = bwd_layout(workspace, E, QL, KL, QH, B, false, false, dtype);
    if (!workspace || workspace_bytes < ws.bytes)
        return fail(NNOP_ERR_WORKSPACE, "flash_attention_bwd: workspace too small (need " + std::to_string(ws.bytes) +
                                            " bytes)");
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
        return fail(NNOP_ERR_ALIGN, "flash_attention_bwd: workspace must be 256-byte aligned");
    fa::Params p{};
    p.q = q; p.k = k; p.v = v; p.pair = pair; p.kmask = kpad_mask; p.o = const_cast<void*>(o);
    p.lse = const_cast<float*>(lse); p.dO = dO;
    p.dq = dq; p.dk = dk; p.dv = dv; p.dpair = dpair;
    p.QL = QL; p.KL = KL; p.E = (int)E; p.QH = (int)QH; p.KH = (int)KH; p.B = (int)B;
    p.n_rep = (int)(QH / KH);
    p.pair_per_head = 1;
    p.delta = ws.delta;
    p.kv_len = kpad_mask ? ws.kv_len : nullptr;
    p.dq_acc = ws.dq_acc;
    const float sc = (float)(1.0 / sqrt((double)E));
    p.scale = dtype == NNOP_BF16 ? __bfloat162float(__float2bfloat16_rn(sc)) : __half2float(__float2half_rn(sc));
    const int64_t rows = B * QH * QL;
    if (kpad_mask && (st = fa_host::launch_kv_len(kpad_mask, ws.kv_len, KL, (int)B, s))) return st;
    if (cudaMemsetAsync(ws.dq_acc, 0, (size_t)rows * E * sizeof(float), s) != cudaSuccess)
        return fail(NNOP_ERR_CUDA, "flash_attention_bwd: memset failed");
    const bool c = causal != 0;
    if (dtype == NNOP_BF16) {
        using T = __nv_bfloat16;
        if ((st = fa_host::launch_preprocess<T>((const T*)dO, (const T*)o, ws.delta, rows, (int)E, s))) return st;
        const int slot = timer_begin(1, s);
        st = fa::sm100_bwd(p, nullptr, nullptr, dtype, c, s);
        timer_end(1, slot, s);
        if (st) return st;
        return fa_host::launch_convert<T>(ws.dq_acc, (T*)dq, rows * E, s);   // dpair zeros: written by the kernel
    }
    using T = __half;
    if ((st = fa_host::launch_preprocess<T>((const T*)dO, (const T*)o, ws.delta, rows, (int)E, s))) return st;
    const int slot = timer_begin(1, s);
    st = fa::sm100_bwd(p, nullptr, nullptr, dtype, c, s);
    timer_end(1, slot, s);
    if (st) return st;
    return fa_host::launch_convert<T>(ws.dq_acc, (T*)dq, rows * E, s);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Llama RoPE fused with attention.
//
// The reference composes `llama_rope` (src/rope/llama_rope.jl:69-98) with
// `flash_attention` (src/attention_crc.jl:4-31): two passes forward (rotate,
// attend) and two backward (attention backward, then the inverse rotation of
// dq and dk).  These entry points keep the forward's rotation as one launch
// (its rotated q and k are the attention backward's inputs, returned to the
// caller to save) and fold the backward's inverse rotation into the
// attention backward's own outputs: dq is rotated while its fp32 accumulator
// is converted to the dtype, dk in the tensor-core kernel's dK epilogue --
// the separate RoPE backward pass (a read and a write of dq and dk) is gone.
// bf16 / f16, E = 64 or 128, no pair bias, q and k of one sequence length L;
// cos, sin [cos_batch][L][E] fp32 with cos_batch = 1 or B.
// ---------------------------------------------------------------------------
namespace nnop {
namespace {

int check_rope_attention(const char* what, int64_t E, int64_t L, int64_t QH, int64_t KH, int64_t B,
                         int64_t cos_batch, int dtype) {
    int st = check_dims(E, L, L, QH, KH, B, dtype);
    if (st) return st;
    if (dtype != NNOP_BF16 && dtype != NNOP_F16)
        return fail(NNOP_ERR_DTYPE, std::string(what) + ": fused RoPE attention takes bf16 or f16");
    if (E != 64 && E != 128)
        return fail(NNOP_ERR_SHAPE, std::string(what) + ": fused RoPE attention takes E = 64 or 128");
    if (cos_batch != 1 && cos_batch != B)
        return fail(NNOP_ERR_SHAPE, std::string(what) + ": cos/sin batch must equal the q/k batch or be 1");
    if ((L + 31) / 32 > 2048) return fail(NNOP_ERR_SHAPE, std::string(what) + ": sequence longer than 65536");
    return NNOP_OK;
}

}  // namespace
}  // namespace nnop

extern "C" {

int nnop_flash_attention_rope_fwd(const void* q, const void* k, const void* v, const float* cos_t,
                                  const float* sin_t, const uint8_t* kpad_mask, void* q_rot, void* k_rot, void* o,
                                  float* lse, int64_t E, int64_t L, int64_t QH, int64_t KH, int64_t B,
                                  int64_t cos_batch, int causal, int dtype, void* stream) {
    int st = check_rope_attention("flash_attention_rope_fwd", E, L, QH, KH, B, cos_batch, dtype);
    if (st) return st;
    if (L == 0 || B == 0) return NNOP_OK;
    if ((st = nnop_llama_rope(q, k, cos_t, sin_t, q_rot, k_rot, E, L, QH, KH, B, cos_batch, 1.0f, dtype, stream)))
        return st;
    return nnop_flash_attention_fwd(q_rot, k_rot, v, nullptr, kpad_mask, o, lse, nullptr, 0, E, L, L, QH, KH, B, causal,
                                    dtype, stream);
}

size_t nnop_flash_attention_rope_bwd_workspace_size(int64_t E, int64_t L, int64_t QH, int64_t KH, int64_t B,
                                                    int dtype) {
    (void)KH;
    if (E <= 0 || L < 0 || QH <= 0 || B < 0) return 0;
    return bwd_layout(nullptr, E, L, L, QH, B, false, false, dtype).bytes;
}

int nnop_flash_attention_rope_bwd(const void* dO, const void* o, const float* lse, const void* q_rot,
                                  const void* k_rot, const void* v, const float* cos_t, const float* sin_t,
                                  const uint8_t* kpad_mask, void* dq, void* dk, void* dv, void* workspace,
                                  size_t workspace_bytes, int64_t E, int64_t L, int64_t QH, int64_t KH, int64_t B,
                                  int64_t cos_batch, int causal, int dtype, void* stream) {
    int st = check_rope_attention("flash_attention_rope_bwd", E, L, QH, KH, B, cos_batch, dtype);
    if (st) return st;
    cudaStream_t s = (cudaStream_t)stream;
    if (L == 0 || B == 0) return NNOP_OK;
    if (!dO || !o || !lse || !q_rot || !k_rot || !v || !cos_t || !sin_t || !dq || !dk || !dv)
        return fail(NNOP_ERR_ARG, "flash_attention_rope_bwd: NULL pointer");
    if (!aligned16(dO) || !aligned16(o) || !aligned16(q_rot) || !aligned16(k_rot) || !aligned16(v) ||
        !aligned16(dq) || !aligned16(dk) || !aligned16(dv) || !aligned16(cos_t) || !aligned16(sin_t))
        return fail(NNOP_ERR_ALIGN, "flash_attention_rope_bwd: tensors must be 16-byte aligned");
    BwdWorkspace ws = bwd_layout(workspace, E, L, L, QH, B, false, false, dtype);
    if (!workspace || workspace_bytes < ws.bytes)
        return fail(NNOP_ERR_WORKSPACE, "flash_attention_rope_bwd: workspace too small (need " +
                                            std::to_string(ws.bytes) + " bytes)");
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
        return fail(NNOP_ERR_ALIGN, "flash_attention_rope_bwd: workspace must be 256-byte aligned");
    fa::Params p{};
    p.q = q_rot; p.k = k_rot; p.v = v; p.kmask = kpad_mask; p.o = const_cast<void*>(o);
    p.lse = const_cast<float*>(lse); p.dO = dO;
    p.dq = dq; p.dk = dk; p.dv = dv;
    p.QL = L; p.KL = L; p.E = (int)E; p.QH = (int)QH; p.KH = (int)KH; p.B = (int)B;
    p.n_rep = (int)(QH / KH);
    p.delta = ws.delta;
    p.kv_len = kpad_mask ? ws.kv_len : nullptr;
    p.dq_acc = ws.dq_acc;
    p.rope_cos = cos_t; p.rope_sin = sin_t; p.rope_cb = cos_batch;
    const float sc = (float)(1.0 / sqrt((double)E));
    p.scale = dtype == NNOP_BF16 ? __bfloat162float(__float2bfloat16_rn(sc)) : __half2float(__float2half_rn(sc));
    const int64_t rows = B * QH * L;
    if (kpad_mask && (st = fa_host::launch_kv_len(kpad_mask, ws.kv_len, L, (int)B, s))) return st;
    if (cudaMemsetAsync(ws.dq_acc, 0, (size_t)rows * E * sizeof(float), s) != cudaSuccess)
        return fail(NNOP_ERR_CUDA, "flash_attention_rope_bwd: memset failed");
    const bool c = causal != 0;
    NNOP_DISPATCH_DTYPE(dtype, T, {
        if constexpr (sizeof(T) == 2) {
            if ((st = fa_host::launch_preprocess<T>((const T*)dO, (const T*)o, ws.delta, rows, (int)E, s))) return st;
            const int slot = timer_begin(1, s);
            st = fa::sm100_bwd(p, nullptr, nullptr, dtype, c, s);
            timer_end(1, slot, s);
            if (st) return st;
            return fa_host::launch_convert_rope<T>(ws.dq_acc, (T*)dq, cos_t, sin_t, cos_batch, B, QH, L, (int)E, s);
        }
    });
    return fail(NNOP_ERR_DTYPE, "flash_attention_rope_bwd: bf16 or f16 only");
}

}  // extern "C"
