/*
 * nnop_b200.h -- C ABI of the B200 (sm_100a) implementation of NNop's fused
 * kernels: flash attention (forward/backward, pair bias, causal, GQA,
 * key-padding mask), online softmax, RMSNorm, LayerNorm and Llama RoPE.
 *
 * Conventions (all entry points)
 * ------------------------------
 * - Pointers are DEVICE pointers owned by the caller; the library allocates
 *   nothing.  Where a kernel needs scratch, a `*_workspace_size` query gives
 *   the byte count and the caller passes the buffer.
 * - Dimension names and order follow the reference's column-major Julia arrays.
 *   A Julia array of size (d1, d2, ..., dn) is the row-major buffer
 *   [dn]...[d2][d1]; so q (E, QL, QH, B) is the buffer [B][QH][QL][E] and the
 *   pair bias (H, QL, KL, B) is [B][KL][QL][H].
 * - `dtype` is one of NNOP_F32 / NNOP_F16 / NNOP_BF16 and applies to every
 *   floating-point tensor argument unless stated otherwise.  Statistics saved
 *   for the backward pass (lse, rstd, mean) are always float32.
 * - `stream` is a cudaStream_t (NULL = legacy default stream).  Every call is
 *   asynchronous on that stream, like the reference's KernelAbstractions
 *   launches.
 * - Return value: NNOP_OK (0) or a negative NNOP_ERR_* code; shape checks happen
 *   before any launch (as the reference's `error(...)`/`@assert` do) and
 *   nnop_last_error() returns the message for the calling thread.
 */
#ifndef NNOP_B200_H
#define NNOP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NNOP_B200_ABI_VERSION 1

typedef enum {
    NNOP_F32 = 0,
    NNOP_F16 = 1,
    NNOP_BF16 = 2
} nnop_dtype_t;

typedef enum {
    NNOP_OK = 0,
    NNOP_ERR_SHAPE = -1,       /* inconsistent or unsupported dimensions  */
    NNOP_ERR_DTYPE = -2,       /* dtype not supported by this entry point */
    NNOP_ERR_ARG = -3,         /* NULL pointer / bad flag                 */
    NNOP_ERR_WORKSPACE = -4,   /* workspace missing or too small          */
    NNOP_ERR_CUDA = -5,        /* CUDA launch / runtime error             */
    NNOP_ERR_ALIGN = -6        /* pointer not aligned as documented       */
} nnop_status_t;

/* ABI version (NNOP_B200_ABI_VERSION). */
int nnop_abi_version(void);

/* Message for the last non-OK status returned on the calling thread. */
const char* nnop_last_error(void);

/* Fixed text for a status code. */
const char* nnop_status_string(int status);

/*
 * Diagnostic (no counterpart in the reference, whose kernels have no waits):
 * every mbarrier wait inside the tcgen05 attention kernels gives up after about
 * one second and records it in a device flag instead of hanging the GPU.  This
 * call synchronises the current device, returns the wait sites that recorded a
 * timeout since the last call (bits 0-15: forward kernel, bits 16-30: backward
 * kernel, one bit per wait site) and clears the flags.  Non-zero means the
 * results of those launches are not valid.
 */
int nnop_device_wait_timeouts(void);

/*
 * Launch timing of the tensor-core attention kernels (no counterpart in the
 * reference; for benchmarks and profiles).  nnop_kernel_timing(1) makes every
 * following forward / backward call record CUDA events on its stream around
 * its attention kernel (up to 256 launches; later ones are not timed);
 * nnop_kernel_timing(0) stops.  nnop_kernel_timing_read(which, &ms, &count)
 * waits for the recorded events, returns the summed milliseconds and number
 * of timed launches of the forward (which = 0) or backward (which = 1) kernel
 * on the current device, and clears that record.
 */
void nnop_kernel_timing(int enable);
int nnop_kernel_timing_read(int which, double* total_ms, int* count);

/* --------------------------------------------------------------------------
 * Flash attention
 * -------------------------------------------------------------------------- */

/*
 * Forward.  Replaces `_flash_attention` (src/attention.jl:145-197) and its
 * kernel `_flash_attention_fwd!` (src/attention.jl:8-143).
 *
 *   q    [B][QH][QL][E]    (Julia q  (E, QL, QH, B))
 *   k, v [B][KH][KL][E]    (Julia k, v (E, KL, KH, B)); k and v share a shape
 *   pair [B][KL][QL][QH]   (Julia pair (QH, QL, KL, B)) or NULL
 *   kpad_mask [B][KL] uint8 (Julia kpad_mask::Matrix{Bool} (KL, B)) or NULL;
 *                           nonzero = key is kept
 *   o    [B][QH][QL][E]    output, dtype
 *   lse  [B][QH][QL] f32   log-sum-exp of each row's logits; it replaces the
 *                          reference's (ms, ls) pair: lse = ms + log(ls)
 *
 * logits s_ij = scale·(q_i·k_j) [+ pair] with key j masked (−Inf) when
 * causal && j > i or kpad_mask[b][j] == 0; scale = dtype(1/sqrt(E)).
 * Checks (src/attention.jl:153-156): E must be a power of two (16..128 here),
 * QH % KH == 0.  dtype: F32, F16, BF16.
 *   workspace: with a pair bias, >= nnop_flash_attention_fwd_workspace_size(...)
 *   bytes, 256-byte aligned, holding per-head copies of the pair tiles for the
 *   tensor-core kernel; NULL (or too small) selects the slower kernel that
 *   reads the head-innermost pair directly.  Unused without a pair bias.
 */
int nnop_flash_attention_fwd(const void* q, const void* k, const void* v,
                             const void* pair, const uint8_t* kpad_mask,
                             void* o, float* lse,
                             void* workspace, size_t workspace_bytes,
                             int64_t E, int64_t QL, int64_t KL,
                             int64_t QH, int64_t KH, int64_t B,
                             int causal, int dtype, void* stream);

/* Bytes of workspace nnop_flash_attention_fwd can use (0 = none needed). */
size_t nnop_flash_attention_fwd_workspace_size(int64_t E, int64_t QL, int64_t KL,
                                               int64_t QH, int64_t KH, int64_t B,
                                               int has_pair, int dtype);

/* Bytes of workspace nnop_flash_attention_bwd needs for these dimensions
 * (has_pair: a pair bias / dpair will be passed). */
size_t nnop_flash_attention_bwd_workspace_size(int64_t E, int64_t QL, int64_t KL,
                                               int64_t QH, int64_t KH, int64_t B,
                                               int has_pair, int dtype);

/*
 * Backward.  Replaces `∇flash_attention` (src/attention_bwd.jl:213-303) with
 * its kernels `_flash_attention_bwd_preprocess!` (:177-211) and
 * `_flash_attention_bwd!` (:1-175).
 *
 *   dO [B][QH][QL][E]; o, lse as returned by the forward; q, k, v, pair,
 *   kpad_mask as given to the forward.
 *   dq like q, dk/dv like k, dpair like pair (every element written; zero where
 *   the logit was masked) -- dpair must be NULL iff pair is NULL.
 *   workspace: >= nnop_flash_attention_bwd_workspace_size(...) bytes,
 *   256-byte aligned.
 */
int nnop_flash_attention_bwd(const void* dO, const void* o, const float* lse,
                             const void* q, const void* k, const void* v,
                             const void* pair, const uint8_t* kpad_mask,
                             void* dq, void* dk, void* dv, void* dpair,
                             void* workspace, size_t workspace_bytes,
                             int64_t E, int64_t QL, int64_t KL,
                             int64_t QH, int64_t KH, int64_t B,
                             int causal, int dtype, void* stream);

/*
 * Backward reusing the forward's workspace: the forward (called with the same
 * tensors, dimensions, causal flag and dtype, and a 256-byte aligned
 * workspace of at least nnop_flash_attention_fwd_workspace_size(...) bytes)
 * left the per-head pair tiles there, so the backward skips rebuilding them.
 * This is the pullback of the reference's rrule (src/attention_crc.jl:16-31),
 * which keeps the forward's state for `∇flash_attention`.  fwd_workspace may
 * be NULL or hold no tiles (no pair bias, a shape or dtype the tensor-core
 * kernels do not cover); the call is then nnop_flash_attention_bwd.  The pair
 * must not change between the two calls.
 *   workspace: >= nnop_flash_attention_bwd_workspace_size_reuse(...) bytes,
 *   256-byte aligned.
 */
int nnop_flash_attention_bwd_reuse(const void* dO, const void* o, const float* lse,
                                   const void* q, const void* k, const void* v,
                                   const void* pair, const uint8_t* kpad_mask,
                                   void* dq, void* dk, void* dv, void* dpair,
                                   const void* fwd_workspace, size_t fwd_workspace_bytes,
                                   void* workspace, size_t workspace_bytes,
                                   int64_t E, int64_t QL, int64_t KL,
                                   int64_t QH, int64_t KH, int64_t B,
                                   int causal, int dtype, void* stream);

/* Bytes of workspace nnop_flash_attention_bwd_reuse needs when the forward
 * had fwd_workspace_bytes of workspace (less than
 * nnop_flash_attention_bwd_workspace_size when the tiles are reused). */
size_t nnop_flash_attention_bwd_workspace_size_reuse(int64_t E, int64_t QL, int64_t KL,
                                                     int64_t QH, int64_t KH, int64_t B,
                                                     int has_pair, size_t fwd_workspace_bytes,
                                                     int dtype);

/*
 * Forward with the pair bias laid out per head: pair [B][QH][KL][QL] (Julia
 * pair (QL, KL, QH, B)) instead of the reference's head-innermost
 * [B][KL][QL][QH].  It relaxes the layout of the reference's pair read
 * (`_flash_attention_fwd!`, src/attention.jl:72); results are those of
 * nnop_flash_attention_fwd on the same bias.  The tensor-core kernel reads
 * the bias in place, so no workspace and no re-layout pass is needed.
 *   dtype BF16 or F16; E = 64; QL a multiple of 8; all tensors 16-byte aligned.
 *   −Inf bias entries are allowed only at keys kpad_mask removes (the bias
 *   enters the scores through an identity matrix product, where 0·(−Inf)
 *   would spread NaN over 16 queries of that key); mask other keys instead.
 */
int nnop_flash_attention_fwd_pair_per_head(const void* q, const void* k, const void* v,
                                           const void* pair, const uint8_t* kpad_mask,
                                           void* o, float* lse,
                                           int64_t E, int64_t QL, int64_t KL,
                                           int64_t QH, int64_t KH, int64_t B,
                                           int causal, int dtype, void* stream);

/* Bytes of workspace nnop_flash_attention_bwd_pair_per_head needs. */
size_t nnop_flash_attention_bwd_pair_per_head_workspace_size(int64_t E, int64_t QL, int64_t KL,
                                                             int64_t QH, int64_t KH, int64_t B,
                                                             int dtype);

/*
 * Backward with the pair bias and dpair laid out per head ([B][QH][KL][QL]).
 * It relaxes the layout of the reference's dpair (`∇flash_attention`,
 * src/attention_bwd.jl:247-252, a head-innermost array zero-filled before the
 * kernel): the backward kernel stores each dS tile straight into dpair and
 * only the entries no tile covers (above the causal diagonal; keys past the
 * last kept key) are zeroed, so every element is written once.  Arguments as
 * nnop_flash_attention_bwd, with the restrictions of the forward above.
 *   workspace: >= nnop_flash_attention_bwd_pair_per_head_workspace_size(...)
 *   bytes, 256-byte aligned.
 */
int nnop_flash_attention_bwd_pair_per_head(const void* dO, const void* o, const float* lse,
                                           const void* q, const void* k, const void* v,
                                           const void* pair, const uint8_t* kpad_mask,
                                           void* dq, void* dk, void* dv, void* dpair,
                                           void* workspace, size_t workspace_bytes,
                                           int64_t E, int64_t QL, int64_t KL,
                                           int64_t QH, int64_t KH, int64_t B,
                                           int causal, int dtype, void* stream);

/*
 * Llama RoPE fused with attention, forward.  No single counterpart in the
 * reference: the composition `flash_attention(llama_rope(q, k; cos, sin)...)`
 * of `llama_rope` (src/rope/llama_rope.jl:69-98) and `_flash_attention`
 * (src/attention.jl:145-197).  Rotates q and k (written to q_rot, k_rot --
 * the backward's inputs) and runs the attention forward on them.
 *   q [B][QH][L][E], k, v [B][KH][L][E]; cos, sin [cos_batch][L][E] f32
 *   (cos_batch = 1 or B); o, lse as nnop_flash_attention_fwd.
 *   bf16 / f16, E = 64 or 128, no pair bias.
 */
int nnop_flash_attention_rope_fwd(const void* q, const void* k, const void* v,
                                  const float* cos_t, const float* sin_t,
                                  const uint8_t* kpad_mask, void* q_rot, void* k_rot,
                                  void* o, float* lse,
                                  int64_t E, int64_t L, int64_t QH, int64_t KH, int64_t B,
                                  int64_t cos_batch, int causal, int dtype, void* stream);

/* Bytes of workspace nnop_flash_attention_rope_bwd needs. */
size_t nnop_flash_attention_rope_bwd_workspace_size(int64_t E, int64_t L, int64_t QH,
                                                    int64_t KH, int64_t B, int dtype);

/*
 * Backward of the fused RoPE attention: the composition of `∇flash_attention`
 * (src/attention_bwd.jl:213-303) and `∇llama_rope` (src/rope/llama_rope.jl:86-92)
 * with the inverse rotation folded into the attention backward's outputs (dq
 * while its fp32 accumulator is converted, dk in the kernel's dK epilogue):
 * dq, dk are the gradients of the UN-rotated q and k; dv as usual.
 *   q_rot, k_rot, o, lse from nnop_flash_attention_rope_fwd.
 *   workspace: >= nnop_flash_attention_rope_bwd_workspace_size(...) bytes,
 *   256-byte aligned.
 */
int nnop_flash_attention_rope_bwd(const void* dO, const void* o, const float* lse,
                                  const void* q_rot, const void* k_rot, const void* v,
                                  const float* cos_t, const float* sin_t,
                                  const uint8_t* kpad_mask, void* dq, void* dk, void* dv,
                                  void* workspace, size_t workspace_bytes,
                                  int64_t E, int64_t L, int64_t QH, int64_t KH, int64_t B,
                                  int64_t cos_batch, int causal, int dtype, void* stream);

/* --------------------------------------------------------------------------
 * Online softmax over the contiguous axis (Julia dims=1)
 * -------------------------------------------------------------------------- */

/*
 * Forward.  Replaces `online_softmax` (src/softmax.jl:60-68) and its kernel
 * `online_softmax!` (src/softmax.jl:19-58).
 *   x, y [cols][n]   (Julia x (n, cols)); softmax over each run of n.
 */
int nnop_online_softmax_fwd(const void* x, void* y, int64_t n, int64_t cols,
                            int dtype, void* stream);

/*
 * Backward.  Replaces `∇online_softmax` (src/softmax.jl:70-80):
 *   dx = dy∘y − y∘Σ(dy∘y)
 */
int nnop_online_softmax_bwd(const void* dy, const void* y, void* dx,
                            int64_t n, int64_t cols, int dtype, void* stream);

/* --------------------------------------------------------------------------
 * RMSNorm over the contiguous axis (Julia x (emb, n))
 * -------------------------------------------------------------------------- */

/*
 * Forward.  Replaces `_rms_norm` (src/rms_norm.jl:117-137) and `_rms_norm!`
 * (src/rms_norm.jl:3-38).
 *   x, y [n][emb] dtype; w [emb] dtype; rstd [n] f32 = 1/sqrt(mean(x²)+eps)
 *   y = (offset + w)·x·rstd
 */
int nnop_rms_norm_fwd(const void* x, const void* w, void* y, float* rstd,
                      int64_t emb, int64_t n, float eps, float offset,
                      int dtype, void* stream);

size_t nnop_rms_norm_bwd_workspace_size(int64_t emb, int64_t n);

/*
 * Backward.  Replaces `∇rms_norm` (src/rms_norm.jl:139-169) and `_∇rms_norm!`
 * (src/rms_norm.jl:43-115).
 *   dy, x, dx [n][emb] dtype; w [emb] dtype; rstd [n] f32 (from the forward);
 *   dw [emb] f32 (the reference returns a Float32 dw as well).
 */
int nnop_rms_norm_bwd(const void* dy, const void* x, const void* w,
                      const float* rstd, void* dx, float* dw,
                      void* workspace, size_t workspace_bytes,
                      int64_t emb, int64_t n, float offset,
                      int dtype, void* stream);

/*
 * Residual add fused into RMSNorm.  No counterpart in the reference's API: it
 * is the composition a transformer block performs around `rms_norm`
 * (src/rms_norm.jl:117-137), h = x + residual then rms_norm(h), in one pass
 * over x and residual instead of an add pass and a norm pass that reads h
 * back.
 *   x, residual, h, y [n][emb] dtype; w [emb]; rstd [n] f32.
 *   h = x + residual (rounded to dtype, the values a separate add stores);
 *   y = (offset + w)·h·rstd, rstd = 1/sqrt(mean(h²) + eps).
 */
int nnop_add_rms_norm_fwd(const void* x, const void* residual, const void* w,
                          void* h, void* y, float* rstd,
                          int64_t emb, int64_t n, float eps, float offset,
                          int dtype, void* stream);

size_t nnop_add_rms_norm_bwd_workspace_size(int64_t emb, int64_t n);

/*
 * Backward of the fused residual add + RMSNorm.
 *   dy [n][emb]: gradient of y; dh [n][emb] or NULL: the gradient reaching h
 *   from its other use (the residual stream); h, rstd from the forward.
 *   dx = ∇rms_norm(dy, h) + dh -- the gradient of both x and residual; dw f32.
 *   workspace: >= nnop_add_rms_norm_bwd_workspace_size(emb, n) bytes.
 */
int nnop_add_rms_norm_bwd(const void* dy, const void* dh, const void* h,
                          const void* w, const float* rstd, void* dx, float* dw,
                          void* workspace, size_t workspace_bytes,
                          int64_t emb, int64_t n, float offset,
                          int dtype, void* stream);

/*
 * RMSNorm backward that allocates nothing.  No counterpart in the reference.
 *
 * For callers that cannot allocate device memory where they need the
 * gradient -- code running inside a memory pool's own callbacks, runtimes that
 * plan all device memory ahead of time, hosts without access to an allocator
 * at the call site -- and so cannot pass the workspace nnop_rms_norm_bwd needs.
 * Same arguments and results as nnop_rms_norm_bwd without the workspace.
 *
 * The scratch is an 8 MiB array inside the library (held on every GPU that
 * loads it until the process exits); emb may be at most 2^21 (2,097,152),
 * larger values return NNOP_ERR_SHAPE.  The first call on a device looks the
 * array's device address up (cudaGetSymbolAddress), so make that first call
 * before any stream capture on that device; the address is kept with the
 * device's context and looked up again after a device reset (a new context
 * loads the array at a new address).  All calls on a device share the
 * one array: calls that can overlap on the GPU (different streams without
 * ordering between them) race on it and must be serialised by the caller.
 */
int nnop_rms_norm_bwd_noalloc(const void* dy, const void* x, const void* w,
                              const float* rstd, void* dx, float* dw,
                              int64_t emb, int64_t n, float offset,
                              int dtype, void* stream);

/* --------------------------------------------------------------------------
 * LayerNorm over the contiguous axis (Julia x (emb, n))
 * -------------------------------------------------------------------------- */

/*
 * Forward.  Replaces `_layer_norm` (src/layer_norm.jl:150-170) and
 * `_layer_norm!` (src/layer_norm.jl:8-63).
 *   x, y [n][emb], w, b [emb] dtype; mean, rstd [n] f32 (the reference's μ, Σ)
 */
int nnop_layer_norm_fwd(const void* x, const void* w, const void* b, void* y,
                        float* mean, float* rstd, int64_t emb, int64_t n,
                        float eps, int dtype, void* stream);

size_t nnop_layer_norm_bwd_workspace_size(int64_t emb, int64_t n);

/*
 * Backward.  Replaces `∇layer_norm` (src/layer_norm.jl:172-204) and
 * `_∇layer_norm!` (src/layer_norm.jl:65-148).
 *   dw, db [emb] in dtype (eltype(w) in the reference).
 */
int nnop_layer_norm_bwd(const void* dy, const void* x, const void* w,
                        const float* mean, const float* rstd,
                        void* dx, void* dw, void* db,
                        void* workspace, size_t workspace_bytes,
                        int64_t emb, int64_t n, int dtype, void* stream);

/* --------------------------------------------------------------------------
 * Llama RoPE
 * -------------------------------------------------------------------------- */

/*
 * Rotation of q and k in one launch.  Replaces `_llama_rope`
 * (src/rope/llama_rope.jl:69-89) and `llama_rope!` (:24-65).
 *   q, q_out [B][QH][L][E]; k, k_out [B][KH][L][E] (dtype)
 *   cos, sin [cos_batch][L][E] f32 (Julia (E, L, batch)); cos_batch is B, or
 *   1 to share one table across the batch.
 *   sign = +1 forward, -1 backward (∇llama_rope, :312).
 * For i < E/2: out[i] = x[i]c − x[i+E/2]s, out[i+E/2] = x[i+E/2]c + x[i]s, with
 * c = cos[i], s = sign·sin[i].  q_out may alias q and k_out may alias k.
 */
int nnop_llama_rope(const void* q, const void* k,
                    const float* cos_t, const float* sin_t,
                    void* q_out, void* k_out,
                    int64_t E, int64_t L, int64_t QH, int64_t KH, int64_t B,
                    int64_t cos_batch, float sign, int dtype, void* stream);

/*
 * cos/sin tables of `LlamaRotaryEmbedding(dim; base)(position_ids)`
 * (src/rope/llama_rope.jl:7-22) computed on the device.
 *   position_ids [B][L] f32 (Julia (L, B)); cos_t, sin_t [B][L][dim] f32.
 */
int nnop_llama_rope_cos_sin(const float* position_ids, float* cos_t, float* sin_t,
                            int64_t dim, int64_t L, int64_t B, int64_t base,
                            void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NNOP_B200_H */
