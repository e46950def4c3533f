"""nnop -- the NNop fused-kernel API over the B200 C-ABI library.

Python mirror of the reference's public Julia API (package ``NNop`` v0.2.0):
same function names, argument meanings, keyword defaults and error behaviour,
with the ChainRules ``rrule``s mapped to ``torch.autograd.Function``s.  Torch is
used only for device memory and streams; every computation is a kernel of
``libnnop_b200.so`` (there is no CPU fallback: CPU tensors are rejected).

Layout: a Julia array of size ``(d1, ..., dn)`` (column-major) is the torch
tensor of shape ``(dn, ..., d1)`` (row-major) over the same memory:

=============================  ===============================
Julia (reference)              torch here
=============================  ===============================
q (E, QL, QH, B)               q (B, QH, QL, E)
k, v (E, KL, KH, B)            k, v (B, KH, KL, E)
pair (QH, QL, KL, B)           pair (B, KL, QL, QH)
kpad_mask::Matrix{Bool} (KL,B) kpad_mask (B, KL) bool / uint8
x (N, cols) [online_softmax]   x (cols, N)
x (emb, n) [norms]             x (n, emb)
cos, sin (E, L, B)             cos, sin (B, L, E) float32
position_ids (L, B)            position_ids (B, L) float32
=============================  ===============================
"""
from __future__ import annotations

import torch

from ._lib import (BF16, F16, F32, NNopError, NNopShapeError, check, lib)

__all__ = [
    "flash_attention", "_flash_attention", "grad_flash_attention",
    "flash_attention_pair_per_head", "_flash_attention_pair_per_head", "grad_flash_attention_pair_per_head",
    "flash_attention_rope", "_flash_attention_rope", "grad_flash_attention_rope",
    "online_softmax", "grad_online_softmax",
    "rms_norm", "_rms_norm", "grad_rms_norm",
    "add_rms_norm", "_add_rms_norm", "grad_add_rms_norm",
    "layer_norm", "_layer_norm", "grad_layer_norm",
    "llama_rope", "grad_llama_rope", "LlamaRotaryEmbedding",
    "within_gradient", "NNopError", "NNopShapeError", "lib",
]

_DT = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}


def _dtype_id(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise NNopError(-2, f"unsupported dtype {t.dtype} (float32, float16, bfloat16)") from None


def _dev(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise NNopError(-3, "nnop operates on CUDA tensors only (no CPU fallback)")
    return ts[0].device


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _contig(t):
    return None if t is None else t.contiguous()


def within_gradient(x) -> bool:
    """``within_gradient`` (src/attention_crc.jl:1-2): true while autograd is
    recording through ``x``."""
    return torch.is_grad_enabled() and isinstance(x, torch.Tensor) and x.requires_grad


# =========================================================================
# flash attention   (src/attention.jl, src/attention_bwd.jl, src/attention_crc.jl)
# =========================================================================

def _mask_u8(kpad_mask):
    if kpad_mask is None:
        return None
    m = kpad_mask
    if m.dtype == torch.bool:
        m = m.view(torch.uint8) if m.is_contiguous() else m.contiguous().view(torch.uint8)
    elif m.dtype != torch.uint8:
        m = (m != 0).to(torch.uint8)
    return m.contiguous()


def _fa_dims(q, k, v, pair, kpad_mask):
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise NNopShapeError(-1, "q, k, v must be 4-d (B, H, L, E)")
    B, QH, QL, QE = q.shape
    KB, KH, KL, KE = k.shape
    if QE != KE:
        raise NNopShapeError(-1, f"Embedding dim of Q `{QE}` must be the same as of K `{KE}`.")
    if tuple(k.shape) != tuple(v.shape):
        raise NNopShapeError(-1, f"Shapes of K `{tuple(k.shape)}` and V `{tuple(v.shape)}` must be the same.")
    if KB != B:
        raise NNopShapeError(-1, f"Batch of K `{KB}` must equal batch of Q `{B}`.")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise NNopError(-2, "q, k, v must share a dtype")
    if pair is not None:
        if tuple(pair.shape) != (B, KL, QL, QH):
            raise NNopShapeError(-1, f"pair must have shape (B, KL, QL, QH) = {(B, KL, QL, QH)}, got {tuple(pair.shape)}")
        if pair.dtype != q.dtype:
            raise NNopError(-2, "pair must have the dtype of q")
    if kpad_mask is not None and tuple(kpad_mask.shape) != (B, KL):
        raise NNopShapeError(-1, f"kpad_mask must have shape (B, KL) = {(B, KL)}")
    return B, QH, QL, QE, KH, KL


def _flash_attention(q, k, v, pair=None, *, causal: bool, kpad_mask=None):
    """Forward returning ``(o, lse)`` (``_flash_attention``, src/attention.jl:145-197,
    which returns ``(o, ms, ls)``; here ``lse = ms + log(ls)`` in float32)."""
    o, lse, _ = _flash_attention_ws(q, k, v, pair, causal=causal, kpad_mask=kpad_mask)
    return o, lse


def _flash_attention_ws(q, k, v, pair=None, *, causal: bool, kpad_mask=None):
    """``_flash_attention`` that also returns its workspace (None or a uint8
    tensor holding the per-head pair tiles) for ``grad_flash_attention``'s
    ``fwd_workspace``: the rrule's forward state."""
    dev = _dev(q, k, v, pair, kpad_mask)
    B, QH, QL, E, KH, KL = _fa_dims(q, k, v, pair, kpad_mask)
    q, k, v, pair = _contig(q), _contig(k), _contig(v), _contig(pair)
    m = _mask_u8(kpad_mask)
    o = torch.empty_like(q)
    lse = torch.empty((B, QH, QL), dtype=torch.float32, device=dev)
    dt = _dtype_id(q)
    ws_bytes = lib.nnop_flash_attention_fwd_workspace_size(E, QL, KL, QH, KH, B, int(pair is not None), dt)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
    check(lib.nnop_flash_attention_fwd(
        _ptr(q), _ptr(k), _ptr(v), _ptr(pair), _ptr(m), _ptr(o), _ptr(lse), _ptr(ws), ws_bytes,
        E, QL, KL, QH, KH, B, int(bool(causal)), dt, _stream(dev)))
    return o, lse, ws


def grad_flash_attention(do, o, lse, q, k, v, pair=None, *, causal: bool, kpad_mask=None, fwd_workspace=None):
    """``∇flash_attention`` (src/attention_bwd.jl:213-303): returns
    ``(dq, dk, dv, dpair)``, dpair None when pair is None.  ``fwd_workspace``:
    the workspace ``_flash_attention_ws`` returned for the same inputs; its
    pair tiles are then reused instead of rebuilt."""
    dev = _dev(do, o, lse, q, k, v, pair, kpad_mask)
    B, QH, QL, E, KH, KL = _fa_dims(q, k, v, pair, kpad_mask)
    do, o, q, k, v, pair = map(_contig, (do, o, q, k, v, pair))
    if do.dtype != q.dtype:
        do = do.to(q.dtype)
    lse = lse.contiguous()
    m = _mask_u8(kpad_mask)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dpair = torch.empty_like(pair) if pair is not None else None
    dt = _dtype_id(q)
    fw_bytes = 0 if fwd_workspace is None else fwd_workspace.numel()
    ws_bytes = lib.nnop_flash_attention_bwd_workspace_size_reuse(E, QL, KL, QH, KH, B, int(pair is not None),
                                                                  fw_bytes, dt)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    check(lib.nnop_flash_attention_bwd_reuse(
        _ptr(do), _ptr(o), _ptr(lse), _ptr(q), _ptr(k), _ptr(v), _ptr(pair), _ptr(m),
        _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dpair), _ptr(fwd_workspace), fw_bytes, _ptr(ws), ws_bytes,
        E, QL, KL, QH, KH, B, int(bool(causal)), dt, _stream(dev)))
    return dq, dk, dv, dpair


class _FlashAttentionFn(torch.autograd.Function):
    """``CRC.rrule(::typeof(_flash_attention), ...)`` (src/attention_crc.jl:16-31)."""

    @staticmethod
    def forward(ctx, q, k, v, pair, kpad_mask, causal):
        o, lse, ws = _flash_attention_ws(q, k, v, pair, causal=causal, kpad_mask=kpad_mask)
        ctx.save_for_backward(o, lse, q, k, v, pair, kpad_mask, ws)
        ctx.causal = causal
        return o

    @staticmethod
    def backward(ctx, do):
        o, lse, q, k, v, pair, kpad_mask, ws = ctx.saved_tensors
        dq, dk, dv, dpair = grad_flash_attention(do, o, lse, q, k, v, pair, causal=ctx.causal,
                                                 kpad_mask=kpad_mask, fwd_workspace=ws)
        return dq, dk, dv, dpair, None, None


def flash_attention(q, k, v, pair=None, *, causal: bool, kpad_mask=None):
    """``NNop.flash_attention(q, k, v, pair=nothing; causal, kpad_mask=nothing)``
    (src/attention_crc.jl:4-14): returns ``o``; differentiable w.r.t. q, k, v,
    pair when autograd records."""
    if any(within_gradient(t) for t in (q, k, v, pair)):
        return _FlashAttentionFn.apply(q, k, v, pair, kpad_mask, bool(causal))
    return _flash_attention(q, k, v, pair, causal=causal, kpad_mask=kpad_mask)[0]


# -------------------------------------------------------------------------
# pair bias laid out per head: Julia (QL, KL, QH, B) = torch (B, QH, KL, QL)
# -------------------------------------------------------------------------

def _per_head_dims(q, k, v, pair, kpad_mask):
    if pair is None:
        raise NNopError(-3, "the per-head entry points take a pair bias")
    if pair.dim() != 4:
        raise NNopShapeError(-1, "pair must be 4-d (B, QH, KL, QL)")
    B, QH, QL, E, KH, KL = _fa_dims(q, k, v, None, kpad_mask)
    if tuple(pair.shape) != (B, QH, KL, QL):
        raise NNopShapeError(-1, f"pair must have shape (B, QH, KL, QL) = {(B, QH, KL, QL)}, got {tuple(pair.shape)}")
    if pair.dtype != q.dtype:
        raise NNopError(-2, "pair must have the dtype of q")
    return B, QH, QL, E, KH, KL


def _flash_attention_pair_per_head(q, k, v, pair, *, causal: bool, kpad_mask=None):
    """``_flash_attention`` with the pair bias laid out per head, torch shape
    (B, QH, KL, QL) (Julia (QL, KL, QH, B)), read in place by the tensor-core
    kernel (no re-layout pass, no workspace).  bf16/f16, E = 64, QL % 8 == 0;
    −Inf bias entries only at keys ``kpad_mask`` removes.  Returns ``(o, lse)``."""
    dev = _dev(q, k, v, pair, kpad_mask)
    B, QH, QL, E, KH, KL = _per_head_dims(q, k, v, pair, kpad_mask)
    q, k, v, pair = _contig(q), _contig(k), _contig(v), _contig(pair)
    m = _mask_u8(kpad_mask)
    o = torch.empty_like(q)
    lse = torch.empty((B, QH, QL), dtype=torch.float32, device=dev)
    check(lib.nnop_flash_attention_fwd_pair_per_head(
        _ptr(q), _ptr(k), _ptr(v), _ptr(pair), _ptr(m), _ptr(o), _ptr(lse),
        E, QL, KL, QH, KH, B, int(bool(causal)), _dtype_id(q), _stream(dev)))
    return o, lse


def grad_flash_attention_pair_per_head(do, o, lse, q, k, v, pair, *, causal: bool, kpad_mask=None):
    """``∇flash_attention`` with pair and dpair laid out per head (B, QH, KL, QL):
    returns ``(dq, dk, dv, dpair)``; dS is stored straight into dpair."""
    dev = _dev(do, o, lse, q, k, v, pair, kpad_mask)
    B, QH, QL, E, KH, KL = _per_head_dims(q, k, v, pair, kpad_mask)
    do, o, q, k, v, pair = map(_contig, (do, o, q, k, v, pair))
    if do.dtype != q.dtype:
        do = do.to(q.dtype)
    lse = lse.contiguous()
    m = _mask_u8(kpad_mask)
    dq, dk, dv, dpair = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty_like(pair)
    dt = _dtype_id(q)
    ws_bytes = lib.nnop_flash_attention_bwd_pair_per_head_workspace_size(E, QL, KL, QH, KH, B, dt)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    check(lib.nnop_flash_attention_bwd_pair_per_head(
        _ptr(do), _ptr(o), _ptr(lse), _ptr(q), _ptr(k), _ptr(v), _ptr(pair), _ptr(m),
        _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dpair), _ptr(ws), ws_bytes,
        E, QL, KL, QH, KH, B, int(bool(causal)), dt, _stream(dev)))
    return dq, dk, dv, dpair


class _FlashAttentionPerHeadFn(torch.autograd.Function):
    """The rrule of ``flash_attention_pair_per_head`` (the structure of
    src/attention_crc.jl:16-31 with the per-head pair layout)."""

    @staticmethod
    def forward(ctx, q, k, v, pair, kpad_mask, causal):
        o, lse = _flash_attention_pair_per_head(q, k, v, pair, causal=causal, kpad_mask=kpad_mask)
        ctx.save_for_backward(o, lse, q, k, v, pair, kpad_mask)
        ctx.causal = causal
        return o

    @staticmethod
    def backward(ctx, do):
        o, lse, q, k, v, pair, kpad_mask = ctx.saved_tensors
        dq, dk, dv, dpair = grad_flash_attention_pair_per_head(do, o, lse, q, k, v, pair, causal=ctx.causal,
                                                               kpad_mask=kpad_mask)
        return dq, dk, dv, dpair, None, None


def flash_attention_pair_per_head(q, k, v, pair, *, causal: bool, kpad_mask=None):
    """``flash_attention`` with the pair bias laid out per head, torch shape
    (B, QH, KL, QL) (Julia (QL, KL, QH, B)); differentiable w.r.t. q, k, v,
    pair.  Same results as ``flash_attention(q, k, v, pair.permute(0, 2, 3, 1))``."""
    if any(within_gradient(t) for t in (q, k, v, pair)):
        return _FlashAttentionPerHeadFn.apply(q, k, v, pair, kpad_mask, bool(causal))
    return _flash_attention_pair_per_head(q, k, v, pair, causal=causal, kpad_mask=kpad_mask)[0]


# -------------------------------------------------------------------------
# Llama RoPE fused with attention: flash_attention(llama_rope(q, k)...)
# -------------------------------------------------------------------------

def _rope_tables(cos, sin, B, L, E):
    cos = cos.contiguous().to(torch.float32)
    sin = sin.contiguous().to(torch.float32)
    if cos.dim() == 2:
        cos, sin = cos[None], sin[None]
    if cos.shape != sin.shape or cos.shape[1] != L or cos.shape[2] != E or cos.shape[0] not in (1, B):
        raise NNopShapeError(-1, "cos/sin must have shape (B or 1, L, E)")
    return cos, sin


def _flash_attention_rope(q, k, v, *, cos, sin, causal: bool, kpad_mask=None):
    """``llama_rope`` then ``_flash_attention`` in one call: returns
    ``(o, lse, q_rot, k_rot)``; the rotated q and k are the backward's inputs.
    bf16/f16, E = 64 or 128, q and k of one length L."""
    dev = _dev(q, k, v, cos, sin, kpad_mask)
    B, QH, QL, E, KH, KL = _fa_dims(q, k, v, None, kpad_mask)
    if QL != KL:
        raise NNopShapeError(-1, "q and k must share the sequence length")
    cos, sin = _rope_tables(cos, sin, B, QL, E)
    q, k, v = _contig(q), _contig(k), _contig(v)
    m = _mask_u8(kpad_mask)
    qr, kr, o = torch.empty_like(q), torch.empty_like(k), torch.empty_like(q)
    lse = torch.empty((B, QH, QL), dtype=torch.float32, device=dev)
    check(lib.nnop_flash_attention_rope_fwd(
        _ptr(q), _ptr(k), _ptr(v), _ptr(cos), _ptr(sin), _ptr(m), _ptr(qr), _ptr(kr), _ptr(o), _ptr(lse),
        E, QL, QH, KH, B, cos.shape[0], int(bool(causal)), _dtype_id(q), _stream(dev)))
    return o, lse, qr, kr


def grad_flash_attention_rope(do, o, lse, q_rot, k_rot, v, *, cos, sin, causal: bool, kpad_mask=None):
    """Backward of ``_flash_attention_rope``: ``(dq, dk, dv)`` with dq, dk the
    gradients of the UN-rotated q and k (``∇llama_rope`` folded into the
    attention backward's outputs)."""
    dev = _dev(do, o, lse, q_rot, k_rot, v, cos, sin, kpad_mask)
    B, QH, L, E, KH, _ = _fa_dims(q_rot, k_rot, v, None, kpad_mask)
    cos, sin = _rope_tables(cos, sin, B, L, E)
    do, o, q_rot, k_rot, v = map(_contig, (do, o, q_rot, k_rot, v))
    if do.dtype != q_rot.dtype:
        do = do.to(q_rot.dtype)
    m = _mask_u8(kpad_mask)
    dq, dk, dv = torch.empty_like(q_rot), torch.empty_like(k_rot), torch.empty_like(v)
    dt = _dtype_id(q_rot)
    ws_bytes = lib.nnop_flash_attention_rope_bwd_workspace_size(E, L, QH, KH, B, dt)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    check(lib.nnop_flash_attention_rope_bwd(
        _ptr(do), _ptr(o), _ptr(lse.contiguous()), _ptr(q_rot), _ptr(k_rot), _ptr(v), _ptr(cos), _ptr(sin), _ptr(m),
        _ptr(dq), _ptr(dk), _ptr(dv), _ptr(ws), ws_bytes, E, L, QH, KH, B, cos.shape[0], int(bool(causal)), dt,
        _stream(dev)))
    return dq, dk, dv


class _FlashAttentionRopeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, cos, sin, kpad_mask, causal):
        o, lse, qr, kr = _flash_attention_rope(q, k, v, cos=cos, sin=sin, causal=causal, kpad_mask=kpad_mask)
        ctx.save_for_backward(o, lse, qr, kr, v, cos, sin, kpad_mask)
        ctx.causal = causal
        return o

    @staticmethod
    def backward(ctx, do):
        o, lse, qr, kr, v, cos, sin, kpad_mask = ctx.saved_tensors
        dq, dk, dv = grad_flash_attention_rope(do, o, lse, qr, kr, v, cos=cos, sin=sin, causal=ctx.causal,
                                               kpad_mask=kpad_mask)
        return dq, dk, dv, None, None, None, None


def flash_attention_rope(q, k, v, *, cos, sin, causal: bool, kpad_mask=None):
    """``flash_attention(llama_rope(q, k; cos, sin)..., v)`` with the RoPE
    backward folded into the attention backward; differentiable w.r.t. the
    un-rotated q, k and v."""
    if any(within_gradient(t) for t in (q, k, v)):
        return _FlashAttentionRopeFn.apply(q, k, v, cos, sin, kpad_mask, bool(causal))
    return _flash_attention_rope(q, k, v, cos=cos, sin=sin, causal=causal, kpad_mask=kpad_mask)[0]


# =========================================================================
# online softmax   (src/softmax.jl)
# =========================================================================

def _softmax_fwd(x):
    dev = _dev(x)
    x = x.contiguous()
    n = x.shape[-1]
    cols = x.numel() // n if n else 0
    y = torch.empty_like(x)
    check(lib.nnop_online_softmax_fwd(_ptr(x), _ptr(y), n, cols, _dtype_id(x), _stream(dev)))
    return y


def grad_online_softmax(dy, y):
    """``∇online_softmax`` (src/softmax.jl:70-80): dy∘y − y∘Σ(dy∘y)."""
    dev = _dev(dy, y)
    y = y.contiguous()
    dy = dy.contiguous().to(y.dtype)
    n = y.shape[-1]
    dx = torch.empty_like(y)
    check(lib.nnop_online_softmax_bwd(_ptr(dy), _ptr(y), _ptr(dx), n, y.numel() // n, _dtype_id(y),
                                      _stream(dev)))
    return dx


class _SoftmaxFn(torch.autograd.Function):
    """``CRC.rrule(::typeof(online_softmax), x)`` (src/softmax.jl:82-86)."""

    @staticmethod
    def forward(ctx, x):
        y = _softmax_fwd(x)
        ctx.save_for_backward(y)
        return y

    @staticmethod
    def backward(ctx, dy):
        (y,) = ctx.saved_tensors
        return grad_online_softmax(dy, y)


def online_softmax(x):
    """``NNop.online_softmax(x)`` (src/softmax.jl:60-68): softmax over the
    contiguous axis (Julia dims=1)."""
    if within_gradient(x):
        return _SoftmaxFn.apply(x)
    return _softmax_fwd(x)


# =========================================================================
# RMSNorm   (src/rms_norm.jl)
# =========================================================================

def _norm_dims(x, w):
    emb = x.shape[-1]
    if w.numel() != emb:
        raise NNopShapeError(-1, f"weight length {w.numel()} must equal emb {emb}")
    return emb, x.numel() // emb if emb else 0


def _rms_norm(x, w, *, eps: float = 1e-6, offset: float = 0.0):
    """``_rms_norm`` (src/rms_norm.jl:117-137): returns ``(y, rstd)``."""
    dev = _dev(x, w)
    x = x.contiguous()
    w = w.contiguous().to(x.dtype)
    emb, n = _norm_dims(x, w)
    y = torch.empty_like(x)
    rstd = torch.empty(x.shape[:-1], dtype=torch.float32, device=dev)
    check(lib.nnop_rms_norm_fwd(_ptr(x), _ptr(w), _ptr(y), _ptr(rstd), emb, n, float(eps), float(offset),
                                _dtype_id(x), _stream(dev)))
    return y, rstd


def grad_rms_norm(dy, rstd, x, w, *, offset: float = 0.0):
    """``∇rms_norm`` (src/rms_norm.jl:139-169): returns ``(dx, dw)``, dw float32."""
    dev = _dev(dy, rstd, x, w)
    x = x.contiguous()
    w = w.contiguous().to(x.dtype)
    dy = dy.contiguous().to(x.dtype)
    emb, n = _norm_dims(x, w)
    dx = torch.empty_like(x)
    dw = torch.empty(emb, dtype=torch.float32, device=dev)
    ws_bytes = lib.nnop_rms_norm_bwd_workspace_size(emb, n)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    check(lib.nnop_rms_norm_bwd(_ptr(dy), _ptr(x), _ptr(w), _ptr(rstd.contiguous()), _ptr(dx), _ptr(dw),
                                _ptr(ws), ws_bytes, emb, n, float(offset), _dtype_id(x), _stream(dev)))
    return dx, dw


class _RmsNormFn(torch.autograd.Function):
    """``CRC.rrule(::typeof(_rms_norm), x, w)`` (src/rms_norm.jl:178-185)."""

    @staticmethod
    def forward(ctx, x, w, eps, offset):
        y, rstd = _rms_norm(x, w, eps=eps, offset=offset)
        ctx.save_for_backward(x, w, rstd)
        ctx.offset = offset
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        dx, dw = grad_rms_norm(dy, rstd, x, w, offset=ctx.offset)
        return dx, dw.to(w.dtype).reshape(w.shape), None, None


def rms_norm(x, w, *, eps: float = 1e-6, offset: float = 0.0):
    """``NNop.rms_norm(x, w; ϵ=1f-6, offset=0f0)`` (src/rms_norm.jl:171-176)."""
    if within_gradient(x) or within_gradient(w):
        return _RmsNormFn.apply(x, w, float(eps), float(offset))
    return _rms_norm(x, w, eps=eps, offset=offset)[0]


# -------------------------------------------------------------------------
# residual add fused into RMSNorm (the composition a transformer block makes
# around rms_norm; no counterpart in the reference's API)
# -------------------------------------------------------------------------

def _add_rms_norm(x, residual, w, *, eps: float = 1e-6, offset: float = 0.0):
    """``h = x + residual`` (rounded to the dtype) and ``rms_norm(h, w)`` in one
    pass: returns ``(y, h, rstd)``."""
    dev = _dev(x, residual, w)
    if residual.shape != x.shape or residual.dtype != x.dtype:
        raise NNopShapeError(-1, "residual must have the shape and dtype of x")
    x, residual = x.contiguous(), residual.contiguous()
    w = w.contiguous().to(x.dtype)
    emb, n = _norm_dims(x, w)
    h, y = torch.empty_like(x), torch.empty_like(x)
    rstd = torch.empty(x.shape[:-1], dtype=torch.float32, device=dev)
    check(lib.nnop_add_rms_norm_fwd(_ptr(x), _ptr(residual), _ptr(w), _ptr(h), _ptr(y), _ptr(rstd), emb, n,
                                    float(eps), float(offset), _dtype_id(x), _stream(dev)))
    return y, h, rstd


def grad_add_rms_norm(dy, dh, h, w, rstd, *, offset: float = 0.0):
    """Backward of ``_add_rms_norm``: ``dx = ∇rms_norm(dy, h) + dh`` (dh, the
    gradient reaching h from the residual stream, may be None) -- the gradient
    of both x and residual -- and ``dw`` (float32)."""
    dev = _dev(dy, h, w, rstd)
    h = h.contiguous()
    w = w.contiguous().to(h.dtype)
    dy = dy.contiguous().to(h.dtype)
    if dh is not None:
        dh = dh.contiguous().to(h.dtype)
    emb, n = _norm_dims(h, w)
    dx = torch.empty_like(h)
    dw = torch.empty(emb, dtype=torch.float32, device=dev)
    ws_bytes = lib.nnop_add_rms_norm_bwd_workspace_size(emb, n)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    check(lib.nnop_add_rms_norm_bwd(_ptr(dy), _ptr(dh), _ptr(h), _ptr(w), _ptr(rstd.contiguous()), _ptr(dx),
                                    _ptr(dw), _ptr(ws), ws_bytes, emb, n, float(offset), _dtype_id(h), _stream(dev)))
    return dx, dw


class _AddRmsNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, residual, w, eps, offset):
        y, h, rstd = _add_rms_norm(x, residual, w, eps=eps, offset=offset)
        ctx.save_for_backward(h, w, rstd)
        ctx.offset = offset
        return y, h

    @staticmethod
    def backward(ctx, dy, dh):
        h, w, rstd = ctx.saved_tensors
        if dy is None:
            dy = torch.zeros_like(h)
        dx, dw = grad_add_rms_norm(dy, dh, h, w, rstd, offset=ctx.offset)
        return dx, dx, dw.to(w.dtype).reshape(w.shape), None, None


def add_rms_norm(x, residual, w, *, eps: float = 1e-6, offset: float = 0.0):
    """Residual add and ``rms_norm`` fused: returns ``(y, h)`` with
    ``h = x + residual`` (the new residual stream) and ``y = rms_norm(h, w)``;
    differentiable w.r.t. x, residual and w."""
    if any(within_gradient(t) for t in (x, residual, w)):
        return _AddRmsNormFn.apply(x, residual, w, float(eps), float(offset))
    y, h, _ = _add_rms_norm(x, residual, w, eps=eps, offset=offset)
    return y, h


# =========================================================================
# LayerNorm   (src/layer_norm.jl)
# =========================================================================

def _layer_norm(x, w, b, *, eps: float = 1e-6):
    """``_layer_norm`` (src/layer_norm.jl:150-170): returns ``(y, mean, rstd)``."""
    dev = _dev(x, w, b)
    x = x.contiguous()
    w = w.contiguous().to(x.dtype)
    b = b.contiguous().to(x.dtype)
    emb, n = _norm_dims(x, w)
    if b.numel() != emb:
        raise NNopShapeError(-1, f"bias length {b.numel()} must equal emb {emb}")
    y = torch.empty_like(x)
    mean = torch.empty(x.shape[:-1], dtype=torch.float32, device=dev)
    rstd = torch.empty(x.shape[:-1], dtype=torch.float32, device=dev)
    check(lib.nnop_layer_norm_fwd(_ptr(x), _ptr(w), _ptr(b), _ptr(y), _ptr(mean), _ptr(rstd), emb, n,
                                  float(eps), _dtype_id(x), _stream(dev)))
    return y, mean, rstd


def grad_layer_norm(dy, mean, rstd, x, w, b=None):
    """``∇layer_norm`` (src/layer_norm.jl:172-204): returns ``(dx, dw, db)`` in
    the dtype of x."""
    dev = _dev(dy, mean, rstd, x, w)
    x = x.contiguous()
    w = w.contiguous().to(x.dtype)
    dy = dy.contiguous().to(x.dtype)
    emb, n = _norm_dims(x, w)
    dx = torch.empty_like(x)
    dw = torch.empty(emb, dtype=x.dtype, device=dev)
    db = torch.empty(emb, dtype=x.dtype, device=dev)
    ws_bytes = lib.nnop_layer_norm_bwd_workspace_size(emb, n)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    check(lib.nnop_layer_norm_bwd(_ptr(dy), _ptr(x), _ptr(w), _ptr(mean.contiguous()), _ptr(rstd.contiguous()),
                                  _ptr(dx), _ptr(dw), _ptr(db), _ptr(ws), ws_bytes, emb, n, _dtype_id(x),
                                  _stream(dev)))
    return dx, dw, db


class _LayerNormFn(torch.autograd.Function):
    """``CRC.rrule(::typeof(_layer_norm), x, w, b)`` (src/layer_norm.jl:213-220)."""

    @staticmethod
    def forward(ctx, x, w, b, eps):
        y, mean, rstd = _layer_norm(x, w, b, eps=eps)
        ctx.save_for_backward(x, w, mean, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, mean, rstd = ctx.saved_tensors
        dx, dw, db = grad_layer_norm(dy, mean, rstd, x, w)
        return dx, dw.to(w.dtype).reshape(w.shape), db.to(w.dtype).reshape(w.shape), None


def layer_norm(x, w, b, *, eps: float = 1e-6):
    """``NNop.layer_norm(x, w, b; ϵ=1f-6)`` (src/layer_norm.jl:206-211)."""
    if any(within_gradient(t) for t in (x, w, b)):
        return _LayerNormFn.apply(x, w, b, float(eps))
    return _layer_norm(x, w, b, eps=eps)[0]


# =========================================================================
# Llama RoPE   (src/rope/llama_rope.jl)
# =========================================================================

class LlamaRotaryEmbedding:
    """``LlamaRotaryEmbedding(dim; base=10000)`` (src/rope/llama_rope.jl:1-22).

    ``emb(position_ids)`` with position_ids (B, L) float32 returns ``(cos, sin)``
    of shape (B, L, dim) float32, computed on the device."""

    def __init__(self, dim: int, *, base: int = 10000):
        if dim <= 0 or dim % 2:
            raise NNopShapeError(-1, "dim must be even and > 0")
        self.dim = int(dim)
        self.base = int(base)

    def __call__(self, position_ids):
        pos = position_ids
        if not isinstance(pos, torch.Tensor):
            pos = torch.as_tensor(pos)
        if not pos.is_cuda:
            pos = pos.cuda()
        pos = pos.to(torch.float32).contiguous()
        if pos.dim() == 1:
            pos = pos[None]
        B, L = pos.shape
        cos = torch.empty((B, L, self.dim), dtype=torch.float32, device=pos.device)
        sin = torch.empty_like(cos)
        check(lib.nnop_llama_rope_cos_sin(_ptr(pos), _ptr(cos), _ptr(sin), self.dim, L, B, self.base,
                                          _stream(pos.device)))
        return cos, sin


def _llama_rope(q, k, cos, sin, *, bwd: bool):
    dev = _dev(q, k, cos, sin)
    if q.dim() != 4 or k.dim() != 4:
        raise NNopShapeError(-1, "q, k must be 4-d (B, H, L, E)")
    B, QH, L, E = q.shape
    if k.shape[0] != B or k.shape[2] != L or k.shape[3] != E:
        raise NNopShapeError(-1, "q and k must share batch, sequence length and embedding dim")
    KH = k.shape[1]
    cos = cos.contiguous().to(torch.float32)
    sin = sin.contiguous().to(torch.float32)
    if cos.dim() == 2:
        cos, sin = cos[None], sin[None]
    if cos.shape != sin.shape or cos.shape[1] != L or cos.shape[2] != E:
        raise NNopShapeError(-1, "cos/sin must have shape (B or 1, L, E)")
    q, k = q.contiguous(), k.contiguous()
    qo, ko = torch.empty_like(q), torch.empty_like(k)
    check(lib.nnop_llama_rope(_ptr(q), _ptr(k), _ptr(cos), _ptr(sin), _ptr(qo), _ptr(ko), E, L, QH, KH, B,
                              cos.shape[0], -1.0 if bwd else 1.0, _dtype_id(q), _stream(dev)))
    return qo, ko


def grad_llama_rope(dq, dk, *, cos, sin):
    """``∇llama_rope`` (src/rope/llama_rope.jl:92): the rotation with sin → −sin."""
    return _llama_rope(dq, dk, cos, sin, bwd=True)


class _RopeFn(torch.autograd.Function):
    """``CRC.rrule(::typeof(llama_rope), q, k; cos, sin)`` (src/rope/llama_rope.jl:94-98)."""

    @staticmethod
    def forward(ctx, q, k, cos, sin):
        ctx.save_for_backward(cos, sin)
        return _llama_rope(q, k, cos, sin, bwd=False)

    @staticmethod
    def backward(ctx, dq, dk):
        cos, sin = ctx.saved_tensors
        dq = torch.zeros_like(dq) if dq is None else dq
        dk = torch.zeros_like(dk) if dk is None else dk
        gq, gk = _llama_rope(dq, dk, cos, sin, bwd=True)
        return gq, gk, None, None


def llama_rope(q, k, *, cos, sin):
    """``NNop.llama_rope(q, k; cos, sin)`` (src/rope/llama_rope.jl:91): returns
    rotated copies ``(q, k)``."""
    if within_gradient(q) or within_gradient(k):
        return _RopeFn.apply(q, k, cos, sin)
    return _llama_rope(q, k, cos, sin, bwd=False)
