"""CPU oracle for the NNop fused-kernel hot path (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it.  The product path (``onionop.jl_b200/nnop``) never calls it and fails
loudly when the CUDA library is missing.

What it restates
----------------
The reference package (Julia ``NNop`` v0.2.0) is tested against naive dense
implementations that live in its test suite.  This file restates those naive
functions in numpy, in float64, on inputs already rounded to the kernel dtype:

* attention forward  -- ``test/attention_testsetup.jl:21-45`` (``naive_attention``)
  with the key-padding term ``log(mask)`` of ``test/attention_testsetup.jl:16-19``
  and GQA expansion ``d l h -> d l (num_q_per_kv h)`` (``:24-30``);
  the attention scale is ``T(1/sqrt(E))`` as in ``src/attention.jl:166``.
* attention backward -- the closed-form rules the reference kernel implements
  (``src/attention_bwd.jl:87-169``): P = softmax(S), dV = Pᵀ dO,
  dP = dO Vᵀ, dS = P ∘ (dP − rowsum(dO ∘ O)), dpair = dS, dQ = scale·dS K,
  dK = scale·dSᵀ Q (GQA: summed over the query heads that share a KV head).
  Zygote's gradient of ``sum(naive_attention(...))`` (the reference tests,
  ``test/attention_tests.jl:33-46``) is the same quantity.
* online softmax     -- ``test/softmax_tests.jl:6-10``; backward
  ``src/softmax.jl:70-80``.
* rms_norm           -- ``test/rmsnorm_tests.jl:7-9``; backward
  ``src/rms_norm.jl:43-115``.
* layer_norm         -- ``test/layernorm_tests.jl:7-11``; backward
  ``src/layer_norm.jl:97-137``.
* llama_rope         -- the kernel ``src/rope/llama_rope.jl:24-65`` (which uses
  cos/sin of the first half of the embedding for both halves) and
  ``LlamaRotaryEmbedding`` ``src/rope/llama_rope.jl:7-22``.

Array layout
------------
Julia arrays are column-major.  A Julia array of size ``(d1, d2, ..., dn)`` has
the same memory as a row-major (numpy / torch) array of shape
``(dn, ..., d2, d1)``.  Every function here takes the row-major view:

==================  ======================  ==========================
Julia (reference)   numpy here              meaning
==================  ======================  ==========================
q (E, QL, QH, B)    q (B, QH, QL, E)        queries
k, v (E, KL, KH, B) k, v (B, KH, KL, E)     keys / values
pair (H, QL, KL, B) pair (B, KL, QL, H)     additive pair-feature bias
kpad_mask (KL, B)   kpad_mask (B, KL) bool  key-padding mask (true = keep)
x (N, cols)         x (cols, N)             softmax input, reduced over N
x (emb, n)          x (n, emb)              norm input, normalised over emb
cos, sin (E, L, B)  cos, sin (B, L, E)      RoPE tables
==================  ======================  ==========================

Parity status
-------------
parity unpinned: the reference cannot be executed here (Julia is absent and
every NNop kernel is declared ``cpu=false``), and its test suite holds no golden
vectors -- inputs are unseeded ``randn``/``rand`` compared against the naive
functions restated above.  The restatement is cross-checked instead against
(a) torch float64 autograd of the same naive forward (the role Zygote plays in
the reference tests) and (b) the one known-answer case the reference tests
hold: RoPE on ``q = k = ones`` (``test/rope_tests.jl:38-44``).  Fixtures under
``tests/golden/`` freeze the oracle's outputs at fixed seeds.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "attention_scale", "round_to", "attention_fwd", "attention_bwd",
    "softmax_fwd", "softmax_bwd", "rms_norm_fwd", "rms_norm_bwd",
    "layer_norm_fwd", "layer_norm_bwd", "rope_fwd", "rope_bwd",
    "add_rms_norm_fwd", "add_rms_norm_bwd",
    "llama_rotary_embedding", "rel_err", "max_abs_err",
]


# ---------------------------------------------------------------------------
# dtype helpers
# ---------------------------------------------------------------------------

def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float values to ``dtype`` ("f32", "f16", "bf16") and return them
    as float64.  bf16 uses round-to-nearest-even on the float32 bit pattern."""
    x = np.asarray(x)
    if dtype == "f32":
        return x.astype(np.float32).astype(np.float64)
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float64)
    if dtype == "bf16":
        f = np.ascontiguousarray(x, dtype=np.float32)
        u = f.view(np.uint32).astype(np.uint64)
        nan = np.isnan(f)
        rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
        out = rounded.astype(np.uint32).view(np.float32).astype(np.float64)
        out[nan] = np.nan
        return out
    raise ValueError(f"unknown dtype {dtype}")


def attention_scale(E: int, dtype: str) -> float:
    """``scale = T(inv(sqrt(QE)))`` -- the scale rounded to the kernel dtype
    (``src/attention.jl:166``, ``src/attention_bwd.jl:235``)."""
    return float(round_to(np.array([1.0 / np.sqrt(E)]), dtype)[0])


def rel_err(a: np.ndarray, b: np.ndarray) -> float:
    """Norm-relative error ``‖a−b‖ / max(‖a‖, ‖b‖)`` -- Julia's array
    ``isapprox`` criterion used by every reference test
    (e.g. ``test/attention_tests.jl:41``)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    d = np.linalg.norm((a - b).ravel())
    s = max(np.linalg.norm(a.ravel()), np.linalg.norm(b.ravel()))
    return float(d / s) if s > 0 else float(d)


def max_abs_err(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b))) if a.size else 0.0


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------

def _expand_kv(x: np.ndarray, n_rep: int) -> np.ndarray:
    """GQA expansion: query head j (0-based) uses KV head j // n_rep.  This is
    Einops ``d l h -> d l (num_q_per_kv h)`` (``test/attention_testsetup.jl:28``)
    and the kernel's ``cld(q_head_idx, n_q_per_kv)`` (``src/attention.jl:68``)."""
    return np.repeat(x, n_rep, axis=1) if n_rep > 1 else x


def _logits(q, k, pair, causal, kpad_mask, scale):
    B, QH, QL, E = q.shape
    KH, KL = k.shape[1], k.shape[2]
    kk = _expand_kv(k, QH // KH)
    s = np.einsum("bhqe,bhke->bhqk", q, kk, optimize=True) * q.dtype.type(scale)
    if causal:
        # NNlib make_causal_mask: key j is visible to query i iff j <= i
        # (top-left aligned), src/attention.jl:76-81.
        qi = np.arange(QL)[:, None]
        kj = np.arange(KL)[None, :]
        s = np.where(kj <= qi, s, s.dtype.type(-np.inf))
    if kpad_mask is not None:
        # + log(Float(mask)) (test/attention_testsetup.jl:16-19,39)
        with np.errstate(divide="ignore"):
            s = s + np.log(kpad_mask.astype(s.dtype))[:, None, None, :]
    if pair is not None:
        # permutedims(pair, (3,2,1,4)) in Julia; here (B,KL,QL,H)->(B,H,QL,KL)
        s = s + np.transpose(pair, (0, 3, 2, 1))
    return s


def attention_fwd(q, k, v, pair=None, *, causal=False, kpad_mask=None, scale=None,
                  work_dtype=np.float64):
    """Returns ``(o, lse)``: o (B,QH,QL,E), lse (B,QH,QL) = log Σ_j exp(s_ij).

    A row whose keys are all masked yields NaN, exactly as the reference's
    naive softmax of an all ``-Inf`` column does.  ``work_dtype`` float32 is
    used only to time the CPU baseline; parity checks use float64."""
    q = np.asarray(q, work_dtype)
    k = np.asarray(k, work_dtype)
    v = np.asarray(v, work_dtype)
    if pair is not None:
        pair = np.asarray(pair, work_dtype)
    if scale is None:
        scale = 1.0 / np.sqrt(q.shape[-1])
    s = _logits(q, k, pair, causal, kpad_mask, scale)
    with np.errstate(invalid="ignore"):
        m = np.max(s, axis=-1, keepdims=True)
        p = np.exp(s - m)
        l = np.sum(p, axis=-1, keepdims=True)
        p = p / l
        lse = (m + np.log(l))[..., 0]
    vv = _expand_kv(v, q.shape[1] // k.shape[1])
    o = np.einsum("bhqk,bhke->bhqe", p, vv, optimize=True)
    return o, lse


def attention_bwd(do, q, k, v, pair=None, *, causal=False, kpad_mask=None, scale=None,
                  work_dtype=np.float64):
    """Gradients of ``sum(do ∘ attention(q,k,v,pair))``.

    Returns ``(dq, dk, dv, dpair)``; ``dpair`` is None when ``pair`` is None and
    is laid out like ``pair`` (B, KL, QL, H)."""
    q = np.asarray(q, work_dtype)
    k = np.asarray(k, work_dtype)
    v = np.asarray(v, work_dtype)
    do = np.asarray(do, work_dtype)
    if pair is not None:
        pair = np.asarray(pair, work_dtype)
    if scale is None:
        scale = 1.0 / np.sqrt(q.shape[-1])
    B, QH, QL, E = q.shape
    KH = k.shape[1]
    n_rep = QH // KH
    s = _logits(q, k, pair, causal, kpad_mask, scale)
    with np.errstate(invalid="ignore"):
        m = np.max(s, axis=-1, keepdims=True)
        p = np.exp(s - m)
        p = p / np.sum(p, axis=-1, keepdims=True)
    kk = _expand_kv(k, n_rep)
    vv = _expand_kv(v, n_rep)
    o = np.einsum("bhqk,bhke->bhqe", p, vv, optimize=True)
    dp = np.einsum("bhqe,bhke->bhqk", do, vv, optimize=True)
    delta = np.sum(do * o, axis=-1, keepdims=True)
    ds = p * (dp - delta)
    dq = np.einsum("bhqk,bhke->bhqe", ds, kk, optimize=True) * q.dtype.type(scale)
    dk_full = np.einsum("bhqk,bhqe->bhke", ds, q, optimize=True) * q.dtype.type(scale)
    dv_full = np.einsum("bhqk,bhqe->bhke", p, do, optimize=True)
    if n_rep > 1:
        dk = dk_full.reshape(B, KH, n_rep, *dk_full.shape[2:]).sum(axis=2)
        dv = dv_full.reshape(B, KH, n_rep, *dv_full.shape[2:]).sum(axis=2)
    else:
        dk, dv = dk_full, dv_full
    dpair = None if pair is None else np.transpose(ds, (0, 3, 2, 1)).copy()
    return dq, dk, dv, dpair


def attention_flops(B, QH, QL, KL, E, causal):
    """FA2 convention: fwd 4·B·QH·QL·KL·E, bwd 2.5× that, halved when causal."""
    c = 0.5 if causal else 1.0
    fwd = 4.0 * B * QH * QL * KL * E * c
    return fwd, 2.5 * fwd


# ---------------------------------------------------------------------------
# online softmax (reduction over the contiguous last axis)
# ---------------------------------------------------------------------------

def softmax_fwd(x):
    """``naive_softmax(x; dims=1)`` of ``test/softmax_tests.jl:6-10``."""
    x = np.asarray(x, np.float64)
    with np.errstate(invalid="ignore"):
        m = np.max(x, axis=-1, keepdims=True)
        t = np.exp(x - m)
        return t / np.sum(t, axis=-1, keepdims=True)


def softmax_bwd(dy, y):
    """``Δ.*y .- y.*sum(Δ.*y; dims=1)`` (``src/softmax.jl:70-80``)."""
    dy = np.asarray(dy, np.float64)
    y = np.asarray(y, np.float64)
    t = dy * y
    return t - y * np.sum(t, axis=-1, keepdims=True)


# ---------------------------------------------------------------------------
# RMSNorm / LayerNorm (normalised over the contiguous last axis)
# ---------------------------------------------------------------------------

def rms_norm_fwd(x, w, *, eps=1e-6, offset=0.0):
    """``(w .+ offset) .* x ./ sqrt.(mean(x.^2; dims=1) .+ ϵ)``
    (``test/rmsnorm_tests.jl:7-9``).  Returns ``(y, rstd)``."""
    x = np.asarray(x, np.float64)
    w = np.asarray(w, np.float64)
    rstd = 1.0 / np.sqrt(np.mean(x * x, axis=-1) + eps)
    return (w + offset) * x * rstd[:, None], rstd


def rms_norm_bwd(dy, x, w, *, eps=1e-6, offset=0.0):
    """dx = rstd·m − rstd³/N·(Σ m∘x)·x with m = Δ∘(w+offset);
    dw = Σ_rows Δ∘x·rstd (``src/rms_norm.jl:43-115``)."""
    dy = np.asarray(dy, np.float64)
    x = np.asarray(x, np.float64)
    w = np.asarray(w, np.float64)
    N = x.shape[-1]
    rstd = 1.0 / np.sqrt(np.mean(x * x, axis=-1) + eps)
    m = dy * (w + offset)
    dd = np.sum(m * x, axis=-1)
    dx = rstd[:, None] * m - (rstd ** 3 * dd / N)[:, None] * x
    dw = np.sum(dy * x * rstd[:, None], axis=0)
    return dx, dw


def add_rms_norm_fwd(x, residual, w, *, eps=1e-6, offset=0.0, dtype="f32"):
    """Residual add followed by ``rms_norm`` -- the composition a transformer
    block performs around the reference's ``rms_norm`` (src/rms_norm.jl:171):
    h = x + residual, rounded to the tensors' dtype as a separate add would
    store it, then ``rms_norm_fwd(h, w)``.  Returns ``(y, h, rstd)``."""
    h = round_to(np.asarray(x, np.float64) + np.asarray(residual, np.float64), dtype)
    y, rstd = rms_norm_fwd(h, w, eps=eps, offset=offset)
    return y, h, rstd


def add_rms_norm_bwd(dy, dh, h, w, *, eps=1e-6, offset=0.0):
    """Gradients of ``add_rms_norm_fwd``: the gradient reaching h is
    ``rms_norm_bwd(dy, h, w)`` plus ``dh`` (the gradient arriving at h from
    its other use, the residual stream; None = 0); it is the gradient of both
    x and residual.  Returns ``(dx, dw)``."""
    dx, dw = rms_norm_bwd(dy, h, w, eps=eps, offset=offset)
    if dh is not None:
        dx = dx + np.asarray(dh, np.float64)
    return dx, dw


def layer_norm_fwd(x, w, b, *, eps=1e-6):
    """``(x .- μ) ./ sqrt.(σ² .+ ϵ) .* w .+ b`` with the biased variance
    (``test/layernorm_tests.jl:7-11``).  Returns ``(y, mean, rstd)``."""
    x = np.asarray(x, np.float64)
    mu = np.mean(x, axis=-1)
    var = np.mean((x - mu[:, None]) ** 2, axis=-1)
    rstd = 1.0 / np.sqrt(var + eps)
    xn = (x - mu[:, None]) * rstd[:, None]
    return xn * np.asarray(w, np.float64) + np.asarray(b, np.float64), mu, rstd


def layer_norm_bwd(dy, x, w, *, eps=1e-6):
    """c1 = mean(w∘Δ∘xn), c2 = mean(w∘Δ); dx = (w∘Δ − (xn·c1 + c2))·rstd;
    dw = Σ Δ∘xn; db = Σ Δ (``src/layer_norm.jl:97-137``)."""
    dy = np.asarray(dy, np.float64)
    x = np.asarray(x, np.float64)
    w = np.asarray(w, np.float64)
    mu = np.mean(x, axis=-1)
    var = np.mean((x - mu[:, None]) ** 2, axis=-1)
    rstd = 1.0 / np.sqrt(var + eps)
    xn = (x - mu[:, None]) * rstd[:, None]
    wdy = w * dy
    c1 = np.mean(wdy * xn, axis=-1)
    c2 = np.mean(wdy, axis=-1)
    dx = (wdy - (xn * c1[:, None] + c2[:, None])) * rstd[:, None]
    return dx, np.sum(dy * xn, axis=0), np.sum(dy, axis=0)


# ---------------------------------------------------------------------------
# Llama RoPE
# ---------------------------------------------------------------------------

def llama_rotary_embedding(dim: int, position_ids, base: int = 10000):
    """``LlamaRotaryEmbedding(dim; base)(position_ids)``
    (``src/rope/llama_rope.jl:7-22``), evaluated in float32 like Julia.

    position_ids: (B, L) float32.  Returns ``(cos, sin)`` of shape (B, L, dim)
    float32."""
    ids = (np.arange(0, dim, 2, dtype=np.float32) / np.float32(dim)).astype(np.float32)
    inv_freq = (np.float32(1.0) / np.power(np.float32(base), ids)).astype(np.float32)
    pos = np.asarray(position_ids, np.float32)
    freqs = (pos[..., None] * inv_freq).astype(np.float32)
    freqs = np.concatenate([freqs, freqs], axis=-1)
    return np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32)


def _rope(x, cos, sin, sign):
    x = np.asarray(x, np.float64)
    half = x.shape[-1] // 2
    c = np.asarray(cos, np.float64)[..., :half][:, None]   # (B,1,L,half)
    s = np.asarray(sin, np.float64)[..., :half][:, None] * sign
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)


def rope_fwd(q, k, cos, sin):
    """``llama_rope`` (kernel ``src/rope/llama_rope.jl:45-61``): pairs
    (i, i+E/2) are rotated with cos/sin of index i (first half)."""
    return _rope(q, cos, sin, 1.0), _rope(k, cos, sin, 1.0)


def rope_bwd(dq, dk, cos, sin):
    """``∇llama_rope`` = the same kernel with ``sin_sign = -1``
    (``src/rope/llama_rope.jl:86,92``)."""
    return _rope(dq, cos, sin, -1.0), _rope(dk, cos, sin, -1.0)
