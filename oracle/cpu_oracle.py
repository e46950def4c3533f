"""ctypes binding of the C restatement under ``oracle/cpu/`` (TEST
INFRASTRUCTURE ONLY).

Multi-threaded fp32 CPU restatements of NNop's hot path: flash attention
forward and backward (``attention_cpu.c``; ``src/attention.jl:8-143``,
``src/attention_bwd.jl:1-175``) and the memory-bound ops (``memops_cpu.c``;
``src/rms_norm.jl``, ``src/layer_norm.jl``, ``src/softmax.jl``,
``src/rope/llama_rope.jl``).  They are the CPU baselines ``bench.py`` times on
the host cores and second checkers for the tests (checked themselves against
the float64 numpy restatement in ``nnop_oracle.py``).  Only ``tests/``,
``__graft_entry__`` and ``bench.py``'s CPU-baseline / reference arm use them;
the product never does.

Arrays are numpy, row-major views of the reference's column-major arrays (the
same table as ``nnop_oracle``): q (B,QH,QL,E), k, v (B,KH,KL,E),
pair (B,KL,QL,QH), kpad_mask (B,KL) bool; norm and softmax rows are the last
axis; RoPE tables cos, sin (B,L,E).
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
SRC = [HERE / "cpu" / "attention_cpu.c", HERE / "cpu" / "memops_cpu.c", HERE / "cpu" / "attention_cpu_impl.h"]
LIB_PATH = HERE / "_build" / "libnnop_cpu_oracle.so"
CFLAGS = ["-O3", "-std=c11", "-Wall", "-Wextra", "-Wno-psabi", "-fPIC", "-shared", "-pthread", "-fno-math-errno",
          "-fno-trapping-math", "-ffp-contract=fast"]
ISAS = {"auto": 0, "generic": 1, "avx2": 2, "avx512": 3}

_lib = None


def build(force: bool = False) -> pathlib.Path:
    """gcc the C restatement into ``oracle/_build/libnnop_cpu_oracle.so`` (when
    missing or older than its sources).  Raises on a compiler error."""
    if not force and LIB_PATH.exists() and all(LIB_PATH.stat().st_mtime >= s.stat().st_mtime for s in SRC):
        return LIB_PATH
    LIB_PATH.parent.mkdir(exist_ok=True)
    tmp = LIB_PATH.with_suffix(f".{os.getpid()}.tmp")
    cmd = [os.environ.get("CC", "gcc"), *CFLAGS, str(SRC[0]), str(SRC[1]), "-o", str(tmp), "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"building the CPU attention oracle failed:\n{' '.join(cmd)}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(str(build()))
        f, i, p = ctypes.c_float, ctypes.c_int, ctypes.c_void_p
        L.nnop_cpu_attention_fwd.argtypes = [p] * 7 + [i] * 7 + [f, i]
        L.nnop_cpu_attention_fwd.restype = i
        L.nnop_cpu_attention_bwd.argtypes = [p] * 12 + [i] * 7 + [f, i]
        L.nnop_cpu_attention_bwd.restype = i
        lg = ctypes.c_long
        L.nnop_cpu_rms_norm_fwd.argtypes = [p] * 4 + [i, lg, f, f, i]
        L.nnop_cpu_rms_norm_bwd.argtypes = [p] * 6 + [i, lg, f, i]
        L.nnop_cpu_layer_norm_fwd.argtypes = [p] * 6 + [i, lg, f, i]
        L.nnop_cpu_layer_norm_bwd.argtypes = [p] * 8 + [i, lg, i]
        L.nnop_cpu_softmax_fwd.argtypes = [p] * 2 + [i, lg, i]
        L.nnop_cpu_softmax_bwd.argtypes = [p] * 3 + [i, lg, i]
        L.nnop_cpu_llama_rope.argtypes = [p] * 6 + [i] * 5 + [f, i]
        for name in ("rms_norm_fwd", "rms_norm_bwd", "layer_norm_fwd", "layer_norm_bwd", "softmax_fwd",
                     "softmax_bwd", "llama_rope"):
            getattr(L, f"nnop_cpu_{name}").restype = i
        L.nnop_cpu_isa.restype = ctypes.c_char_p
        L.nnop_cpu_force_isa.argtypes = [i]
        L.nnop_cpu_force_isa.restype = i
        _lib = L
    return _lib


def host_threads() -> int:
    """Cores this process may run on (the container's CPU set)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def isa() -> str:
    return lib().nnop_cpu_isa().decode()


def force_isa(name: str) -> str:
    """Use ``name`` ("auto", "generic", "avx2", "avx512") for later calls; a set
    the CPU lacks falls back to the best it has.  Returns the set in use."""
    lib().nnop_cpu_force_isa(ISAS[name])
    return isa()


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a):
    return None if a is None else a.ctypes.data


def _dims(q, k):
    B, QH, QL, E = q.shape
    KH, KL = k.shape[1], k.shape[2]
    return E, QL, KL, QH, KH, B


def _mask(kpad_mask):
    return None if kpad_mask is None else np.ascontiguousarray(kpad_mask, dtype=np.uint8)


def _check_out(arrays, shapes):
    for a, shape in zip(arrays, shapes):
        if (a is None) != (shape is None) or (a is not None and (a.dtype != np.float32 or a.shape != tuple(shape)
                                                                 or not a.flags.c_contiguous)):
            raise ValueError(f"output array must be C-contiguous float32 of shape {shape}")


def _check(rc, what):
    if rc != 0:
        raise ValueError(f"{what}: status {rc} (-1: E must be a multiple of 16 up to 512 and QH a multiple "
                         f"of KH; -3: out of memory or threads)")


def attention_fwd(q, k, v, pair=None, *, causal=False, kpad_mask=None, scale=None, threads=None, out=None):
    """Returns ``(o, lse)`` in float32: o (B,QH,QL,E), lse (B,QH,QL).  ``out``:
    optional ``(o, lse)`` arrays to write into (a timing loop reuses them, so
    first-touch page faults of fresh host memory stay out of the measurement)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    pair = None if pair is None else _f32(pair)
    mask = _mask(kpad_mask)
    E, QL, KL, QH, KH, B = _dims(q, k)
    scale = 1.0 / np.sqrt(E) if scale is None else scale
    o, lse = out if out is not None else (np.empty_like(q), np.empty((B, QH, QL), np.float32))
    _check_out((o, lse), (q.shape, (B, QH, QL)))
    rc = lib().nnop_cpu_attention_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(pair), _ptr(mask), _ptr(o), _ptr(lse),
                                      E, QL, KL, QH, KH, B, int(bool(causal)), float(scale),
                                      int(threads or host_threads()))
    _check(rc, "nnop_cpu_attention_fwd")
    return o, lse


def attention_bwd(do, o, lse, q, k, v, pair=None, *, causal=False, kpad_mask=None, scale=None, threads=None,
                  out=None):
    """Gradients from the saved ``(o, lse)``: ``(dq, dk, dv, dpair)`` in
    float32; dpair is None without a pair bias and laid out like pair.
    ``out``: optional ``(dq, dk, dv, dpair)`` arrays to write into."""
    do, o, lse, q, k, v = (_f32(a) for a in (do, o, lse, q, k, v))
    pair = None if pair is None else _f32(pair)
    mask = _mask(kpad_mask)
    E, QL, KL, QH, KH, B = _dims(q, k)
    scale = 1.0 / np.sqrt(E) if scale is None else scale
    if out is None:
        out = (np.empty_like(q), np.empty_like(k), np.empty_like(v), None if pair is None else np.empty_like(pair))
    dq, dk, dv, dpair = out
    _check_out(out, (q.shape, k.shape, v.shape, None if pair is None else pair.shape))
    rc = lib().nnop_cpu_attention_bwd(_ptr(do), _ptr(o), _ptr(lse), _ptr(q), _ptr(k), _ptr(v), _ptr(pair),
                                      _ptr(mask), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dpair),
                                      E, QL, KL, QH, KH, B, int(bool(causal)), float(scale),
                                      int(threads or host_threads()))
    _check(rc, "nnop_cpu_attention_bwd")
    return dq, dk, dv, dpair


# ------------------------------------------------------------ memory-bound ops
def _rows(x):
    emb = x.shape[-1]
    return emb, x.size // emb if emb else 0


def _thr(threads):
    return int(threads or host_threads())


def _outs(out, shapes):
    """Caller-provided output arrays (a timing loop reuses them) or fresh ones."""
    if out is None:
        return tuple(np.empty(s, np.float32) for s in shapes)
    _check_out(out, shapes)
    return tuple(out)


def rms_norm_fwd(x, w, *, eps=1e-6, offset=0.0, threads=None, out=None):
    """``(y, rstd)`` of RMSNorm over the last axis (src/rms_norm.jl:3-38)."""
    x, w = _f32(x), _f32(w)
    emb, n = _rows(x)
    y, rstd = _outs(out, (x.shape, x.shape[:-1]))
    _check(lib().nnop_cpu_rms_norm_fwd(_ptr(x), _ptr(w), _ptr(y), _ptr(rstd), emb, n, eps, offset, _thr(threads)),
           "nnop_cpu_rms_norm_fwd")
    return y, rstd


def rms_norm_bwd(dy, rstd, x, w, *, offset=0.0, threads=None, out=None):
    """``(dx, dw)`` from the saved rstd (src/rms_norm.jl:43-115)."""
    dy, rstd, x, w = _f32(dy), _f32(rstd), _f32(x), _f32(w)
    emb, n = _rows(x)
    dx, dw = _outs(out, (x.shape, (emb,)))
    _check(lib().nnop_cpu_rms_norm_bwd(_ptr(dy), _ptr(x), _ptr(w), _ptr(rstd), _ptr(dx), _ptr(dw), emb, n, offset,
                                       _thr(threads)), "nnop_cpu_rms_norm_bwd")
    return dx, dw


def layer_norm_fwd(x, w, b, *, eps=1e-6, threads=None, out=None):
    """``(y, mean, rstd)`` of LayerNorm over the last axis (src/layer_norm.jl:8-63)."""
    x, w, b = _f32(x), _f32(w), _f32(b)
    emb, n = _rows(x)
    y, mean, rstd = _outs(out, (x.shape, x.shape[:-1], x.shape[:-1]))
    _check(lib().nnop_cpu_layer_norm_fwd(_ptr(x), _ptr(w), _ptr(b), _ptr(y), _ptr(mean), _ptr(rstd), emb, n, eps,
                                         _thr(threads)), "nnop_cpu_layer_norm_fwd")
    return y, mean, rstd


def layer_norm_bwd(dy, mean, rstd, x, w, *, threads=None, out=None):
    """``(dx, dw, db)`` from the saved mean and rstd (src/layer_norm.jl:65-148)."""
    dy, mean, rstd, x, w = (_f32(a) for a in (dy, mean, rstd, x, w))
    emb, n = _rows(x)
    dx, dw, db = _outs(out, (x.shape, (emb,), (emb,)))
    _check(lib().nnop_cpu_layer_norm_bwd(_ptr(dy), _ptr(x), _ptr(w), _ptr(mean), _ptr(rstd), _ptr(dx), _ptr(dw),
                                         _ptr(db), emb, n, _thr(threads)), "nnop_cpu_layer_norm_bwd")
    return dx, dw, db


def softmax_fwd(x, *, threads=None, out=None):
    """Softmax over the last axis (src/softmax.jl:1-58)."""
    x = _f32(x)
    N, rows = _rows(x)
    (y,) = _outs(None if out is None else (out,), (x.shape,))
    _check(lib().nnop_cpu_softmax_fwd(_ptr(x), _ptr(y), N, rows, _thr(threads)), "nnop_cpu_softmax_fwd")
    return y


def softmax_bwd(dy, y, *, threads=None, out=None):
    """``dy∘y − y∘Σ(dy∘y)`` over the last axis (src/softmax.jl:70-80)."""
    dy, y = _f32(dy), _f32(y)
    N, rows = _rows(y)
    (dx,) = _outs(None if out is None else (out,), (y.shape,))
    _check(lib().nnop_cpu_softmax_bwd(_ptr(dy), _ptr(y), _ptr(dx), N, rows, _thr(threads)), "nnop_cpu_softmax_bwd")
    return dx


def llama_rope(q, k, cos, sin, *, sign=1.0, threads=None, out=None):
    """Rotated copies of q (B,QH,L,E) and k (B,KH,L,E) (src/rope/llama_rope.jl:24-98);
    ``sign=-1`` is the backward."""
    q, k, cos, sin = _f32(q), _f32(k), _f32(cos), _f32(sin)
    B, QH, L, E = q.shape
    qo, ko = _outs(out, (q.shape, k.shape))
    _check(lib().nnop_cpu_llama_rope(_ptr(q), _ptr(k), _ptr(cos), _ptr(sin), _ptr(qo), _ptr(ko), E, L, QH,
                                     k.shape[1], B, sign, _thr(threads)), "nnop_cpu_llama_rope")
    return qo, ko
