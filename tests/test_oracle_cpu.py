"""The multi-threaded C restatement of the attention (oracle/cpu, fp32) against
the float64 numpy restatement and the golden fixtures, on CPU: every
instruction-set build, ragged and masked shapes, GQA with and without the pair
bias, thread-count independence, and its argument errors.  It is the CPU
baseline bench.py times, so its results are held to the fp32 parity target
(1e-5 relative, Julia-style norm)."""
import pathlib

import numpy as np
import pytest

from _util import isapprox
from oracle import cpu_oracle as ca
from oracle import nnop_oracle as orc

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "oracle_golden.npz"
TOL = dict(atol=0.0, rtol=1e-5)


@pytest.fixture(autouse=True)
def _auto_isa():
    yield
    ca.force_isa("auto")


def _inputs(E, QL, KL, QH, KH, B, pair, mask, seed=0):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, QH, QL, E)).astype(np.float32)
    k = rng.standard_normal((B, KH, KL, E)).astype(np.float32)
    v = rng.standard_normal((B, KH, KL, E)).astype(np.float32)
    do = rng.standard_normal((B, QH, QL, E)).astype(np.float32)
    p = rng.standard_normal((B, KL, QL, QH)).astype(np.float32) if pair else None
    m = None
    if mask:
        m = np.ones((B, KL), bool)
        for b in range(B):
            m[b, rng.integers(1, KL + 1):] = False      # key 0 stays: no row is fully masked
            if p is not None:
                p[b, ~m[b]] = -np.inf                     # as the variable-length workload has it
    return q, k, v, do, p, m


def _compare(q, k, v, do, p, m, causal, scale, threads=None):
    o, lse = ca.attention_fwd(q, k, v, p, causal=causal, kpad_mask=m, scale=scale, threads=threads)
    oo, lo = orc.attention_fwd(q, k, v, p, causal=causal, kpad_mask=m, scale=scale)
    assert isapprox(o, oo, **TOL) and isapprox(lse, lo, **TOL)
    got = ca.attention_bwd(do, o, lse, q, k, v, p, causal=causal, kpad_mask=m, scale=scale, threads=threads)
    want = orc.attention_bwd(do, q, k, v, p, causal=causal, kpad_mask=m, scale=scale)
    for name, a, b in zip(("dq", "dk", "dv", "dpair"), got, want):
        assert (a is None) == (b is None), name
        if a is not None:
            assert isapprox(a, b, **TOL), name
    return o, lse, got


@pytest.mark.parametrize("isa", ["avx512", "avx2", "generic"])
def test_every_instruction_set(isa):
    used = ca.force_isa(isa)
    assert used in ("avx512", "avx2", "generic")
    q, k, v, do, p, m = _inputs(64, 130, 130, 4, 2, 2, pair=True, mask=True)
    _compare(q, k, v, do, p, m, causal=True, scale=0.125)


@pytest.mark.parametrize("E,QL,KL,QH,KH,B,causal,pair,mask", [
    (16, 7, 200, 1, 1, 1, False, False, False),      # one ragged query block, ragged keys
    (128, 300, 257, 8, 2, 2, True, False, False),    # GQA, E = 128, QL > KL causal
    (64, 256, 256, 4, 4, 1, False, True, True),      # full blocks, pair and key mask
    (32, 65, 63, 2, 1, 3, True, True, False),        # GQA with pair, one key block short
    (64, 64, 300, 2, 2, 2, True, True, True),        # causal with KL > QL (keys past the last query)
    (48, 100, 100, 3, 3, 1, False, False, True),     # E not a power of two
])
def test_against_float64_oracle(E, QL, KL, QH, KH, B, causal, pair, mask):
    q, k, v, do, p, m = _inputs(E, QL, KL, QH, KH, B, pair, mask, seed=E + QL)
    _compare(q, k, v, do, p, m, causal, scale=1.0 / np.sqrt(E))


def test_golden_fixture():
    g = np.load(GOLDEN)
    args = dict(causal=True, kpad_mask=g["att_mask"].astype(bool), scale=orc.attention_scale(16, "bf16"))
    o, lse = ca.attention_fwd(g["att_q"], g["att_k"], g["att_v"], g["att_pair"], **args)
    assert isapprox(o, g["att_o"], **TOL) and isapprox(lse, g["att_lse"], **TOL)
    dq, dk, dv, dp = ca.attention_bwd(g["att_do"], o, lse, g["att_q"], g["att_k"], g["att_v"], g["att_pair"], **args)
    for a, name in ((dq, "att_dq"), (dk, "att_dk"), (dv, "att_dv"), (dp, "att_dpair")):
        assert isapprox(a, g[name], **TOL), name


def test_thread_count_does_not_change_results():
    q, k, v, do, p, m = _inputs(64, 200, 200, 4, 2, 2, pair=True, mask=True, seed=3)
    a = dict(causal=True, kpad_mask=m, scale=0.125)
    o1, l1 = ca.attention_fwd(q, k, v, p, threads=1, **a)
    o4, l4 = ca.attention_fwd(q, k, v, p, threads=4, **a)
    assert np.array_equal(o1, o4) and np.array_equal(l1, l4)      # tasks are independent
    g1 = ca.attention_bwd(do, o1, l1, q, k, v, p, threads=1, **a)
    g4 = ca.attention_bwd(do, o1, l1, q, k, v, p, threads=4, **a)
    for x, y in zip(g1[1:], g4[1:]):                                 # dk, dv, dpair: owned by one task
        assert np.array_equal(x, y)
    assert isapprox(g1[0], g4[0], atol=0.0, rtol=1e-6)              # dq: summation order varies


def test_fully_masked_rows_are_nan_like_the_naive_softmax():
    q, k, v, do, p, _ = _inputs(16, 40, 40, 2, 2, 2, pair=False, mask=False)
    m = np.ones((2, 40), bool)
    m[1] = False
    o, lse = ca.attention_fwd(q, k, v, None, kpad_mask=m, scale=0.25)
    oo, lo = orc.attention_fwd(q, k, v, None, kpad_mask=m, scale=0.25)
    assert np.isnan(o[1]).all() and np.isnan(lse[1]).all()
    assert np.isnan(oo[1]).all() and np.isnan(lo[1]).all()
    assert isapprox(o[0], oo[0], **TOL)


def test_empty_query_and_batch():
    q, k, v, do, p, _ = _inputs(16, 0, 10, 2, 1, 1, pair=False, mask=False)
    o, lse = ca.attention_fwd(q, k, v, None, scale=0.25)
    assert o.shape == (1, 2, 0, 16) and lse.shape == (1, 2, 0)
    dq, dk, dv, _ = ca.attention_bwd(do, o, lse, q, k, v, None, scale=0.25)
    assert dq.shape == q.shape and not dk.any() and not dv.any()
    q, k, v, do, p, _ = _inputs(16, 5, 5, 1, 1, 0, pair=True, mask=False)
    o, lse = ca.attention_fwd(q, k, v, p, scale=0.25)
    assert o.shape == (0, 1, 5, 16)


def test_output_reuse_and_errors():
    q, k, v, do, p, _ = _inputs(32, 70, 70, 2, 1, 1, pair=True, mask=False)
    out = (np.full_like(q, 7.0), np.full((1, 2, 70), 7.0, np.float32))
    o, lse = ca.attention_fwd(q, k, v, p, causal=True, scale=0.2, out=out)
    assert o is out[0] and lse is out[1]
    ref = ca.attention_fwd(q, k, v, p, causal=True, scale=0.2)
    assert np.array_equal(o, ref[0]) and np.array_equal(lse, ref[1])
    bout = tuple(np.full_like(a, 7.0) for a in (q, k, v, p))        # dpair fully rewritten (zeros included)
    got = ca.attention_bwd(do, o, lse, q, k, v, p, causal=True, scale=0.2, out=bout)
    want = ca.attention_bwd(do, o, lse, q, k, v, p, causal=True, scale=0.2)
    assert all(x is y for x, y in zip(got, bout))
    assert all(np.array_equal(x, y) for x, y in zip(got[1:], want[1:]))
    with pytest.raises(ValueError):
        ca.attention_fwd(q, k, v, p, scale=0.2, out=(np.empty((1, 2, 70, 31), np.float32), out[1]))
    with pytest.raises(ValueError):                                  # E must be a multiple of 16
        ca.attention_fwd(q[..., :24], k[..., :24], v[..., :24], None, scale=0.2)
    with pytest.raises(ValueError):                                  # QH must be a multiple of KH
        ca.attention_fwd(q, np.concatenate([k, k, k], 1), np.concatenate([v, v, v], 1), None, scale=0.2)


# ------------------------------------------------------------ memory-bound ops
@pytest.mark.parametrize("emb,n", [(4096, 33), (513, 25), (15, 7), (1024, 1)])
@pytest.mark.parametrize("threads", [1, 4])
def test_norms_against_float64_oracle(emb, n, threads):
    rng = np.random.default_rng(emb + n)
    x = rng.standard_normal((n, emb)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(emb)).astype(np.float32)
    b = (0.1 * rng.standard_normal(emb)).astype(np.float32)
    dy = rng.standard_normal((n, emb)).astype(np.float32)
    for offset in (0.0, 1.0):
        y, rstd = ca.rms_norm_fwd(x, w, offset=offset, threads=threads)
        yo, ro = orc.rms_norm_fwd(x, w, offset=offset)
        assert isapprox(y, yo, **TOL) and isapprox(rstd, ro, **TOL)
        dx, dw = ca.rms_norm_bwd(dy, rstd, x, w, offset=offset, threads=threads)
        dxo, dwo = orc.rms_norm_bwd(dy, x, w, offset=offset)
        assert isapprox(dx, dxo, **TOL) and isapprox(dw, dwo, **TOL)
    y, mu, rs = ca.layer_norm_fwd(x, w, b, threads=threads)
    yo, muo, rso = orc.layer_norm_fwd(x, w, b)
    assert isapprox(y, yo, **TOL) and isapprox(mu, muo, atol=1e-6, rtol=1e-5) and isapprox(rs, rso, **TOL)
    got = ca.layer_norm_bwd(dy, mu, rs, x, w, threads=threads)
    for a, o in zip(got, orc.layer_norm_bwd(dy, x, w)):
        assert isapprox(a, o, **TOL)


@pytest.mark.parametrize("rows,N", [(7, 9), (33, 1000), (1, 4), (5, 8193)])
def test_softmax_against_float64_oracle(rows, N):
    rng = np.random.default_rng(rows * N)
    x = (4 * rng.standard_normal((rows, N))).astype(np.float32)
    x[0, ::3] = -np.inf
    dy = rng.standard_normal((rows, N)).astype(np.float32)
    y = ca.softmax_fwd(x, threads=3)
    assert isapprox(y, orc.softmax_fwd(x), **TOL) and not y[0, ::3].any()
    # gradient: the reference tests' absolute floor (1e-6) covers rows whose
    # dx cancels to far below dy (a row with one dominant probability)
    assert isapprox(ca.softmax_bwd(dy, y, threads=3), orc.softmax_bwd(dy, y), atol=1e-6, rtol=1e-5)
    if rows > 1:
        x[1] = -np.inf                                 # an all -Inf row: NaN like the naive softmax
        assert np.isnan(ca.softmax_fwd(x)[1]).all() and np.isnan(orc.softmax_fwd(x)[1]).all()


@pytest.mark.parametrize("E,L,QH,KH,B", [(128, 300, 8, 2, 3), (64, 1025, 3, 5, 2), (16, 7, 1, 1, 1)])
def test_rope_against_float64_oracle(E, L, QH, KH, B):
    rng = np.random.default_rng(E + L)
    q = rng.standard_normal((B, QH, L, E)).astype(np.float32)
    k = rng.standard_normal((B, KH, L, E)).astype(np.float32)
    pos = np.tile(np.arange(L, dtype=np.float32), (B, 1))
    cos, sin = orc.llama_rotary_embedding(E, pos)
    for sign, fn in ((1.0, orc.rope_fwd), (-1.0, orc.rope_bwd)):
        qo, ko = ca.llama_rope(q, k, cos, sin, sign=sign, threads=4)
        qw, kw = fn(q, k, cos, sin)
        assert isapprox(qo, qw, **TOL) and isapprox(ko, kw, **TOL)
    ones = np.ones((1, 1, L, E), np.float32)             # the reference's q = k = ones case
    qo, _ = ca.llama_rope(ones, ones, cos[:1], sin[:1])
    assert isapprox(qo, orc.rope_fwd(ones, ones, cos[:1], sin[:1])[0], **TOL)
