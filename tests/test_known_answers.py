"""Closed-form known answers that pin both the oracle and the kernels without
going through the oracle's code.

The reference holds no golden vectors (its tests compare unseeded random inputs
with naive functions), so parity of the oracle rests on reading the reference.
These cases have answers derived by hand from the definitions the reference
implements, computed here with plain loops:

* attention (src/attention.jl:8-143, test/attention_testsetup.jl:21-45):
  - all keys of a head equal: every visible key gets the same weight, so
    o_i = mean of the visible v rows, lse_i = log(n_i) + scale·q_i·k, dq = 0
    (Σ_j dS_ij = 0 and k_j is the same for every j), dv_j = Σ_{i sees j} dO_i/n_i;
  - causal row 0 sees key 0 only: o_0 = v_0, lse_0 = scale·q_0·k_0;
  - q = 0 with a pair bias of c on one key: weights e^c/(e^c+n−1) and
    1/(e^c+n−1), dpair_ij = P_ij·dO_i·(v_j − o_i);
* online_softmax (src/softmax.jl:60-80): softmax of log(a) is a/Σa;
* rms_norm (src/rms_norm.jl:3-38): a constant row a gives y = (w+offset)·a/√(a²+ϵ);
* layer_norm (src/layer_norm.jl:8-63): a ramp x_i = α + β·i has mean α+β(N−1)/2
  and biased variance β²(N²−1)/12; with dy = 1 and w = 1, dx = 0;
* llama_rope (src/rope/llama_rope.jl:7-65): position 0 is the identity; a unit
  vector at dimension i < E/2 rotates to (cos θ_i, sin θ_i) at (i, i+E/2) with
  θ_i = pos/base^(2i/E).

The CPU tests check the oracle against these answers; the GPU tests check the
kernels against the same answers."""
import math

import numpy as np
import pytest

from _util import isapprox, to_dev, to_np
from oracle import nnop_oracle as orc


# ----------------------------------------------------------------- answers
def equal_keys_case(B=2, H=2, QL=37, KL=53, E=16, causal=False, seed=0, kept=None):
    """Inputs whose keys are all equal within a (batch, head), and the closed-form
    o, lse, dq, dv.  `kept`: per-batch number of kept keys (key mask) or None."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, H, QL, E))
    k = np.repeat(rng.standard_normal((B, H, 1, E)), KL, axis=2)
    v = rng.standard_normal((B, H, KL, E))
    do = rng.standard_normal((B, H, QL, E))
    mask = None
    if kept is not None:
        mask = np.zeros((B, KL), bool)
        for b, n in enumerate(kept):
            mask[b, :n] = True
    return q, k, v, do, mask


def equal_keys_answer(q, k, v, do, mask, causal, scale):
    B, H, QL, E = q.shape
    KL = k.shape[2]
    o = np.zeros_like(q)
    lse = np.zeros((B, H, QL))
    dv = np.zeros_like(v)
    for b in range(B):
        for h in range(H):
            for i in range(QL):
                vis = [j for j in range(KL) if (not causal or j <= i) and (mask is None or mask[b, j])]
                n = len(vis)
                o[b, h, i] = sum(v[b, h, j] for j in vis) / n
                lse[b, h, i] = math.log(n) + scale * float(q[b, h, i] @ k[b, h, 0])
                for j in vis:
                    dv[b, h, j] += do[b, h, i] / n
    return o, lse, np.zeros_like(q), dv


def pair_one_key_case(B=1, H=2, L=40, E=64, c=1.5, seed=1):
    """q = 0 (scores are the pair bias alone); pair = c on key jstar(i) of each
    query row, 0 elsewhere.  Layout pair (B, KL, QL, H)."""
    rng = np.random.default_rng(seed)
    q = np.zeros((B, H, L, E))
    k = rng.standard_normal((B, H, L, E))
    v = rng.standard_normal((B, H, L, E))
    do = rng.standard_normal((B, H, L, E))
    pair = np.zeros((B, L, L, H))
    jstar = (np.arange(L) * 7 + 3) % L
    for i in range(L):
        pair[:, jstar[i], i, :] = c
    return q, k, v, do, pair, jstar


def pair_one_key_answer(v, do, jstar, c):
    B, H, L, E = v.shape
    o = np.zeros_like(v)
    lse = np.zeros((B, H, L))
    dpair = np.zeros((B, L, L, H))
    den = math.exp(c) + (L - 1)
    for b in range(B):
        for h in range(H):
            for i in range(L):
                w = np.full(L, 1.0 / den)
                w[jstar[i]] = math.exp(c) / den
                o[b, h, i] = w @ v[b, h]
                lse[b, h, i] = math.log(den)
                dpair[b, :, i, h] = w * ((v[b, h] - o[b, h, i]) @ do[b, h, i])
    return o, lse, dpair


def rope_unit_answer(E, L, base=10000):
    """q[b,h,l] = unit vector at dimension i = l % (E/2): rotated to cos/sin of
    θ_i = l / base^(2i/E) at dimensions i and i + E/2."""
    half = E // 2
    q = np.zeros((1, 1, L, E))
    want = np.zeros_like(q)
    for l in range(L):
        i = l % half
        q[0, 0, l, i] = 1.0
        theta = l / base ** (2 * i / E)
        want[0, 0, l, i] = math.cos(theta)
        want[0, 0, l, i + half] = math.sin(theta)
    return q, want


# ----------------------------------------------------------------- oracle (CPU)
@pytest.mark.parametrize("causal,kept", [(False, None), (True, None), (False, [20, 53]), (True, [53, 9])])
def test_oracle_equal_keys(causal, kept):
    q, k, v, do, mask = equal_keys_case(causal=causal, kept=kept)
    scale = 0.25
    o_w, lse_w, dq_w, dv_w = equal_keys_answer(q, k, v, do, mask, causal, scale)
    o, lse = orc.attention_fwd(q, k, v, causal=causal, kpad_mask=mask, scale=scale)
    dq, _, dv, _ = orc.attention_bwd(do, q, k, v, causal=causal, kpad_mask=mask, scale=scale)
    assert np.allclose(o, o_w, atol=1e-12) and np.allclose(lse, lse_w, atol=1e-12)
    assert np.allclose(dq, dq_w, atol=1e-12) and np.allclose(dv, dv_w, atol=1e-12)


def test_oracle_causal_row_zero():
    rng = np.random.default_rng(3)
    q, k, v = (rng.standard_normal((1, 2, 9, 16)) for _ in range(3))
    o, lse = orc.attention_fwd(q, k, v, causal=True, scale=0.25)
    assert np.allclose(o[:, :, 0], v[:, :, 0], atol=1e-14)
    assert np.allclose(lse[:, :, 0], 0.25 * np.einsum("bhe,bhe->bh", q[:, :, 0], k[:, :, 0]), atol=1e-14)


def test_oracle_pair_on_one_key():
    c = 1.5
    q, k, v, do, pair, jstar = pair_one_key_case(c=c)
    o_w, lse_w, dp_w = pair_one_key_answer(v, do, jstar, c)
    o, lse = orc.attention_fwd(q, k, v, pair, scale=0.125)
    _, _, _, dpair = orc.attention_bwd(do, q, k, v, pair, scale=0.125)
    assert np.allclose(o, o_w, atol=1e-12) and np.allclose(lse, lse_w, atol=1e-12)
    assert np.allclose(dpair, dp_w, atol=1e-12)


def test_oracle_softmax_of_logs():
    a = np.array([[1.0, 2.0, 5.0, 0.5], [3.0, 3.0, 3.0, 3.0]])
    assert np.allclose(orc.softmax_fwd(np.log(a)), a / a.sum(axis=1, keepdims=True), atol=1e-15)


def test_oracle_rms_norm_constant_row():
    for a in (2.0, -0.5):
        x = np.full((1, 64), a)
        w = np.linspace(0.5, 1.5, 64)
        y, _ = orc.rms_norm_fwd(x, w, eps=1e-6, offset=0.25)
        assert np.allclose(y[0], (w + 0.25) * a / math.sqrt(a * a + 1e-6), atol=1e-14)


def test_oracle_layer_norm_ramp():
    N, alpha, beta = 100, 0.3, 0.02
    x = (alpha + beta * np.arange(N))[None]
    y, mu, rstd = orc.layer_norm_fwd(x, np.ones(N), np.zeros(N), eps=1e-6)
    var = beta ** 2 * (N * N - 1) / 12
    assert math.isclose(mu[0], alpha + beta * (N - 1) / 2, rel_tol=1e-14)
    assert math.isclose(rstd[0], 1 / math.sqrt(var + 1e-6), rel_tol=1e-12)
    dx, _, _ = orc.layer_norm_bwd(np.ones((1, N)), x, np.ones(N), eps=1e-6)
    assert np.allclose(dx, 0.0, atol=1e-12)


def test_oracle_rope_unit_vectors():
    E, L = 16, 24
    q, want = rope_unit_answer(E, L)
    cos, sin = orc.llama_rotary_embedding(E, np.arange(L, dtype=np.float32)[None])
    qo, _ = orc.rope_fwd(q, q, cos, sin)
    assert np.allclose(qo, want, atol=2e-6)   # cos/sin are float32, as in the reference


# ----------------------------------------------------------------- kernels (GPU)
TOL = {"f32": 1e-5, "f16": 2e-2, "bf16": 2e-2}


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("E", [64, 128])
@pytest.mark.parametrize("causal,kept", [(False, None), (True, None), (False, [100, 300]), (True, [300, 37])])
def test_kernel_equal_keys(dtype, E, causal, kept):
    import torch

    import nnop
    q, k, v, do, mask = equal_keys_case(B=2, H=2, QL=300, KL=300, E=E, causal=causal, kept=kept, seed=E)
    qd, kd, vd, dod = (to_dev(a, dtype) for a in (q, k, v, do))
    md = torch.from_numpy(mask).cuda() if mask is not None else None
    o, lse = nnop._flash_attention(qd, kd, vd, causal=causal, kpad_mask=md)
    dq, _, dv, _ = nnop.grad_flash_attention(dod, o, lse, qd, kd, vd, causal=causal, kpad_mask=md)
    torch.cuda.synchronize()
    scale = orc.attention_scale(E, dtype)
    o_w, lse_w, _, dv_w = equal_keys_answer(*(to_np(t) for t in (qd, kd, vd, dod)), mask, causal, scale)
    tol = TOL[dtype]
    assert isapprox(to_np(o), o_w, atol=0, rtol=tol)
    assert isapprox(to_np(lse), lse_w, atol=0, rtol=tol)
    assert isapprox(to_np(dv), dv_w, atol=0, rtol=tol)
    # dq is analytically zero: its entries are rounding noise of the dS·K sum
    dq_np = to_np(dq)
    assert np.sqrt(np.mean(dq_np ** 2)) <= (1e-6 if dtype == "f32" else 2e-2) * np.sqrt(np.mean(to_np(dod) ** 2))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("E", [64, 128])
def test_kernel_causal_row_zero(dtype, E):
    import torch

    import nnop
    rng = np.random.default_rng(11)
    q, k, v = (to_dev(rng.standard_normal((2, 3, 200, E)), dtype) for _ in range(3))
    o, lse = nnop._flash_attention(q, k, v, causal=True)
    torch.cuda.synchronize()
    vv = to_np(v)[:, :, 0]
    assert isapprox(to_np(o)[:, :, 0], vv, atol=0, rtol=TOL[dtype] / 4)
    want = orc.attention_scale(E, dtype) * np.einsum("bhe,bhe->bh", to_np(q)[:, :, 0], to_np(k)[:, :, 0])
    assert np.allclose(to_np(lse)[:, :, 0], want, atol=1e-4 if dtype == "f32" else 3e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_kernel_pair_on_one_key(dtype):
    import torch

    import nnop
    c = 1.5
    q, k, v, do, pair, jstar = pair_one_key_case(B=2, H=4, L=200, E=64, c=c, seed=2)
    qd, kd, vd, dod, pd = (to_dev(a, dtype) for a in (q, k, v, do, pair))
    o, lse, ws = nnop._flash_attention_ws(qd, kd, vd, pd, causal=False)
    _, _, _, dpair = nnop.grad_flash_attention(dod, o, lse, qd, kd, vd, pd, causal=False, fwd_workspace=ws)
    torch.cuda.synchronize()
    o_w, lse_w, dp_w = pair_one_key_answer(to_np(vd), to_np(dod), jstar, c)
    tol = TOL[dtype]
    assert isapprox(to_np(o), o_w, atol=0, rtol=tol)
    assert isapprox(to_np(lse), lse_w, atol=0, rtol=tol)
    assert isapprox(to_np(dpair), dp_w, atol=0, rtol=tol)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_kernel_softmax_rms_layer_norm_known_answers(dtype):
    import torch

    import nnop
    a = np.abs(np.random.default_rng(4).standard_normal((7, 1000))) + 0.1
    y = nnop.online_softmax(to_dev(np.log(a), "f32"))
    assert isapprox(to_np(y), a / a.sum(axis=1, keepdims=True), atol=0, rtol=1e-5)
    x = np.full((3, 4096), -0.75)
    w = np.linspace(0.5, 1.5, 4096)
    yd, _ = nnop._rms_norm(to_dev(x, dtype), to_dev(w, dtype), offset=0.25)
    want = (to_np(to_dev(w, dtype)) + 0.25) * -0.75 / math.sqrt(0.75 ** 2 + 1e-6)
    assert isapprox(to_np(yd), np.broadcast_to(want, (3, 4096)), atol=0, rtol=1e-6 if dtype == "f32" else 1e-2)
    N = 4096
    ramp = (0.3 + 1e-3 * np.arange(N))[None].repeat(2, axis=0)
    xd = to_dev(ramp, "f32")
    yl, mu, rstd = nnop._layer_norm(xd, torch.ones(N, device="cuda"), torch.zeros(N, device="cuda"))
    var = 1e-6 * (N * N - 1) / 12
    assert np.allclose(to_np(mu), 0.3 + 1e-3 * (N - 1) / 2, rtol=1e-6)
    assert np.allclose(to_np(rstd), 1 / math.sqrt(var + 1e-6), rtol=1e-5)
    dx, _, _ = nnop.grad_layer_norm(torch.ones_like(xd), mu, rstd, xd, torch.ones(N, device="cuda"))
    torch.cuda.synchronize()
    assert np.max(np.abs(to_np(dx))) <= 1e-4


@pytest.mark.gpu
def test_kernel_rope_unit_vectors():
    import torch

    import nnop
    E, L = 128, 96
    q, want = rope_unit_answer(E, L)
    cos, sin = nnop.LlamaRotaryEmbedding(E)(torch.arange(L, dtype=torch.float32)[None])
    qd = to_dev(q, "f32")
    qo, ko = nnop.llama_rope(qd, qd.clone(), cos=cos, sin=sin)
    torch.cuda.synchronize()
    # the tables are float32 (LlamaRotaryEmbedding computes them in Float32)
    assert np.allclose(to_np(qo), want, atol=1e-4)
    assert np.allclose(to_np(ko), want, atol=1e-4)
    assert np.array_equal(to_np(qo)[0, 0, 0], q[0, 0, 0])   # position 0: identity
