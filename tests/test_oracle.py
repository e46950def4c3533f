"""CPU checks of the oracle itself (no GPU).

The reference cannot run here (Julia is absent, its kernels are cpu=false) and
its tests hold no golden vectors, so the oracle is checked the way the
reference's tests check NNop: against automatic differentiation of the naive
forward functions (Zygote there, torch.autograd in float64 here), plus the one
known-answer case of the reference tests (RoPE on q = k = ones) and the frozen
fixtures in tests/golden/."""
import pathlib

import numpy as np
import pytest
import torch

from _util import isapprox
from oracle import nnop_oracle as orc

GOLDEN = pathlib.Path(__file__).parent / "golden" / "oracle_golden.npz"


def _t(a):
    return torch.tensor(np.asarray(a, np.float64), requires_grad=True)


def torch_naive_attention(q, k, v, pair, causal, kpad_mask, scale):
    """Line-by-line torch restatement of naive_attention
    (test/attention_testsetup.jl:21-45), differentiated by autograd."""
    B, QH, QL, E = q.shape
    KH, KL = k.shape[1], k.shape[2]
    n_rep = QH // KH
    kk = k.repeat_interleave(n_rep, dim=1)
    vv = v.repeat_interleave(n_rep, dim=1)
    a = torch.einsum("bhqe,bhke->bhqk", q, kk) * scale
    if causal:
        m = torch.arange(KL)[None, :] <= torch.arange(QL)[:, None]
        a = torch.where(m, a, torch.tensor(-torch.inf, dtype=a.dtype))
    if kpad_mask is not None:
        a = a + torch.log(torch.tensor(kpad_mask, dtype=torch.float64))[:, None, None, :]
    if pair is not None:
        a = a + pair.permute(0, 3, 2, 1)
    p = torch.softmax(a, dim=-1)
    return torch.einsum("bhqk,bhke->bhqe", p, vv)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("use_pair", [False, True])
@pytest.mark.parametrize("use_mask", [False, True])
@pytest.mark.parametrize("QH,KH", [(2, 2), (4, 2), (6, 1)])
def test_attention_oracle_vs_autograd(causal, use_pair, use_mask, QH, KH):
    rng = np.random.default_rng(QH * 7 + KH)
    B, QL, KL, E = 2, 37, 37 if causal else 45, 16
    q = rng.standard_normal((B, QH, QL, E))
    k = rng.standard_normal((B, KH, KL, E))
    v = rng.standard_normal((B, KH, KL, E))
    do = rng.standard_normal((B, QH, QL, E))
    pair = rng.standard_normal((B, KL, QL, QH)) if use_pair else None
    mask = None
    if use_mask:
        mask = np.ones((B, KL), bool)
        mask[-1, -11:] = False
    scale = 1 / np.sqrt(E)
    o, lse = orc.attention_fwd(q, k, v, pair, causal=causal, kpad_mask=mask, scale=scale)
    dq, dk, dv, dp = orc.attention_bwd(do, q, k, v, pair, causal=causal, kpad_mask=mask, scale=scale)
    tq, tk, tv = _t(q), _t(k), _t(v)
    tp = _t(pair) if use_pair else None
    to = torch_naive_attention(tq, tk, tv, tp, causal, mask, scale)
    (to * torch.tensor(do)).sum().backward()
    assert isapprox(o, to.detach().numpy(), atol=0, rtol=1e-12)
    assert isapprox(dq, tq.grad.numpy(), atol=0, rtol=1e-12)
    assert isapprox(dk, tk.grad.numpy(), atol=0, rtol=1e-12)
    assert isapprox(dv, tv.grad.numpy(), atol=0, rtol=1e-12)
    if use_pair:
        assert isapprox(dp, tp.grad.numpy(), atol=0, rtol=1e-12)
    # lse consistency: o = Σ exp(s − lse) v
    assert np.all(np.isfinite(lse))


def test_attention_flops_convention():
    fwd, bwd = orc.attention_flops(8, 16, 4096, 4096, 64, True)
    assert abs((fwd + bwd) / 1e12 - 0.962) < 1e-3   # config 2: 0.962 TFLOP


def test_softmax_oracle_vs_autograd():
    rng = np.random.default_rng(0)
    x = rng.random((4, 513))
    dy = rng.standard_normal((4, 513))
    tx = _t(x)
    y = torch.softmax(tx, dim=-1)
    (y * torch.tensor(dy)).sum().backward()
    assert isapprox(orc.softmax_fwd(x), y.detach().numpy(), atol=0, rtol=1e-13)
    assert isapprox(orc.softmax_bwd(dy, orc.softmax_fwd(x)), tx.grad.numpy(), atol=0, rtol=1e-12)


@pytest.mark.parametrize("offset", [0.0, 1.0])
def test_rms_norm_oracle_vs_autograd(offset):
    rng = np.random.default_rng(1)
    x, w, dy = rng.random((17, 257)), rng.random(257), rng.standard_normal((17, 257))
    tx, tw = _t(x), _t(w)
    y = (tw + offset) * tx / torch.sqrt((tx ** 2).mean(dim=-1, keepdim=True) + 1e-6)
    (y * torch.tensor(dy)).sum().backward()
    assert isapprox(orc.rms_norm_fwd(x, w, offset=offset)[0], y.detach().numpy(), atol=0, rtol=1e-13)
    dx, dw = orc.rms_norm_bwd(dy, x, w, offset=offset)
    assert isapprox(dx, tx.grad.numpy(), atol=0, rtol=1e-12)
    assert isapprox(dw, tw.grad.numpy(), atol=0, rtol=1e-12)


def test_layer_norm_oracle_vs_autograd():
    rng = np.random.default_rng(2)
    x, w, b, dy = rng.random((15, 513)), rng.random(513), rng.random(513), rng.standard_normal((15, 513))
    tx, tw, tb = _t(x), _t(w), _t(b)
    mu = tx.mean(dim=-1, keepdim=True)
    var = ((tx - mu) ** 2).mean(dim=-1, keepdim=True)
    y = (tx - mu) / torch.sqrt(var + 1e-6) * tw + tb
    (y * torch.tensor(dy)).sum().backward()
    assert isapprox(orc.layer_norm_fwd(x, w, b)[0], y.detach().numpy(), atol=0, rtol=1e-13)
    dx, dw, db = orc.layer_norm_bwd(dy, x, w)
    assert isapprox(dx, tx.grad.numpy(), atol=0, rtol=1e-11)
    assert isapprox(dw, tw.grad.numpy(), atol=0, rtol=1e-12)
    assert isapprox(db, tb.grad.numpy(), atol=0, rtol=1e-12)


def test_rope_oracle_vs_autograd_and_naive():
    """The kernel form (first-half cos/sin) equals the reference test's
    naive_llama_rope (test/rope_tests.jl:6-19) for tables made by
    LlamaRotaryEmbedding, whose two halves are equal."""
    rng = np.random.default_rng(3)
    B, QH, KH, L, E = 2, 3, 2, 29, 16
    cos, sin = orc.llama_rotary_embedding(E, np.tile(np.arange(L, dtype=np.float32), (B, 1)))
    q, k = rng.standard_normal((B, QH, L, E)), rng.standard_normal((B, KH, L, E))

    def rotate_half(x):
        h = x.shape[-1] // 2
        return torch.cat([-x[..., h:], x[..., :h]], dim=-1)

    tq, tk = _t(q), _t(k)
    c = torch.tensor(cos, dtype=torch.float64)[:, None]
    s = torch.tensor(sin, dtype=torch.float64)[:, None]
    qn, kn = tq * c + rotate_half(tq) * s, tk * c + rotate_half(tk) * s
    (qn.sum() + kn.sum()).backward()
    q1, k1 = orc.rope_fwd(q, k, cos, sin)
    assert isapprox(q1, qn.detach().numpy(), atol=0, rtol=1e-14)
    assert isapprox(k1, kn.detach().numpy(), atol=0, rtol=1e-14)
    gq, gk = orc.rope_bwd(np.ones_like(q), np.ones_like(k), cos, sin)
    assert isapprox(gq, tq.grad.numpy(), atol=0, rtol=1e-14)
    assert isapprox(gk, tk.grad.numpy(), atol=0, rtol=1e-14)


def test_rope_known_answer_ones():
    """test/rope_tests.jl:38-44: q = k = ones, so out[i] = cos_i − sin_i and
    out[i + E/2] = cos_i + sin_i, with θ_i = pos · 10000^(−2i/E)."""
    L, E = 1025, 16
    pos = np.arange(L, dtype=np.float32)[None]
    cos, sin = orc.llama_rotary_embedding(E, pos)
    theta = pos[0][:, None].astype(np.float64) * 10000.0 ** (-np.arange(0, E, 2) / E)
    assert np.max(np.abs(cos[0, :, : E // 2] - np.cos(theta))) < 2e-3   # float32 phase at pos ~1e3
    q = np.ones((1, 1, L, E))
    q1, _ = orc.rope_fwd(q, q, cos, sin)
    c, s = cos[0, :, : E // 2].astype(np.float64), sin[0, :, : E // 2].astype(np.float64)
    assert np.allclose(q1[0, 0, :, : E // 2], c - s, atol=1e-15)
    assert np.allclose(q1[0, 0, :, E // 2:], c + s, atol=1e-15)


def test_bf16_rounding():
    x = np.array([1.0, 1.00390625, 1.005859375, 3.14159265, -2.5e-3, np.inf, np.nan], np.float64)
    r = orc.round_to(x, "bf16")
    t = torch.tensor(x, dtype=torch.float32).to(torch.bfloat16).to(torch.float64).numpy()
    assert np.array_equal(np.isnan(r), np.isnan(t))
    assert np.array_equal(r[~np.isnan(r)], t[~np.isnan(t)])
    assert orc.attention_scale(64, "bf16") == 0.125
    assert orc.attention_scale(128, "bf16") == float(torch.tensor(1 / np.sqrt(128)).to(torch.bfloat16))


def test_golden_fixtures_reproduce():
    """The oracle still produces the frozen fixtures (tests/golden/make_golden.py)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN.parent / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    ref = np.load(GOLDEN)
    fresh = mg.compute()
    assert set(ref.files) == set(fresh)
    for key in ref.files:
        a, b = ref[key], fresh[key]
        assert a.shape == b.shape, key
        assert np.allclose(a, b, rtol=1e-12, atol=1e-12, equal_nan=True), key
