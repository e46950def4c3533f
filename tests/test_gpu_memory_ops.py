"""GPU parity of online_softmax, rms_norm, layer_norm and llama_rope against the
CPU oracle, on the reference's test grids (test/softmax_tests.jl,
test/rmsnorm_tests.jl, test/layernorm_tests.jl, test/rope_tests.jl) plus the
dtypes and sizes the reference does not test (bf16/f16, long rows, batches).

Tolerances (norm-based, Julia isapprox): the reference's own -- forward
rtol=√eps(Float32), gradients atol=rtol=1e-6 -- for fp32; 2e-2 relative for
bf16/f16 (the parity target of this implementation)."""
import numpy as np
import pytest

from _util import isapprox, to_dev, to_np
from oracle import nnop_oracle as orc

pytestmark = pytest.mark.gpu

EMBS = (15, 255, 256, 257, 511, 512, 513, 1024)
NS = (1, 2, 4, 15, 16, 17, 23, 25)
FWD_RTOL_F32 = float(np.sqrt(np.finfo(np.float32).eps))
TOL_HALF = 2e-2


def _nnop():
    import nnop
    return nnop


def _tols(dtype):
    if dtype == "f32":
        return dict(atol=0.0, rtol=FWD_RTOL_F32), dict(atol=1e-6, rtol=1e-6)
    return dict(atol=0.0, rtol=TOL_HALF), dict(atol=0.0, rtol=TOL_HALF)


# ----------------------------------------------------------------- RMSNorm
@pytest.mark.parametrize("offset", [0.0, 1.0])
@pytest.mark.parametrize("emb", EMBS)
def test_rms_norm_reference_grid(emb, offset):
    nnop = _nnop()
    for n in NS:
        rng = np.random.default_rng(emb * 100 + n)
        x = rng.random((n, emb), dtype=np.float32)
        w = rng.random(emb, dtype=np.float32)
        dy = np.ones((n, emb), np.float32)            # gradient of sum(y)
        xd, wd, dyd = to_dev(x, "f32"), to_dev(w, "f32"), to_dev(dy, "f32")
        y, rstd = nnop._rms_norm(xd, wd, offset=offset)
        dx, dw = nnop.grad_rms_norm(dyd, rstd, xd, wd, offset=offset)
        y_o, rstd_o = orc.rms_norm_fwd(x, w, offset=offset)
        dx_o, dw_o = orc.rms_norm_bwd(dy, x, w, offset=offset)
        assert isapprox(to_np(y), y_o, atol=0, rtol=FWD_RTOL_F32), (emb, n)
        assert isapprox(to_np(rstd), rstd_o, atol=0, rtol=FWD_RTOL_F32)
        assert isapprox(to_np(dx), dx_o, atol=1e-6, rtol=1e-6), (emb, n)
        assert isapprox(to_np(dw), dw_o, atol=1e-6, rtol=1e-6), (emb, n)


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("emb,n", [(4096, 257), (4096, 1), (768, 1000), (8192, 33), (40000, 3), (1000, 5)])
def test_rms_norm_dtypes(dtype, emb, n):
    nnop = _nnop()
    rng = np.random.default_rng(7)
    x = rng.standard_normal((n, emb)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(emb)).astype(np.float32)
    dy = rng.standard_normal((n, emb)).astype(np.float32)
    xd, wd, dyd = to_dev(x, dtype), to_dev(w, dtype), to_dev(dy, dtype)
    xr, wr, dyr = to_np(xd), to_np(wd), to_np(dyd)
    y, rstd = nnop._rms_norm(xd, wd, offset=0.5)
    dx, dw = nnop.grad_rms_norm(dyd, rstd, xd, wd, offset=0.5)
    ftol, gtol = _tols(dtype)
    assert isapprox(to_np(y), orc.rms_norm_fwd(xr, wr, offset=0.5)[0], **ftol)
    dx_o, dw_o = orc.rms_norm_bwd(dyr, xr, wr, offset=0.5)
    gt = gtol if dtype != "f32" else dict(atol=0, rtol=1e-5)
    assert isapprox(to_np(dx), dx_o, **gt)
    assert isapprox(to_np(dw), dw_o, **gt)


# ----------------------------------------------------------------- LayerNorm
@pytest.mark.parametrize("emb", EMBS)
def test_layer_norm_reference_grid(emb):
    nnop = _nnop()
    for n in NS:
        rng = np.random.default_rng(emb * 1000 + n)
        x = rng.random((n, emb), dtype=np.float32)
        w = rng.random(emb, dtype=np.float32)
        b = rng.random(emb, dtype=np.float32)
        dy = np.ones((n, emb), np.float32)
        xd, wd, bd, dyd = (to_dev(a, "f32") for a in (x, w, b, dy))
        y, mu, rstd = nnop._layer_norm(xd, wd, bd)
        dx, dw, db = nnop.grad_layer_norm(dyd, mu, rstd, xd, wd)
        y_o, mu_o, rstd_o = orc.layer_norm_fwd(x, w, b)
        dx_o, dw_o, db_o = orc.layer_norm_bwd(dy, x, w)
        assert isapprox(to_np(y), y_o, atol=0, rtol=FWD_RTOL_F32), (emb, n)
        assert isapprox(to_np(mu), mu_o, atol=0, rtol=FWD_RTOL_F32)
        assert isapprox(to_np(dx), dx_o, atol=1e-6, rtol=1e-6), (emb, n)
        assert isapprox(to_np(dw), dw_o, atol=1e-6, rtol=1e-6), (emb, n)
        assert isapprox(to_np(db), db_o, atol=1e-6, rtol=1e-6), (emb, n)


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("emb,n", [(4096, 257), (768, 1000), (8192, 33), (40000, 3), (1000, 5)])
def test_layer_norm_dtypes(dtype, emb, n):
    nnop = _nnop()
    rng = np.random.default_rng(11)
    x = rng.standard_normal((n, emb)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(emb)).astype(np.float32)
    b = (0.1 * rng.standard_normal(emb)).astype(np.float32)
    dy = rng.standard_normal((n, emb)).astype(np.float32)
    xd, wd, bd, dyd = (to_dev(a, dtype) for a in (x, w, b, dy))
    xr, wr, br, dyr = (to_np(a) for a in (xd, wd, bd, dyd))
    y, mu, rstd = nnop._layer_norm(xd, wd, bd)
    dx, dw, db = nnop.grad_layer_norm(dyd, mu, rstd, xd, wd)
    ftol, gtol = _tols(dtype)
    assert isapprox(to_np(y), orc.layer_norm_fwd(xr, wr, br)[0], **ftol)
    dx_o, dw_o, db_o = orc.layer_norm_bwd(dyr, xr, wr)
    gt = gtol if dtype != "f32" else dict(atol=0, rtol=1e-5)
    assert isapprox(to_np(dx), dx_o, **gt)
    assert isapprox(to_np(dw), dw_o, **gt)
    assert isapprox(to_np(db), db_o, **gt)


# ----------------------------------------------------------------- softmax
@pytest.mark.parametrize("seq_len", [32, 33, 63, 255, 256, 511, 512, 513, 1024])
def test_softmax_reference_grid(seq_len):
    nnop = _nnop()
    rng = np.random.default_rng(seq_len)
    x = rng.random((4, seq_len), dtype=np.float32)
    xd = to_dev(x, "f32")
    y = nnop.online_softmax(xd)
    assert isapprox(to_np(y), orc.softmax_fwd(x), atol=0, rtol=FWD_RTOL_F32)
    dy = np.ones_like(x)
    dx = nnop.grad_online_softmax(to_dev(dy, "f32"), y)
    assert isapprox(to_np(dx), orc.softmax_bwd(dy, to_np(y)), atol=1e-6, rtol=1e-6)


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("n,cols", [(8192, 17), (8193, 3), (100000, 2), (7, 9), (1, 4), (4096, 64)])
def test_softmax_dtypes(dtype, n, cols):
    nnop = _nnop()
    rng = np.random.default_rng(n + cols)
    x = (4.0 * rng.standard_normal((cols, n))).astype(np.float32)
    dy = rng.standard_normal((cols, n)).astype(np.float32)
    xd, dyd = to_dev(x, dtype), to_dev(dy, dtype)
    y = nnop.online_softmax(xd)
    dx = nnop.grad_online_softmax(dyd, y)
    ftol, gtol = _tols(dtype)
    assert isapprox(to_np(y), orc.softmax_fwd(to_np(xd)), **ftol)
    gt = gtol if dtype != "f32" else dict(atol=0, rtol=1e-5)
    assert isapprox(to_np(dx), orc.softmax_bwd(to_np(dyd), to_np(y)), **gt)


def test_softmax_neg_inf_entries():
    """−Inf entries give exact zeros; an all −Inf row gives NaN like the
    reference's md_reduce (src/softmax.jl:6-16,54)."""
    import torch
    nnop = _nnop()
    x = torch.randn(3, 64, device="cuda")
    x[0, :10] = -float("inf")
    x[2, :] = -float("inf")
    y = nnop.online_softmax(x)
    assert torch.all(y[0, :10] == 0)
    assert torch.allclose(y[0].sum(), torch.tensor(1.0, device="cuda"), atol=1e-6)
    assert torch.all(torch.isnan(y[2]))


# ----------------------------------------------------------------- RoPE
@pytest.mark.parametrize("L", [13, 255, 256, 257, 1024, 1025])
def test_rope_reference_grid(L):
    """q = k = ones, dim 16, batch 1 (test/rope_tests.jl:21-56)."""
    nnop = _nnop()
    dim = 16
    pos = np.arange(L, dtype=np.float32)[None]
    cos_o, sin_o = orc.llama_rotary_embedding(dim, pos)
    cos, sin = nnop.LlamaRotaryEmbedding(dim)(pos)
    assert isapprox(to_np(cos), cos_o, atol=1e-6, rtol=1e-6)
    assert isapprox(to_np(sin), sin_o, atol=1e-6, rtol=1e-6)
    for QH in (1, 3, 4, 5):
        for KH in (1, 3, 4, 5):
            q = np.ones((1, QH, L, dim), np.float32)
            k = np.ones((1, KH, L, dim), np.float32)
            qd, kd = to_dev(q, "f32"), to_dev(k, "f32")
            q1, k1 = nnop.llama_rope(qd, kd, cos=cos, sin=sin)
            q2, k2 = orc.rope_fwd(q, k, to_np(cos), to_np(sin))
            assert isapprox(to_np(q1), q2, atol=1e-6, rtol=1e-6)
            assert isapprox(to_np(k1), k2, atol=1e-6, rtol=1e-6)
            # gradient of sum(qr) + sum(kr)
            g1q, g1k = nnop.grad_llama_rope(to_dev(np.ones_like(q), "f32"), to_dev(np.ones_like(k), "f32"),
                                            cos=cos, sin=sin)
            g2q, g2k = orc.rope_bwd(np.ones_like(q), np.ones_like(k), to_np(cos), to_np(sin))
            assert isapprox(to_np(g1q), g2q, atol=1e-6, rtol=1e-6)
            assert isapprox(to_np(g1k), g2k, atol=1e-6, rtol=1e-6)


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("E,L,QH,KH,B,cb", [(128, 300, 8, 2, 3, 3), (64, 1025, 3, 5, 2, 1), (16, 7, 1, 1, 1, 1),
                                            (6, 9, 2, 3, 2, 2), (128, 4096, 4, 1, 1, 1)])
def test_rope_dtypes(dtype, E, L, QH, KH, B, cb):
    nnop = _nnop()
    rng = np.random.default_rng(E + L)
    pos = np.tile(np.arange(L, dtype=np.float32), (cb, 1)) + np.arange(cb, dtype=np.float32)[:, None]
    cos, sin = nnop.LlamaRotaryEmbedding(E)(pos)
    q = rng.standard_normal((B, QH, L, E)).astype(np.float32)
    k = rng.standard_normal((B, KH, L, E)).astype(np.float32)
    qd, kd = to_dev(q, dtype), to_dev(k, dtype)
    q1, k1 = nnop.llama_rope(qd, kd, cos=cos, sin=sin)
    c = np.broadcast_to(to_np(cos), (B, L, E))
    s = np.broadcast_to(to_np(sin), (B, L, E))
    q2, k2 = orc.rope_fwd(to_np(qd), to_np(kd), c, s)
    tol = dict(atol=1e-6, rtol=1e-6) if dtype == "f32" else dict(atol=0, rtol=TOL_HALF)
    assert isapprox(to_np(q1), q2, **tol)
    assert isapprox(to_np(k1), k2, **tol)
    g1q, g1k = nnop.grad_llama_rope(q1, k1, cos=cos, sin=sin)
    g2q, g2k = orc.rope_bwd(to_np(q1), to_np(k1), c, s)
    assert isapprox(to_np(g1q), g2q, **tol)
    assert isapprox(to_np(g1k), g2k, **tol)
    # backward undoes forward (rotation by −θ)
    assert isapprox(to_np(g1q), to_np(qd), atol=0, rtol=1e-5 if dtype == "f32" else TOL_HALF)


def test_rope_autograd_matches_oracle():
    import torch
    nnop = _nnop()
    B, QH, KH, L, E = 2, 4, 2, 33, 32
    cos, sin = nnop.LlamaRotaryEmbedding(E)(np.tile(np.arange(L, dtype=np.float32), (B, 1)))
    q = torch.randn(B, QH, L, E, device="cuda", requires_grad=True)
    k = torch.randn(B, KH, L, E, device="cuda", requires_grad=True)
    qr, kr = nnop.llama_rope(q, k, cos=cos, sin=sin)
    (qr.sum() + 2 * kr.sum()).backward()
    g2q, g2k = orc.rope_bwd(np.ones((B, QH, L, E)), 2 * np.ones((B, KH, L, E)), to_np(cos), to_np(sin))
    assert isapprox(to_np(q.grad), g2q, atol=1e-6, rtol=1e-6)
    assert isapprox(to_np(k.grad), g2k, atol=1e-6, rtol=1e-6)


def test_norm_autograd_matches_oracle():
    import torch
    nnop = _nnop()
    x = torch.rand(25, 513, device="cuda", requires_grad=True)
    w = torch.rand(513, device="cuda", requires_grad=True)
    b = torch.rand(513, device="cuda", requires_grad=True)
    nnop.rms_norm(x, w, offset=1.0).sum().backward()
    dx_o, dw_o = orc.rms_norm_bwd(np.ones((25, 513)), to_np(x), to_np(w), offset=1.0)
    assert isapprox(to_np(x.grad), dx_o, atol=1e-6, rtol=1e-6)
    assert isapprox(to_np(w.grad), dw_o, atol=1e-6, rtol=1e-6)
    x.grad = None
    w.grad = None
    dy = torch.randn(25, 513, device="cuda")
    (nnop.layer_norm(x, w, b) * dy).sum().backward()
    dx_o, dw_o, db_o = orc.layer_norm_bwd(to_np(dy), to_np(x), to_np(w))
    assert isapprox(to_np(x.grad), dx_o, atol=0, rtol=1e-5)
    assert isapprox(to_np(w.grad), dw_o, atol=0, rtol=1e-5)
    assert isapprox(to_np(b.grad), db_o, atol=0, rtol=1e-5)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_norm_row_shards_sum_to_whole_job(dtype):
    """Three ranks' row shards run on one GPU: the per-shard dx rows and the sum
    of the per-shard dw / db are the whole job's gradients (the cross-rank sum
    that ``allreduce_norm_grads`` performs, here summed on the host); without a
    process group the sharded calls are the plain ones."""
    import torch

    from nnop import shards
    nnop = _nnop()
    rng = np.random.default_rng(12)
    n, emb, world = 1000, 768, 3
    x = rng.standard_normal((n, emb)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(emb)).astype(np.float32)
    b = (0.1 * rng.standard_normal(emb)).astype(np.float32)
    dy = rng.standard_normal((n, emb)).astype(np.float32)
    xd, wd, bd, dyd = (to_dev(a, dtype) for a in (x, w, b, dy))
    xr, wr, dyr = (to_np(a) for a in (xd, wd, dyd))
    _, rstd = nnop._rms_norm(xd, wd)
    _, mu, rs = nnop._layer_norm(xd, wd, bd)
    dx_rms, dx_ln, dw_rms, dw_ln, db_ln = [], [], 0.0, 0.0, 0.0
    for r in range(world):
        s = shards.row_shard(n, r, world)
        dx, dw = shards.grad_rms_norm_sharded(dyd[s], rstd[s], xd[s], wd)
        dx_rms.append(to_np(dx))
        dw_rms = dw_rms + to_np(dw)
        dx, dw, db = shards.grad_layer_norm_sharded(dyd[s], mu[s], rs[s], xd[s], wd)
        dx_ln.append(to_np(dx))
        dw_ln, db_ln = dw_ln + to_np(dw), db_ln + to_np(db)
    tol = dict(atol=0, rtol=1e-5) if dtype == "f32" else dict(atol=0, rtol=TOL_HALF)
    dx_o, dw_o = orc.rms_norm_bwd(dyr, xr, wr)
    assert isapprox(np.concatenate(dx_rms), dx_o, **tol) and isapprox(dw_rms, dw_o, **tol)
    dx_o, dw_o, db_o = orc.layer_norm_bwd(dyr, xr, wr)
    assert isapprox(np.concatenate(dx_ln), dx_o, **tol)
    assert isapprox(dw_ln, dw_o, **tol) and isapprox(db_ln, db_o, **tol)
    whole = nnop.grad_rms_norm(dyd, rstd, xd, wd)
    one = shards.grad_rms_norm_sharded(dyd, rstd, xd, wd)
    assert all(torch.equal(a, c) for a, c in zip(whole, one))
