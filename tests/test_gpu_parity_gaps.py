"""GPU parity on the paths and sizes the smaller grids leave out.

* the mma.sync kernel family (fa_mma.cu), selected for every shape by
  NNOP_B200_FA=mma: the E = 64 pair-bias cases, GQA and E = 128;
* the one-tile tcgen05 forward (fa_fwd_sm100.cu), selected by
  NNOP_B200_FA=one_tile;
* the C-ABI forward called with a NULL workspace (the pair bias is then read
  in the reference layout by the mma.sync forward) followed by the tcgen05
  backward, which rebuilds the per-head pair tiles itself;
* rows whose every kept key carries a −Inf pair bias: the reference gives NaN
  (its naive softmax of an all −Inf column).  The bf16 tensor-core path gives
  NaN as well; the f16 path gives the softmax of the other logits (−Inf is
  stored as −65504 in the per-head tiles, and a row of equal biases cancels
  out), which these tests pin, together with every other row matching the
  oracle;
* the memory-bound workload at its full size (x (4096, 65536) for the norms in
  bf16 and fp32, x (8192, 16384) fp32 for the softmax): sampled rows against the
  oracle element by element, the weight/bias gradients over every row (the
  oracle's per-row-chunk gradients summed), and size-independent properties on
  every row (softmax rows sum to one, its gradient rows to zero)."""
import ctypes as C

import numpy as np
import pytest

from _util import isapprox, to_dev, to_np
from oracle import nnop_oracle as orc
from test_gpu_attention import check, run_case

pytestmark = pytest.mark.gpu


# ----------------------------------------------------------------- mma.sync family
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("causal", [False, True])
def test_mma_family_pair_cases(monkeypatch, dtype, causal):
    monkeypatch.setenv("NNOP_B200_FA", "mma")
    for (B, QH, KH, QL, KL, use_mask) in [(2, 4, 4, 300, 421, True), (1, 8, 2, 257, 257, False),
                                          (3, 2, 2, 128, 64, True)]:
        if causal:
            KL = QL
        got, want = run_case(B, QH, KH, QL, KL, 64, dtype, causal, True, use_mask, seed=QL + QH)
        check(got, want, dtype, tag=f"mma QL={QL} KL={KL} QH={QH}")


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_mma_family_gqa_and_e128(monkeypatch, dtype):
    monkeypatch.setenv("NNOP_B200_FA", "mma")
    for (QH, KH, L, E, causal) in [(8, 2, 300, 64, True), (6, 1, 257, 32, False), (4, 2, 513, 128, True),
                                   (2, 2, 200, 128, False)]:
        got, want = run_case(2, QH, KH, L, L, E, dtype, causal, False, False, seed=L + E)
        check(got, want, dtype, tag=f"mma E={E} L={L}")


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_one_tile_forward_family(monkeypatch, dtype):
    """NNOP_B200_FA=one_tile: the one-query-tile tcgen05 forward
    (fa_fwd_sm100.cu) that the two-tile kernel replaced by default, on pair,
    mask, GQA and E = 128 cases."""
    monkeypatch.setenv("NNOP_B200_FA", "one_tile")
    for (B, QH, KH, QL, KL, E, causal, pair, use_mask) in [(2, 4, 4, 300, 421, 64, False, True, True),
                                                           (1, 4, 4, 384, 384, 64, True, True, False),
                                                           (2, 8, 2, 257, 257, 128, True, False, True),
                                                           (1, 2, 1, 200, 77, 64, False, False, False)]:
        got, want = run_case(B, QH, KH, QL, KL, E, dtype, causal, pair, use_mask, seed=QL + E)
        check(got, want, dtype, tag=f"one_tile E={E} QL={QL} KL={KL} pair={pair}")


def test_c_abi_forward_without_workspace():
    """nnop_flash_attention_fwd with workspace = NULL: the pair bias takes the
    mma.sync forward; the backward (tcgen05, tiles rebuilt) matches the oracle."""
    import torch

    import nnop
    from nnop._lib import lib
    for dtype, causal in (("bf16", True), ("f16", False)):
        rng = np.random.default_rng(8)
        B, H, L, E = 2, 4, 300, 64
        q, k, v, do = (rng.standard_normal((B, H, L, E)) for _ in range(4))
        pair = rng.standard_normal((B, L, L, H))
        qd, kd, vd, dod, pd = (to_dev(a, dtype) for a in (q, k, v, do, pair))
        o = torch.empty_like(qd)
        lse = torch.empty(B, H, L, dtype=torch.float32, device="cuda")
        dt = {"bf16": 2, "f16": 1}[dtype]
        st = lib.nnop_flash_attention_fwd(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), pd.data_ptr(), None,
                                          o.data_ptr(), lse.data_ptr(), None, 0, E, L, L, H, H, B, int(causal), dt,
                                          torch.cuda.current_stream().cuda_stream)
        assert st == 0, lib.nnop_last_error()
        dq, dk, dv, dpair = nnop.grad_flash_attention(dod, o, lse, qd, kd, vd, pd, causal=causal)
        torch.cuda.synchronize()
        args = dict(causal=causal, scale=orc.attention_scale(E, dtype))
        ref = [to_np(t) for t in (qd, kd, vd, pd, dod)]
        o_o, lse_o = orc.attention_fwd(*ref[:4], **args)
        g = orc.attention_bwd(ref[4], *ref[:4], **args)
        check(dict(o=to_np(o), lse=to_np(lse), dq=to_np(dq), dk=to_np(dk), dv=to_np(dv), dpair=to_np(dpair)),
              dict(o=o_o, lse=lse_o, dq=g[0], dk=g[1], dv=g[2], dpair=g[3]), dtype, tag=f"{dtype} NULL ws")


# ----------------------------------------------------------------- all −Inf pair rows
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_rows_with_all_neg_inf_pair(dtype):
    import torch

    import nnop
    rng = np.random.default_rng(31)
    B, H, L, E = 1, 2, 256, 64
    q, k, v, do = (rng.standard_normal((B, H, L, E)) for _ in range(4))
    pair = 0.5 * rng.standard_normal((B, L, L, H))
    bad = [5, 130, 255]                  # query rows whose every key has pair = −Inf
    for i in bad:
        pair[:, :, i, :] = -np.inf
    qd, kd, vd, dod, pd = (to_dev(a, dtype) for a in (q, k, v, do, pair))
    o, lse, ws = nnop._flash_attention_ws(qd, kd, vd, pd, causal=False)
    torch.cuda.synchronize()
    on = to_np(o)
    good = [i for i in range(L) if i not in bad]
    ref = [to_np(t) for t in (qd, kd, vd, pd)]
    scale = orc.attention_scale(E, dtype)
    o_o, _ = orc.attention_fwd(*ref, causal=False, scale=scale)
    assert np.isnan(o_o[:, :, bad]).all()            # the reference: NaN
    assert isapprox(on[:, :, good], o_o[:, :, good], atol=0, rtol=2e-2)
    if dtype == "bf16":
        assert np.isnan(on[:, :, bad]).all()
    else:
        # f16: the softmax of the q·k logits alone (pinned deviation)
        o_qk, _ = orc.attention_fwd(*ref[:3], causal=False, scale=scale)
        assert np.isfinite(on[:, :, bad]).all()
        assert isapprox(on[:, :, bad], o_qk[:, :, bad], atol=0, rtol=2e-2)


# ----------------------------------------------------------------- config 3 at full size
def test_gqa_rope_full_size_kv_head_grads():
    """GQA + RoPE workload (bf16, E=128, L=8192, QH=32, KH=8, B=4, causal):
    dk and dv of one kv head (the sum over its 4 query heads) and the
    gradients through the RoPE backward (w.r.t. the un-rotated q and k)
    against the oracle."""
    import torch

    import nnop
    B, QH, KH, L, E = 4, 32, 8, 8192, 128
    g = torch.Generator(device="cuda")
    g.manual_seed(33)
    mk = lambda *s: torch.randn(*s, device="cuda", dtype=torch.bfloat16, generator=g)  # noqa: E731
    q, k, v, do = mk(B, QH, L, E), mk(B, KH, L, E), mk(B, KH, L, E), mk(B, QH, L, E)
    pos = torch.arange(L, device="cuda", dtype=torch.float32).repeat(B, 1)
    cos, sin = nnop.LlamaRotaryEmbedding(E)(pos)
    qr, kr = nnop.llama_rope(q, k, cos=cos, sin=sin)
    o, lse = nnop._flash_attention(qr, kr, v, causal=True)
    dqr, dkr, dv, _ = nnop.grad_flash_attention(do, o, lse, qr, kr, v, causal=True)
    dq, dk = nnop.grad_llama_rope(dqr, dkr, cos=cos, sin=sin)
    torch.cuda.synchronize()
    b, kvh = 1, 6
    n_rep = QH // KH
    scale = orc.attention_scale(E, "bf16")
    ks, vs = to_np(kr[b:b + 1, kvh:kvh + 1]), to_np(v[b:b + 1, kvh:kvh + 1])
    dk_o = np.zeros_like(ks)
    dv_o = np.zeros_like(vs)
    cos_o, sin_o = to_np(cos[b:b + 1]), to_np(sin[b:b + 1])
    for h in range(kvh * n_rep, (kvh + 1) * n_rep):
        qs, dos = to_np(qr[b:b + 1, h:h + 1]), to_np(do[b:b + 1, h:h + 1])
        dq_h, dk_h, dv_h, _ = orc.attention_bwd(dos, qs, ks, vs, causal=True, scale=scale)
        dk_o += dk_h
        dv_o += dv_h
        if h == kvh * n_rep + 1:
            dq_un, _ = orc.rope_bwd(dq_h, dq_h, cos_o, sin_o)
            check(dict(dq_rope=to_np(dq[b:b + 1, h:h + 1])), dict(dq_rope=dq_un), "bf16", tag="dq through RoPE")
    dk_un, _ = orc.rope_bwd(dk_o, dk_o, cos_o, sin_o)
    check(dict(dk=to_np(dkr[b:b + 1, kvh:kvh + 1]), dv=to_np(dv[b:b + 1, kvh:kvh + 1]),
               dk_rope=to_np(dk[b:b + 1, kvh:kvh + 1])),
          dict(dk=dk_o, dv=dv_o, dk_rope=dk_un), "bf16", tag="kv head grads")


# ----------------------------------------------------------------- config 5 at full size
def _sample_rows(n, count=48, seed=0):
    rng = np.random.default_rng(seed)
    return np.unique(np.concatenate([[0, n - 1], rng.integers(0, n, size=count)]))


def _chunked_weight_grads(fn, dy, x, chunk=4096):
    """Σ over row chunks of the oracle's weight (and bias) gradients: the whole
    job's dw (db) without materialising it all in float64 at once."""
    out = None
    for lo in range(0, x.shape[0], chunk):
        g = fn(dy[lo:lo + chunk], x[lo:lo + chunk])
        out = list(g) if out is None else [a + b for a, b in zip(out, g)]
    return out


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_norms_full_size(dtype):
    import torch

    import nnop
    emb, n = 4096, 65536
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    g = torch.Generator(device="cuda")
    g.manual_seed(55)
    x = torch.randn(n, emb, device="cuda", generator=g).to(tdt)
    dy = torch.randn(n, emb, device="cuda", generator=g).to(tdt)
    w = (1 + 0.1 * torch.randn(emb, device="cuda", generator=g)).to(tdt)
    b = (0.1 * torch.randn(emb, device="cuda", generator=g)).to(tdt)
    rows = _sample_rows(n)
    tol = dict(atol=0, rtol=2e-2) if dtype == "bf16" else dict(atol=0, rtol=1e-5)
    wn, bn = to_np(w), to_np(b)
    xs, dys = to_np(x[rows]), to_np(dy[rows])
    # rms_norm
    y, rstd = nnop._rms_norm(x, w)
    dx, dw = nnop.grad_rms_norm(dy, rstd, x, w)
    torch.cuda.synchronize()
    y_o, rstd_o = orc.rms_norm_fwd(xs, wn)
    dx_o, _ = orc.rms_norm_bwd(dys, xs, wn)
    assert isapprox(to_np(y[rows]), y_o, **tol) and isapprox(to_np(rstd[rows]), rstd_o, **tol)
    assert isapprox(to_np(dx[rows]), dx_o, **tol)
    xa, dya = to_np(x), to_np(dy)
    (dw_o,) = _chunked_weight_grads(lambda d_, x_: orc.rms_norm_bwd(d_, x_, wn)[1:], dya, xa)
    assert isapprox(to_np(dw), dw_o, **tol)
    del y, rstd, dx, dw
    # layer_norm
    y, mu, rs = nnop._layer_norm(x, w, b)
    dx, dw, db = nnop.grad_layer_norm(dy, mu, rs, x, w)
    torch.cuda.synchronize()
    y_o, mu_o, rs_o = orc.layer_norm_fwd(xs, wn, bn)
    assert isapprox(to_np(y[rows]), y_o, **tol)
    assert isapprox(to_np(mu[rows]), mu_o, atol=1e-6, rtol=1e-5) and isapprox(to_np(rs[rows]), rs_o, **tol)
    dx_o, _, _ = orc.layer_norm_bwd(dys, xs, wn)
    assert isapprox(to_np(dx[rows]), dx_o, **tol)
    dw_o, db_o = _chunked_weight_grads(lambda d_, x_: orc.layer_norm_bwd(d_, x_, wn)[1:], dya, xa)
    assert isapprox(to_np(dw), dw_o, **tol) and isapprox(to_np(db), db_o, **tol)


def test_softmax_full_size():
    import torch

    import nnop
    N, cols = 8192, 16384
    g = torch.Generator(device="cuda")
    g.manual_seed(56)
    x = 4 * torch.randn(cols, N, device="cuda", generator=g)
    dy = torch.randn(cols, N, device="cuda", generator=g)
    y = nnop.online_softmax(x)
    dx = nnop.grad_online_softmax(dy, y)
    torch.cuda.synchronize()
    # every row: Σ y = 1 and Σ dx = 0 (float64 sums on the device)
    assert torch.allclose(y.double().sum(dim=1), torch.ones(cols, dtype=torch.float64, device="cuda"), atol=1e-5)
    scale = (dy.double() * y.double()).abs().sum(dim=1)
    assert bool((dx.double().sum(dim=1).abs() <= 1e-5 * scale + 1e-7).all())
    rows = _sample_rows(cols, seed=1)
    xs, dys = to_np(x[rows]), to_np(dy[rows])
    y_o = orc.softmax_fwd(xs)
    assert isapprox(to_np(y[rows]), y_o, atol=0, rtol=1e-5)
    assert isapprox(to_np(dx[rows]), orc.softmax_bwd(dys, to_np(y[rows])), atol=1e-6, rtol=1e-6)
