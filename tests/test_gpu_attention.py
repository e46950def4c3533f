"""GPU parity of flash attention (forward + backward) against the CPU oracle.

Grids follow the reference's tests -- test/attention_tests.jl (pad mask × pair ×
dtype × E × QL × KL, H=2, B=3), test/causal_attention_tests.jl and
test/gqa_attention_tests.jl -- extended with bf16 and E=128, which the
reference does not test.  Each case checks o, dq, dk, dv and dpair at two
tolerances, both norm-based (Julia isapprox):
* the reference's own: atol=rtol=1e-3 (fp32), 1e-1 (f16/bf16);
* this implementation's parity target: ≤1e-5 relative (fp32), ≤2e-2 relative (f16/bf16)."""
import numpy as np
import pytest

from _util import isapprox, to_dev, to_np
from oracle import nnop_oracle as orc

pytestmark = pytest.mark.gpu

REF_TOL = {"f32": 1e-3, "f16": 1e-1, "bf16": 1e-1}
TARGET = {"f32": 1e-5, "f16": 2e-2, "bf16": 2e-2}
ABS_FLOOR = {"f32": 1e-6, "f16": 1e-3, "bf16": 1e-3}


def run_case(B, QH, KH, QL, KL, E, dtype, causal, use_pair, use_mask, seed=0, dO_ones=False,
             mask_fn=None, pair_scale=1.0, reuse=False, pair_fn=None):
    import nnop
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, QH, QL, E)).astype(np.float32)
    k = rng.standard_normal((B, KH, KL, E)).astype(np.float32)
    v = rng.standard_normal((B, KH, KL, E)).astype(np.float32)
    do = np.ones((B, QH, QL, E), np.float32) if dO_ones else rng.standard_normal((B, QH, QL, E)).astype(np.float32)
    pair = (pair_scale * rng.standard_normal((B, KL, QL, QH))).astype(np.float32) if use_pair else None
    if pair_fn is not None:
        pair_fn(pair, rng)
    mask = None
    if use_mask:
        mask = np.ones((B, KL), bool)
        if mask_fn is None:
            # test/attention_tests.jl:27-28 masks the last 11 keys of the last
            # batch; short sequences keep at least one key.
            mask[-1, KL - min(11, KL - 1):] = False
        else:
            mask_fn(mask, pair)
    qd, kd, vd, dod = (to_dev(a, dtype) for a in (q, k, v, do))
    pd = to_dev(pair, dtype) if use_pair else None
    import torch
    md = torch.from_numpy(mask).cuda() if use_mask else None
    if reuse:
        o, lse, ws = nnop._flash_attention_ws(qd, kd, vd, pd, causal=causal, kpad_mask=md)
        dq, dk, dv, dpair = nnop.grad_flash_attention(dod, o, lse, qd, kd, vd, pd, causal=causal, kpad_mask=md,
                                                      fwd_workspace=ws)
    else:
        o, lse = nnop._flash_attention(qd, kd, vd, pd, causal=causal, kpad_mask=md)
        dq, dk, dv, dpair = nnop.grad_flash_attention(dod, o, lse, qd, kd, vd, pd, causal=causal, kpad_mask=md)
    torch.cuda.synchronize()
    scale = orc.attention_scale(E, dtype)
    args = dict(causal=causal, kpad_mask=mask, scale=scale)
    qr, kr, vr, dor = (to_np(a) for a in (qd, kd, vd, dod))
    pr = to_np(pd) if use_pair else None
    o_o, lse_o = orc.attention_fwd(qr, kr, vr, pr, **args)
    dq_o, dk_o, dv_o, dp_o = orc.attention_bwd(dor, qr, kr, vr, pr, **args)
    got = dict(o=to_np(o), lse=to_np(lse), dq=to_np(dq), dk=to_np(dk), dv=to_np(dv))
    want = dict(o=o_o, lse=lse_o, dq=dq_o, dk=dk_o, dv=dv_o)
    if use_pair:
        got["dpair"] = to_np(dpair)
        want["dpair"] = dp_o
    else:
        assert dpair is None
    return got, want


def check(got, want, dtype, tag=""):
    for name in got:
        g, w = got[name], want[name]
        assert g.shape == w.shape, (name, g.shape, w.shape)
        assert np.array_equal(np.isnan(g), np.isnan(w)), f"{tag} {name}: NaN pattern differs"
        fin = ~np.isnan(w)
        g, w = g[fin], w[fin]
        tol = REF_TOL[dtype]
        assert isapprox(g, w, atol=tol, rtol=tol), f"{tag} {name}: reference tolerance"
        err = orc.rel_err(g, w)
        # Relative error of a tensor that is analytically zero (e.g. dq when a
        # row sees a single key) compares rounding noise with rounding noise;
        # there an absolute floor applies: RMS error per element ≤ ABS_FLOOR.
        floor = ABS_FLOOR[dtype] * np.sqrt(max(g.size, 1))
        ok = err <= TARGET[dtype] or np.linalg.norm(g - w) <= floor
        assert ok, f"{tag} {name}: rel err {err:.3e} > {TARGET[dtype]} (max abs {orc.max_abs_err(g, w):.3e})"


# test/attention_tests.jl grid (non-causal), reduced over (QL, KL) pairs
@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("E", [16, 32, 64, 128])
@pytest.mark.parametrize("use_pair", [False, True])
@pytest.mark.parametrize("use_mask", [False, True])
def test_attention_noncausal(dtype, E, use_pair, use_mask):
    for (QL, KL) in [(255, 511), (256, 256), (1024, 255), (511, 1024)]:
        got, want = run_case(3, 2, 2, QL, KL, E, dtype, False, use_pair, use_mask, seed=QL + KL + E)
        check(got, want, dtype, tag=f"QL={QL} KL={KL}")


# test/causal_attention_tests.jl grid
@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("E", [16, 32, 64, 128])
@pytest.mark.parametrize("use_pair", [False, True])
@pytest.mark.parametrize("use_mask", [False, True])
def test_attention_causal(dtype, E, use_pair, use_mask):
    for L in (255, 256, 511, 1024):
        got, want = run_case(3, 2, 2, L, L, E, dtype, True, use_pair, use_mask, seed=L + E)
        check(got, want, dtype, tag=f"L={L}")


# test/gqa_attention_tests.jl grid
@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("QH,KVH", [(4, 1), (4, 2), (6, 1), (6, 2), (8, 1), (8, 2)])
@pytest.mark.parametrize("causal", [False, True])
def test_attention_gqa(dtype, QH, KVH, causal):
    for E in (32, 64):
        for L in (255, 256, 257, 512):
            got, want = run_case(2, QH, KVH, L, L, E, dtype, causal, False, False, seed=QH * 10 + KVH + L)
            check(got, want, dtype, tag=f"E={E} L={L}")


# E = 128 without a pair bias: the GQA workload's shape family (tcgen05 backward
# with E on the TMEM lanes for dQ), causal and not, ragged lengths, key mask
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("QH,KVH", [(4, 1), (8, 2), (6, 3), (2, 2)])
@pytest.mark.parametrize("causal", [False, True])
def test_attention_gqa_e128(dtype, QH, KVH, causal):
    for (QL, KL, use_mask) in [(255, 255, False), (256, 256, True), (513, 513, False), (100, 300, True),
                               (300, 100, False), (64, 64, False), (1, 129, True)]:
        if causal and QL != KL and (QL, KL) != (100, 300):
            continue
        got, want = run_case(2, QH, KVH, QL, KL, 128, dtype, causal, False, use_mask, seed=QH * 100 + QL + KL)
        check(got, want, dtype, tag=f"QL={QL} KL={KL} mask={use_mask}")


def test_attention_gqa_e128_pair_mask():
    for dtype in ("bf16", "f16", "f32"):
        got, want = run_case(2, 8, 2, 300, 300, 128, dtype, True, True, True, seed=5)
        check(got, want, dtype)


def test_attention_causal_ragged_lengths():
    """QL != KL under the causal mask (key j visible to query i iff j <= i)."""
    for dtype in ("bf16", "f32"):
        for QL, KL in [(100, 300), (300, 100), (1, 64), (65, 1)]:
            got, want = run_case(1, 2, 1, QL, KL, 64, dtype, True, True, True, seed=QL * KL)
            check(got, want, dtype, tag=f"QL={QL} KL={KL}")


def test_attention_varlen_masked_tiles():
    """Key-padding masks that blank whole key tiles (the varlen workload's shape,
    small): pair is −Inf on padded keys like the config."""
    def mask_fn(mask, pair):
        B, KL = mask.shape
        for b, n in enumerate([17, 200, 64, 129][:B]):
            mask[b, n:] = False
            if pair is not None:
                pair[b, n:, :, :] = -np.inf
    for dtype in ("f16", "bf16", "f32"):
        got, want = run_case(4, 4, 4, 256, 256, 64, dtype, False, True, True, seed=9, mask_fn=mask_fn,
                             pair_scale=0.5)
        check(got, want, dtype)


def test_attention_fully_masked_batch_gives_nan():
    """A batch whose keys are all masked has no valid key: o is NaN for all its
    rows, like the reference's naive softmax of an all −Inf column."""
    def mask_fn(mask, pair):
        mask[0, :] = False
    import nnop
    import torch
    rng = np.random.default_rng(3)
    B, H, L, E = 2, 2, 70, 32
    q, k, v = (torch.from_numpy(rng.standard_normal((B, H, L, E)).astype(np.float32)).cuda().half() for _ in range(3))
    m = torch.ones(B, L, dtype=torch.bool, device="cuda")
    m[0] = False
    o = nnop.flash_attention(q, k, v, causal=False, kpad_mask=m)
    assert torch.isnan(o[0]).all()
    assert not torch.isnan(o[1]).any()


def test_attention_grad_of_sum_dO_ones():
    """The benchmark measures ∇ sum(o) (dO = ones)."""
    for dtype in ("bf16", "f32"):
        got, want = run_case(2, 4, 4, 512, 512, 64, dtype, False, False, False, seed=1, dO_ones=True)
        check(got, want, dtype)


def test_attention_tiny_shapes():
    for dtype in ("bf16", "f16", "f32"):
        for (QL, KL, E) in [(1, 1, 16), (3, 5, 16), (64, 64, 128), (65, 129, 32)]:
            got, want = run_case(1, 1, 1, QL, KL, E, dtype, False, True, True, seed=QL + KL)
            check(got, want, dtype, tag=f"{QL}x{KL}x{E}")


def test_attention_autograd_api():
    """flash_attention under autograd (the rrule path) equals grad_flash_attention."""
    import nnop
    import torch
    rng = np.random.default_rng(2)
    B, H, L, E = 2, 4, 200, 64
    mk = lambda *s: torch.from_numpy(rng.standard_normal(s).astype(np.float32)).cuda().bfloat16().requires_grad_()
    q, k, v = mk(B, H, L, E), mk(B, H, L, E), mk(B, H, L, E)
    pair = mk(B, L, L, H)
    o = nnop.flash_attention(q, k, v, pair, causal=True)
    o.sum().backward()
    o2, lse = nnop._flash_attention(q.detach(), k.detach(), v.detach(), pair.detach(), causal=True)
    g = nnop.grad_flash_attention(torch.ones_like(o2), o2, lse, q.detach(), k.detach(), v.detach(), pair.detach(),
                                  causal=True)
    for a, b in zip((q.grad, k.grad, v.grad, pair.grad), g):
        assert torch.equal(a, b)


def test_attention_errors():
    import nnop
    import torch
    q = torch.zeros(1, 3, 8, 48, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(nnop.NNopShapeError, match="power-of-2"):
        nnop.flash_attention(q, q, q, causal=False)
    q = torch.zeros(1, 3, 8, 64, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(1, 2, 8, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(nnop.NNopShapeError, match="divisible"):
        nnop.flash_attention(q, k, k, causal=False)
    with pytest.raises(nnop.NNopShapeError, match="Shapes of K"):
        nnop.flash_attention(q, k, torch.zeros(1, 2, 9, 64, device="cuda", dtype=torch.bfloat16), causal=False)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_attention_bwd_reuses_forward_tiles(dtype):
    """nnop_flash_attention_bwd_reuse: the backward reads the pair tiles the
    forward left in its workspace; results equal the rebuilding backward's
    bit for bit (dq aside: its fp32 reductions land in any order) and match
    the oracle (causal, padding mask, GQA, ragged)."""
    for (B, QH, KH, QL, KL, causal, use_mask) in [(2, 4, 2, 300, 421, False, True), (2, 4, 4, 257, 257, True, True),
                                                  (1, 8, 2, 513, 300, True, False), (1, 2, 2, 128, 128, False, False)]:
        kw = dict(seed=QL + KL, use_pair=True, use_mask=use_mask)
        got_r, want = run_case(B, QH, KH, QL, KL, 64, dtype, causal, reuse=True, **kw)
        got_n, _ = run_case(B, QH, KH, QL, KL, 64, dtype, causal, reuse=False, **kw)
        for name in got_r:
            if name != "dq":
                assert np.array_equal(got_r[name], got_n[name], equal_nan=True), name
        check(got_r, want, dtype, tag=f"QL={QL} KL={KL} causal={causal}")


def test_attention_pair_neg_inf_entries():
    """−Inf pair entries scattered through rows that keep finite scores: each
    such logit is masked exactly (probability 0, dpair 0), as in the
    reference, on the tensor-core path whose pair bias goes through an
    identity UMMA."""
    def pair_fn(pair, rng):
        pair[rng.random(pair.shape) < 0.2] = -np.inf
        pair[:, 0, :, :] = 0.0   # key 0 stays finite for every query
    for dtype in ("bf16", "f16", "f32"):
        for causal in (False, True):
            got, want = run_case(2, 4, 4, 200, 200, 64, dtype, causal, True, False, seed=21, pair_fn=pair_fn)
            check(got, want, dtype, tag=f"causal={causal}")


def test_attention_autograd_pair_bf16():
    """flash_attention under autograd (the rrule: forward keeps its workspace,
    the pullback reuses the pair tiles) against the oracle."""
    import nnop
    import torch
    rng = np.random.default_rng(77)
    B, H, L, E = 2, 4, 300, 64
    q, k, v, do = (rng.standard_normal((B, H, L, E)).astype(np.float32) for _ in range(4))
    pair = rng.standard_normal((B, L, L, H)).astype(np.float32)
    ts = [to_dev(a, "bf16").requires_grad_(True) for a in (q, k, v, pair)]
    o = nnop.flash_attention(*ts[:3], ts[3], causal=True)
    o.backward(to_dev(do, "bf16"))
    torch.cuda.synchronize()
    qr, kr, vr, pr = (to_np(t.detach()) for t in ts)
    dor = to_np(to_dev(do, "bf16"))
    scale = orc.attention_scale(E, "bf16")
    o_o, lse_o = orc.attention_fwd(qr, kr, vr, pr, causal=True, scale=scale)
    grads = orc.attention_bwd(dor, qr, kr, vr, pr, causal=True, scale=scale)
    got = dict(o=to_np(o.detach()), dq=to_np(ts[0].grad), dk=to_np(ts[1].grad), dv=to_np(ts[2].grad),
               dpair=to_np(ts[3].grad))
    want = dict(o=o_o, dq=grads[0], dk=grads[1], dv=grads[2], dpair=grads[3])
    check(got, want, "bf16")
