"""GPU parity of the per-head pair-bias entry points
(nnop_flash_attention_{fwd,bwd}_pair_per_head): the pair bias and dpair laid
out per head, torch (B, QH, KL, QL) = Julia (QL, KL, QH, B), read and written
in place by the tensor-core kernels.

The reference's attention (src/attention.jl:72, src/attention_bwd.jl:247-252)
takes the bias head-innermost; these entry points compute the same function
on the same values in another layout, so every case is checked against the
oracle (on the bias permuted to the reference layout) and against the drop-in
entry points, whose o, lse, dk, dv and dpair they must equal bit for bit (dq
aside: its fp32 reductions land in any order)."""
import numpy as np
import pytest

from _util import to_dev, to_np
from oracle import nnop_oracle as orc
from test_gpu_attention import check

pytestmark = pytest.mark.gpu


def _case(B, QH, KH, QL, KL, dtype, causal, kept, seed):
    import torch

    import nnop
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, QH, QL, 64))
    k, v = rng.standard_normal((B, KH, KL, 64)), rng.standard_normal((B, KH, KL, 64))
    do = rng.standard_normal((B, QH, QL, 64))
    pair = rng.standard_normal((B, KL, QL, QH))          # reference layout
    mask = None
    if kept is not None:
        mask = np.zeros((B, KL), bool)
        for b, n in enumerate(kept):
            mask[b, :n] = True
            pair[b, n:] = -np.inf                         # the varlen workload's convention
    qd, kd, vd, dod, pd = (to_dev(a, dtype) for a in (q, k, v, do, pair))
    md = torch.from_numpy(mask).cuda() if mask is not None else None
    ph = pd.permute(0, 3, 1, 2).contiguous()             # per head (B, QH, KL, QL)
    o, lse = nnop._flash_attention_pair_per_head(qd, kd, vd, ph, causal=causal, kpad_mask=md)
    dq, dk, dv, dph = nnop.grad_flash_attention_pair_per_head(dod, o, lse, qd, kd, vd, ph, causal=causal,
                                                              kpad_mask=md)
    # the drop-in entry points on the same values
    o2, lse2, ws = nnop._flash_attention_ws(qd, kd, vd, pd, causal=causal, kpad_mask=md)
    g2 = nnop.grad_flash_attention(dod, o2, lse2, qd, kd, vd, pd, causal=causal, kpad_mask=md, fwd_workspace=ws)
    torch.cuda.synchronize()
    dpair = dph.permute(0, 2, 3, 1)                      # back to the reference layout
    got = dict(o=to_np(o), lse=to_np(lse), dq=to_np(dq), dk=to_np(dk), dv=to_np(dv), dpair=to_np(dpair))
    same = dict(o=to_np(o2), lse=to_np(lse2), dk=to_np(g2[1]), dv=to_np(g2[2]), dpair=to_np(g2[3]))
    args = dict(causal=causal, kpad_mask=mask, scale=orc.attention_scale(64, dtype))
    ref = [to_np(t) for t in (qd, kd, vd, pd, dod)]
    o_o, lse_o = orc.attention_fwd(*ref[:4], **args)
    dq_o, dk_o, dv_o, dp_o = orc.attention_bwd(ref[4], *ref[:4], **args)
    want = dict(o=o_o, lse=lse_o, dq=dq_o, dk=dk_o, dv=dv_o, dpair=dp_o)
    return got, want, same


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("B,QH,KH,QL,KL,causal,kept", [
    (2, 4, 4, 256, 256, True, None),
    (2, 4, 2, 296, 421, False, [421, 130]),
    (1, 8, 2, 512, 512, True, [512]),
    (3, 2, 2, 64, 200, False, None),
    (1, 2, 1, 8, 70, True, [70]),
    (2, 3, 3, 1024, 1024, True, [1000, 77]),
    (1, 2, 2, 136, 300, False, [1]),
])
def test_pair_per_head_matches_oracle_and_drop_in(dtype, B, QH, KH, QL, KL, causal, kept):
    got, want, same = _case(B, QH, KH, QL, KL, dtype, causal, kept, seed=QL + KL + QH)
    check(got, want, dtype, tag=f"QL={QL} KL={KL} causal={causal}")
    for name, ref in same.items():
        assert np.array_equal(got[name], ref, equal_nan=True), name


def test_pair_per_head_dpair_zero_where_masked():
    """Called through the C ABI with a dpair buffer full of NaN: every entry
    above the causal diagonal and at padded keys comes back exactly zero and
    every other entry finite -- each element is written."""
    import torch

    import nnop
    from nnop._lib import lib
    B, H, L = 2, 4, 640
    g = torch.Generator(device="cuda").manual_seed(9)
    mk = lambda *s: torch.randn(*s, device="cuda", dtype=torch.bfloat16, generator=g)  # noqa: E731
    q, k, v, do = mk(B, H, L, 64), mk(B, H, L, 64), mk(B, H, L, 64), mk(B, H, L, 64)
    ph = mk(B, H, L, L)
    mask = torch.ones(B, L, dtype=torch.bool, device="cuda")
    mask[1, 300:] = False
    m8 = mask.view(torch.uint8)
    o, lse = nnop._flash_attention_pair_per_head(q, k, v, ph, causal=True, kpad_mask=mask)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dph = torch.full_like(ph, float("nan"))
    nws = lib.nnop_flash_attention_bwd_pair_per_head_workspace_size(64, L, L, H, H, B, 2)
    ws = torch.empty(nws, dtype=torch.uint8, device="cuda")
    st = lib.nnop_flash_attention_bwd_pair_per_head(
        do.data_ptr(), o.data_ptr(), lse.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), ph.data_ptr(),
        m8.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dph.data_ptr(), ws.data_ptr(), nws,
        64, L, L, H, H, B, 1, 2, torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.nnop_last_error()
    torch.cuda.synchronize()
    assert bool(torch.isfinite(dph).all())
    upper = torch.triu(torch.ones(L, L, dtype=torch.bool, device="cuda"), diagonal=1)   # key j > query i
    assert int((dph.transpose(2, 3)[:, :, upper] != 0).sum()) == 0
    assert int((dph[1, :, 300:] != 0).sum()) == 0
    assert int((dph[0] != 0).sum()) > 0


def test_pair_per_head_autograd():
    import torch

    import nnop
    rng = np.random.default_rng(12)
    B, H, L = 2, 4, 200
    ts = [to_dev(rng.standard_normal(s), "bf16").requires_grad_(True)
          for s in ((B, H, L, 64), (B, H, L, 64), (B, H, L, 64), (B, H, L, L))]
    o = nnop.flash_attention_pair_per_head(*ts, causal=True)
    o.sum().backward()
    torch.cuda.synchronize()
    qd, kd, vd, ph = (t.detach() for t in ts)
    o2, lse = nnop._flash_attention_pair_per_head(qd, kd, vd, ph, causal=True)
    dq, dk, dv, dph = nnop.grad_flash_attention_pair_per_head(torch.ones_like(o2), o2, lse, qd, kd, vd, ph,
                                                              causal=True)
    assert torch.equal(o.detach(), o2)
    assert torch.equal(ts[1].grad, dk) and torch.equal(ts[2].grad, dv) and torch.equal(ts[3].grad, dph)
    assert torch.allclose(ts[0].grad.float(), dq.float(), rtol=1e-2, atol=1e-2)   # dq: reductions in any order


def test_pair_per_head_errors():
    import torch

    import nnop
    z = lambda *s, dt=torch.bfloat16: torch.zeros(*s, device="cuda", dtype=dt)  # noqa: E731
    with pytest.raises(nnop.NNopShapeError, match="E = 64"):
        nnop.flash_attention_pair_per_head(z(1, 2, 64, 128), z(1, 2, 64, 128), z(1, 2, 64, 128), z(1, 2, 64, 64),
                                           causal=False)
    with pytest.raises(nnop.NNopShapeError, match="multiple of 8"):
        nnop.flash_attention_pair_per_head(z(1, 2, 60, 64), z(1, 2, 64, 64), z(1, 2, 64, 64), z(1, 2, 64, 60),
                                           causal=False)
    with pytest.raises(nnop.NNopError, match="bf16 or f16"):
        f = torch.float32
        nnop.flash_attention_pair_per_head(z(1, 2, 64, 64, dt=f), z(1, 2, 64, 64, dt=f), z(1, 2, 64, 64, dt=f),
                                           z(1, 2, 64, 64, dt=f), causal=False)
    with pytest.raises(nnop.NNopShapeError, match="pair must have shape"):
        nnop.flash_attention_pair_per_head(z(1, 2, 64, 64), z(1, 2, 64, 64), z(1, 2, 64, 64), z(1, 64, 64, 2),
                                           causal=False)


def test_pair_per_head_benchmark_full_size():
    """The pair-bias benchmark (bf16, E=64, L=4096, H=16, B=8, causal) through the
    per-head entry points: every dpair element above the causal diagonal is
    exactly zero, every element finite, and sampled (batch, head) slices match
    the oracle element by element."""
    import torch

    import nnop
    B, H, L, E = 8, 16, 4096, 64
    g = torch.Generator(device="cuda").manual_seed(2025)
    mk = lambda *s: torch.randn(*s, device="cuda", dtype=torch.bfloat16, generator=g)  # noqa: E731
    q, k, v, do = mk(B, H, L, E), mk(B, H, L, E), mk(B, H, L, E), mk(B, H, L, E)
    ph = mk(B, H, L, L)
    o, lse = nnop._flash_attention_pair_per_head(q, k, v, ph, causal=True)
    dq, dk, dv, dph = nnop.grad_flash_attention_pair_per_head(do, o, lse, q, k, v, ph, causal=True)
    torch.cuda.synchronize()
    upper = torch.triu(torch.ones(L, L, dtype=torch.bool, device="cuda"), diagonal=1)   # [query][key], key > query
    for b in range(B):
        assert bool(torch.isfinite(dph[b]).all())
        assert int((dph[b].transpose(1, 2)[:, upper] != 0).sum()) == 0, b
    scale = orc.attention_scale(E, "bf16")
    for b, h in ((0, 0), (B - 1, H - 1), (5, 9)):
        sl = lambda t: to_np(t[b:b + 1, h:h + 1])  # noqa: E731
        pair_ref = np.transpose(sl(ph), (0, 2, 3, 1))        # (1, KL, QL, 1)
        o_o, lse_o = orc.attention_fwd(sl(q), sl(k), sl(v), pair_ref, causal=True, scale=scale)
        dq_o, dk_o, dv_o, dp_o = orc.attention_bwd(sl(do), sl(q), sl(k), sl(v), pair_ref, causal=True, scale=scale)
        got = dict(o=sl(o), lse=to_np(lse[b:b + 1, h:h + 1]), dq=sl(dq), dk=sl(dk), dv=sl(dv),
                   dpair=np.transpose(sl(dph), (0, 2, 3, 1)))
        check(got, dict(o=o_o, lse=lse_o, dq=dq_o, dk=dk_o, dv=dv_o, dpair=dp_o), "bf16", tag=f"b={b} h={h}")
