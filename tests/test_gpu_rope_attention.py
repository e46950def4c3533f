"""GPU parity of Llama RoPE fused with attention (nnop_flash_attention_rope_fwd
/ _bwd): the composition of llama_rope (src/rope/llama_rope.jl:69-98) and
flash_attention, whose backward folds the inverse rotation into the attention
backward's outputs (dq at its fp32-to-dtype conversion, dk in the dK
epilogue).  Checked against the oracle's composition (rope_fwd, attention,
attention_bwd, rope_bwd) and against the unfused calls of this library."""
import numpy as np
import pytest

from _util import to_dev, to_np
from oracle import nnop_oracle as orc
from test_gpu_attention import check

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("E", [64, 128])
@pytest.mark.parametrize("B,QH,KH,L,causal,masked,cos_b", [
    (2, 4, 1, 300, True, False, 2), (1, 8, 2, 513, False, True, 1), (2, 2, 2, 256, True, True, 1),
    (1, 6, 3, 64, False, False, 1)])
def test_rope_attention_matches_oracle(dtype, E, B, QH, KH, L, causal, masked, cos_b):
    import torch

    import nnop
    rng = np.random.default_rng(L + E + QH)
    q, do = rng.standard_normal((B, QH, L, E)), rng.standard_normal((B, QH, L, E))
    k, v = rng.standard_normal((B, KH, L, E)), rng.standard_normal((B, KH, L, E))
    mask = None
    if masked:
        mask = np.ones((B, L), bool)
        mask[-1, L - 37:] = False
    pos = np.stack([np.arange(L, dtype=np.float32) + 3 * b for b in range(cos_b)])
    qd, kd, vd, dod = (to_dev(a, dtype) for a in (q, k, v, do))
    md = torch.from_numpy(mask).cuda() if masked else None
    cos, sin = nnop.LlamaRotaryEmbedding(E)(torch.from_numpy(pos).cuda())
    o, lse, qr, kr = nnop._flash_attention_rope(qd, kd, vd, cos=cos, sin=sin, causal=causal, kpad_mask=md)
    dq, dk, dv = nnop.grad_flash_attention_rope(dod, o, lse, qr, kr, vd, cos=cos, sin=sin, causal=causal,
                                                kpad_mask=md)
    # the unfused calls on the same tensors
    qr2, kr2 = nnop.llama_rope(qd, kd, cos=cos, sin=sin)
    o2, lse2 = nnop._flash_attention(qr2, kr2, vd, causal=causal, kpad_mask=md)
    g2 = nnop.grad_flash_attention(dod, o2, lse2, qr2, kr2, vd, causal=causal, kpad_mask=md)
    torch.cuda.synchronize()
    assert torch.equal(qr, qr2) and torch.equal(kr, kr2) and torch.equal(o, o2) and torch.equal(g2[2], dv)
    # oracle: rope, attention, attention backward, inverse rope
    cos_o, sin_o = to_np(cos), to_np(sin)
    if cos_b == 1 and B > 1:
        cos_o, sin_o = np.repeat(cos_o, B, axis=0), np.repeat(sin_o, B, axis=0)
    qr_o, kr_o = orc.rope_fwd(to_np(qd), to_np(kd), cos_o, sin_o)
    check(dict(q_rot=to_np(qr), k_rot=to_np(kr)), dict(q_rot=qr_o, k_rot=kr_o), dtype, tag="rotation")
    qr_o, kr_o = to_np(qr), to_np(kr)               # attention on the stored (rounded) rotations
    args = dict(causal=causal, kpad_mask=mask, scale=orc.attention_scale(E, dtype))
    o_o, lse_o = orc.attention_fwd(qr_o, kr_o, to_np(vd), **args)
    dqr_o, dkr_o, dv_o, _ = orc.attention_bwd(to_np(dod), qr_o, kr_o, to_np(vd), **args)
    dq_o, dk_o = orc.rope_bwd(dqr_o, dkr_o, cos_o, sin_o)
    check(dict(o=to_np(o), lse=to_np(lse), dq=to_np(dq), dk=to_np(dk), dv=to_np(dv)),
          dict(o=o_o, lse=lse_o, dq=dq_o, dk=dk_o, dv=dv_o), dtype, tag=f"E={E} L={L}")


def test_rope_attention_gqa_full_size():
    """The GQA + RoPE workload (bf16, E=128, L=8192, QH=32, KH=8, B=4, causal)
    through the fused entry points: dk of one kv head and dq of one query head
    against the oracle's composition."""
    import torch

    import nnop
    B, QH, KH, L, E = 4, 32, 8, 8192, 128
    g = torch.Generator(device="cuda").manual_seed(34)
    mk = lambda *s: torch.randn(*s, device="cuda", dtype=torch.bfloat16, generator=g)  # noqa: E731
    q, k, v, do = mk(B, QH, L, E), mk(B, KH, L, E), mk(B, KH, L, E), mk(B, QH, L, E)
    pos = torch.arange(L, device="cuda", dtype=torch.float32).repeat(B, 1)
    cos, sin = nnop.LlamaRotaryEmbedding(E)(pos)
    o, lse, qr, kr = nnop._flash_attention_rope(q, k, v, cos=cos, sin=sin, causal=True)
    dq, dk, dv = nnop.grad_flash_attention_rope(do, o, lse, qr, kr, v, cos=cos, sin=sin, causal=True)
    torch.cuda.synchronize()
    b, kvh = 3, 2
    scale = orc.attention_scale(E, "bf16")
    cos_o, sin_o = to_np(cos[b:b + 1]), to_np(sin[b:b + 1])
    ks, vs = to_np(kr[b:b + 1, kvh:kvh + 1]), to_np(v[b:b + 1, kvh:kvh + 1])
    dk_r = np.zeros_like(ks)
    for h in range(kvh * 4, kvh * 4 + 4):
        qs, dos = to_np(qr[b:b + 1, h:h + 1]), to_np(do[b:b + 1, h:h + 1])
        dq_h, dk_h, _, _ = orc.attention_bwd(dos, qs, ks, vs, causal=True, scale=scale)
        dk_r += dk_h
        if h == kvh * 4:
            dq_u, _ = orc.rope_bwd(dq_h, dq_h, cos_o, sin_o)
            check(dict(dq=to_np(dq[b:b + 1, h:h + 1])), dict(dq=dq_u), "bf16", tag="dq")
    _, dk_u = orc.rope_bwd(dk_r, dk_r, cos_o, sin_o)
    check(dict(dk=to_np(dk[b:b + 1, kvh:kvh + 1])), dict(dk=dk_u), "bf16", tag="dk")


def test_rope_attention_errors():
    import torch

    import nnop
    z = lambda *s, dt=torch.bfloat16: torch.zeros(*s, device="cuda", dtype=dt)  # noqa: E731
    cos = torch.zeros(1, 64, 32, device="cuda")
    with pytest.raises(nnop.NNopShapeError, match="E = 64 or 128"):
        nnop.flash_attention_rope(z(1, 2, 64, 32), z(1, 2, 64, 32), z(1, 2, 64, 32), cos=cos, sin=cos, causal=True)
    cos = torch.zeros(1, 64, 64, device="cuda")
    with pytest.raises(nnop.NNopError, match="bf16 or f16"):
        f = torch.float32
        nnop.flash_attention_rope(z(1, 2, 64, 64, dt=f), z(1, 2, 64, 64, dt=f), z(1, 2, 64, 64, dt=f), cos=cos,
                                  sin=cos, causal=True)
