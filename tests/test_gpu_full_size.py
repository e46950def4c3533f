"""Parity at the benchmark workloads' full sizes.

The whole job runs on the GPU at the real size; the CPU oracle (float64) then
checks sampled (batch, head) slices element by element, and size-independent
properties are checked on every element on the device:
* the pair-bias benchmark (bf16, E=64, L=4096, H=16, B=8, causal, pair bias):
  every dpair element above the causal diagonal is exactly zero;
* the variable-length workload (fp16, E=64, H=8, B=16, L=4096, lengths in
  [256, 4096] behind a key mask, pair ~ N(0, 0.5) with −Inf at masked keys):
  dk, dv and dpair of every padded key are exactly zero;
* the GQA workload with RoPE (bf16, E=128, L=8192, QH=32, KH=8, B=4, causal):
  the rotation of q and k, and o, lse, dq of a query head.
Tolerances are those of the small-size tests."""
import numpy as np
import pytest

from _util import to_np
from oracle import nnop_oracle as orc
from test_gpu_attention import check

pytestmark = pytest.mark.gpu


def _slice(t, b, h):
    return to_np(t[b:b + 1, h:h + 1])


def _pair_slice(t, b, h):
    return to_np(t[b:b + 1, :, :, h:h + 1])


def _oracle_slice(q, k, v, pair, do, b, h, kvh, causal, mask, dtype, E):
    qs, ks, vs, dos = _slice(q, b, h), _slice(k, b, kvh), _slice(v, b, kvh), _slice(do, b, h)
    ps = _pair_slice(pair, b, h) if pair is not None else None
    ms = None if mask is None else to_np(mask[b:b + 1]).astype(bool)
    args = dict(causal=causal, kpad_mask=ms, scale=orc.attention_scale(E, dtype))
    o, lse = orc.attention_fwd(qs, ks, vs, ps, **args)
    grads = orc.attention_bwd(dos, qs, ks, vs, ps, **args)
    return o, lse, grads


def test_pair_bias_benchmark_full_size():
    import torch

    import nnop
    B, H, L, E = 8, 16, 4096, 64
    g = torch.Generator(device="cuda")
    g.manual_seed(2024)
    mk = lambda *s: torch.randn(*s, device="cuda", dtype=torch.bfloat16, generator=g)  # noqa: E731
    q, k, v, do = mk(B, H, L, E), mk(B, H, L, E), mk(B, H, L, E), mk(B, H, L, E)
    pair = mk(B, L, L, H)
    o, lse, ws = nnop._flash_attention_ws(q, k, v, pair, causal=True)
    dq, dk, dv, dpair = nnop.grad_flash_attention(do, o, lse, q, k, v, pair, causal=True, fwd_workspace=ws)
    torch.cuda.synchronize()
    assert torch.isfinite(o).all() and torch.isfinite(lse).all()
    upper = torch.tril(torch.ones(L, L, dtype=torch.bool, device="cuda"), diagonal=-1)   # key j > query i
    for b in range(B):
        assert int((dpair[b][upper] != 0).sum()) == 0, b
    for b, h in ((0, 0), (B - 1, H - 1), (3, 7)):
        o_o, lse_o, (dq_o, dk_o, dv_o, dp_o) = _oracle_slice(q, k, v, pair, do, b, h, h, True, None, "bf16", E)
        got = dict(o=_slice(o, b, h), lse=to_np(lse[b:b + 1, h:h + 1]), dq=_slice(dq, b, h), dk=_slice(dk, b, h),
                   dv=_slice(dv, b, h), dpair=_pair_slice(dpair, b, h))
        want = dict(o=o_o, lse=lse_o, dq=dq_o, dk=dk_o, dv=dv_o, dpair=dp_o)
        check(got, want, "bf16", tag=f"b={b} h={h}")


def test_varlen_pair_full_size():
    import torch

    import nnop
    B, H, L, E = 16, 8, 4096, 64
    rng = np.random.default_rng(4)
    lens = rng.integers(256, 4097, size=B)
    g = torch.Generator(device="cuda")
    g.manual_seed(4)
    mk = lambda *s: torch.randn(*s, device="cuda", dtype=torch.float16, generator=g)  # noqa: E731
    q, k, v, do = mk(B, H, L, E), mk(B, H, L, E), mk(B, H, L, E), mk(B, H, L, E)
    pair = (0.5 * torch.randn(B, L, L, H, device="cuda", generator=g)).to(torch.float16)
    mask = torch.zeros(B, L, dtype=torch.bool, device="cuda")
    for b, n in enumerate(lens):
        mask[b, :n] = True
        pair[b, n:] = -float("inf")
    o, lse, ws = nnop._flash_attention_ws(q, k, v, pair, causal=False, kpad_mask=mask)
    dq, dk, dv, dpair = nnop.grad_flash_attention(do, o, lse, q, k, v, pair, causal=False, kpad_mask=mask,
                                                  fwd_workspace=ws)
    torch.cuda.synchronize()
    assert torch.isfinite(o).all()
    for b, n in enumerate(lens):
        if n < L:
            assert int((dk[b, :, n:] != 0).sum()) == 0 and int((dv[b, :, n:] != 0).sum()) == 0, b
            assert int((dpair[b, n:] != 0).sum()) == 0, b
    for b in (int(np.argmin(lens)), int(np.argmax(lens))):
        h = b % H
        o_o, lse_o, (dq_o, dk_o, dv_o, dp_o) = _oracle_slice(q, k, v, pair, do, b, h, h, False, mask, "f16", E)
        got = dict(o=_slice(o, b, h), lse=to_np(lse[b:b + 1, h:h + 1]), dq=_slice(dq, b, h), dk=_slice(dk, b, h),
                   dv=_slice(dv, b, h), dpair=_pair_slice(dpair, b, h))
        want = dict(o=o_o, lse=lse_o, dq=dq_o, dk=dk_o, dv=dv_o, dpair=dp_o)
        check(got, want, "f16", tag=f"b={b} len={lens[b]}")


def test_gqa_rope_full_size():
    import torch

    import nnop
    B, QH, KH, L, E = 4, 32, 8, 8192, 128
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    mk = lambda *s: torch.randn(*s, device="cuda", dtype=torch.bfloat16, generator=g)  # noqa: E731
    q, k, v, do = mk(B, QH, L, E), mk(B, KH, L, E), mk(B, KH, L, E), mk(B, QH, L, E)
    pos = torch.arange(L, device="cuda", dtype=torch.float32).repeat(B, 1)
    cos, sin = nnop.LlamaRotaryEmbedding(E)(pos)
    qr, kr = nnop.llama_rope(q, k, cos=cos, sin=sin)
    o, lse = nnop._flash_attention(qr, kr, v, causal=True)
    dqr, dkr, dv, _ = nnop.grad_flash_attention(do, o, lse, qr, kr, v, causal=True)
    dq, dk = nnop.grad_llama_rope(dqr, dkr, cos=cos, sin=sin)
    torch.cuda.synchronize()
    assert torch.isfinite(o).all() and torch.isfinite(dq).all() and torch.isfinite(dk).all()
    # the rotation of one batch, every head, against the oracle
    cos_o, sin_o = orc.llama_rotary_embedding(E, to_np(pos[:1]))
    qo_o, ko_o = orc.rope_fwd(to_np(q[:1]), to_np(k[:1]), cos_o, sin_o)
    from _util import isapprox
    assert isapprox(to_np(qr[:1]), qo_o, atol=0, rtol=2e-2)
    assert isapprox(to_np(kr[:1]), ko_o, atol=0, rtol=2e-2)
    # attention on the rotated q, k: o, lse, dq of query head 5 (kv head 1)
    b, h = 2, 5
    kvh = h // (QH // KH)
    o_o, lse_o, (dq_o, _, _, _) = _oracle_slice(qr, kr, v, None, do, b, h, kvh, True, None, "bf16", E)
    got = dict(o=_slice(o, b, h), lse=to_np(lse[b:b + 1, h:h + 1]), dq=_slice(dqr, b, h))
    want = dict(o=o_o, lse=lse_o, dq=dq_o)
    check(got, want, "bf16", tag="gqa rope")
