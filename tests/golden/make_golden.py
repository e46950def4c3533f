"""Generates tests/golden/oracle_golden.npz: seeded small inputs and the
oracle's float64 outputs for every op of the hot path.

Run from the repository root: ``python tests/golden/make_golden.py``.
The fixtures freeze the oracle (tests/test_oracle.py re-computes them) and give
the GPU tests inputs whose expected outputs do not depend on the oracle code
of the day.  No reference-produced vectors exist (the reference runs only in
Julia on a GPU and its tests are unseeded), so these are oracle outputs."""
from __future__ import annotations

import pathlib
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import nnop_oracle as orc  # noqa: E402

OUT = pathlib.Path(__file__).resolve().parent / "oracle_golden.npz"


def compute() -> dict:
    d = {}
    rng = np.random.default_rng(2024)
    # attention: B=2, QH=4, KH=2 (GQA), QL=KL=33, E=16, causal + pair + mask, bf16-rounded inputs
    B, QH, KH, L, E = 2, 4, 2, 33, 16
    q = orc.round_to(rng.standard_normal((B, QH, L, E)), "bf16")
    k = orc.round_to(rng.standard_normal((B, KH, L, E)), "bf16")
    v = orc.round_to(rng.standard_normal((B, KH, L, E)), "bf16")
    pair = orc.round_to(rng.standard_normal((B, L, L, QH)), "bf16")
    do = orc.round_to(rng.standard_normal((B, QH, L, E)), "bf16")
    mask = np.ones((B, L), bool)
    mask[-1, -11:] = False
    scale = orc.attention_scale(E, "bf16")
    o, lse = orc.attention_fwd(q, k, v, pair, causal=True, kpad_mask=mask, scale=scale)
    dq, dk, dv, dp = orc.attention_bwd(do, q, k, v, pair, causal=True, kpad_mask=mask, scale=scale)
    d.update(att_q=q, att_k=k, att_v=v, att_pair=pair, att_do=do, att_mask=mask.astype(np.uint8),
             att_o=o, att_lse=lse, att_dq=dq, att_dk=dk, att_dv=dv, att_dpair=dp)
    # softmax (cols=4, n=37)
    x = orc.round_to(4 * rng.standard_normal((4, 37)), "f32")
    dy = orc.round_to(rng.standard_normal((4, 37)), "f32")
    y = orc.softmax_fwd(x)
    d.update(sm_x=x, sm_dy=dy, sm_y=y, sm_dx=orc.softmax_bwd(dy, y))
    # norms (n=5, emb=19)
    x = orc.round_to(rng.standard_normal((5, 19)), "f32")
    w = orc.round_to(1 + 0.1 * rng.standard_normal(19), "f32")
    b = orc.round_to(0.1 * rng.standard_normal(19), "f32")
    dy = orc.round_to(rng.standard_normal((5, 19)), "f32")
    y, rstd = orc.rms_norm_fwd(x, w, offset=1.0)
    dx, dw = orc.rms_norm_bwd(dy, x, w, offset=1.0)
    d.update(nm_x=x, nm_w=w, nm_b=b, nm_dy=dy, rms_y=y, rms_rstd=rstd, rms_dx=dx, rms_dw=dw)
    y, mu, rstd = orc.layer_norm_fwd(x, w, b)
    dx, dw, db = orc.layer_norm_bwd(dy, x, w)
    d.update(ln_y=y, ln_mean=mu, ln_rstd=rstd, ln_dx=dx, ln_dw=dw, ln_db=db)
    # rope (B=1, QH=2, KH=1, L=13, E=16) on the LlamaRotaryEmbedding tables
    cos, sin = orc.llama_rotary_embedding(16, np.arange(13, dtype=np.float32)[None])
    qr = orc.round_to(rng.standard_normal((1, 2, 13, 16)), "f32")
    kr = orc.round_to(rng.standard_normal((1, 1, 13, 16)), "f32")
    q1, k1 = orc.rope_fwd(qr, kr, cos, sin)
    g1, g2 = orc.rope_bwd(qr, kr, cos, sin)
    d.update(rope_cos=cos.astype(np.float64), rope_sin=sin.astype(np.float64), rope_q=qr, rope_k=kr,
             rope_qo=q1, rope_ko=k1, rope_dq=g1, rope_dk=g2)
    return d


if __name__ == "__main__":
    np.savez_compressed(OUT, **compute())
    print(OUT, OUT.stat().st_size, "bytes")
