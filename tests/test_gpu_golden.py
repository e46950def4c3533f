"""GPU outputs on the frozen golden inputs (tests/golden/oracle_golden.npz)."""
import pathlib

import numpy as np
import pytest

from _util import isapprox, to_dev, to_np

pytestmark = pytest.mark.gpu
G = np.load(pathlib.Path(__file__).parent / "golden" / "oracle_golden.npz")


def test_golden_attention_bf16():
    import nnop
    import torch
    q, k, v, pair, do = (to_dev(G[f"att_{n}"], "bf16") for n in ("q", "k", "v", "pair", "do"))
    mask = torch.from_numpy(G["att_mask"].astype(bool)).cuda()
    o, lse = nnop._flash_attention(q, k, v, pair, causal=True, kpad_mask=mask)
    dq, dk, dv, dp = nnop.grad_flash_attention(do, o, lse, q, k, v, pair, causal=True, kpad_mask=mask)
    for got, key in ((o, "o"), (lse, "lse"), (dq, "dq"), (dk, "dk"), (dv, "dv"), (dp, "dpair")):
        assert isapprox(to_np(got), G[f"att_{key}"], atol=0, rtol=2e-2), key


def test_golden_softmax_norms_rope_f32():
    import nnop
    x, dy = to_dev(G["sm_x"], "f32"), to_dev(G["sm_dy"], "f32")
    y = nnop.online_softmax(x)
    assert isapprox(to_np(y), G["sm_y"], atol=0, rtol=1e-6)
    assert isapprox(to_np(nnop.grad_online_softmax(dy, y)), G["sm_dx"], atol=1e-6, rtol=1e-6)

    x, w, b, dy = (to_dev(G[f"nm_{n}"], "f32") for n in ("x", "w", "b", "dy"))
    y, rstd = nnop._rms_norm(x, w, offset=1.0)
    dx, dw = nnop.grad_rms_norm(dy, rstd, x, w, offset=1.0)
    for got, key in ((y, "rms_y"), (rstd, "rms_rstd"), (dx, "rms_dx"), (dw, "rms_dw")):
        assert isapprox(to_np(got), G[key], atol=1e-6, rtol=1e-6), key
    y, mu, rstd = nnop._layer_norm(x, w, b)
    dx, dw, db = nnop.grad_layer_norm(dy, mu, rstd, x, w)
    for got, key in ((y, "ln_y"), (mu, "ln_mean"), (rstd, "ln_rstd"), (dx, "ln_dx"), (dw, "ln_dw"), (db, "ln_db")):
        assert isapprox(to_np(got), G[key], atol=1e-6, rtol=1e-6), key

    cos, sin = nnop.LlamaRotaryEmbedding(16)(np.arange(13, dtype=np.float32)[None])
    assert isapprox(to_np(cos), G["rope_cos"], atol=1e-6, rtol=1e-6)
    assert isapprox(to_np(sin), G["rope_sin"], atol=1e-6, rtol=1e-6)
    q, k = to_dev(G["rope_q"], "f32"), to_dev(G["rope_k"], "f32")
    qo, ko = nnop.llama_rope(q, k, cos=cos, sin=sin)
    assert isapprox(to_np(qo), G["rope_qo"], atol=1e-6, rtol=1e-6)
    assert isapprox(to_np(ko), G["rope_ko"], atol=1e-6, rtol=1e-6)
    gq, gk = nnop.grad_llama_rope(q, k, cos=cos, sin=sin)
    assert isapprox(to_np(gq), G["rope_dq"], atol=1e-6, rtol=1e-6)
    assert isapprox(to_np(gk), G["rope_dk"], atol=1e-6, rtol=1e-6)
