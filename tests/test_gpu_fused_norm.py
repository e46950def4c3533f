"""GPU parity of the residual add fused into RMSNorm
(nnop_add_rms_norm_fwd / _bwd): h = x + residual, then rms_norm(h), the
composition a transformer block performs around the reference's rms_norm
(src/rms_norm.jl:117-169).  h must equal a separate add bit for bit (the same
rounding); y, rstd, dx (= the gradient of x and of residual) and dw match the
oracle's composition; both the shared-memory ring kernels (16-byte rows) and
the composed fallback (other rows) are covered, with and without the residual
stream's gradient dh."""
import numpy as np
import pytest

from _util import isapprox, to_dev, to_np
from oracle import nnop_oracle as orc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("emb,n", [(4096, 300), (768, 1000), (1001, 37), (8192, 65), (16, 5)])
@pytest.mark.parametrize("with_dh", [True, False])
def test_add_rms_norm_matches_oracle(dtype, emb, n, with_dh):
    import torch

    import nnop
    rng = np.random.default_rng(emb + n)
    x, r, dy, dh = (rng.standard_normal((n, emb)) for _ in range(4))
    w = 1 + 0.1 * rng.standard_normal(emb)
    xd, rd, wd, dyd, dhd = (to_dev(a, dtype) for a in (x, r, w, dy, dh))
    y, h, rstd = nnop._add_rms_norm(xd, rd, wd, offset=0.25)
    dx, dw = nnop.grad_add_rms_norm(dyd, dhd if with_dh else None, h, wd, rstd, offset=0.25)
    torch.cuda.synchronize()
    assert torch.equal(h, xd + rd)                    # the rounding of a separate add
    y_o, h_o, rstd_o = orc.add_rms_norm_fwd(to_np(xd), to_np(rd), to_np(wd), offset=0.25, dtype=dtype)
    dx_o, dw_o = orc.add_rms_norm_bwd(to_np(dyd), to_np(dhd) if with_dh else None, h_o, to_np(wd), offset=0.25)
    tol = dict(atol=0, rtol=1e-5) if dtype == "f32" else dict(atol=0, rtol=2e-2)
    assert isapprox(to_np(y), y_o, **tol) and isapprox(to_np(rstd), rstd_o, **tol)
    assert isapprox(to_np(dx), dx_o, **tol) and isapprox(to_np(dw), dw_o, **tol)


def test_add_rms_norm_autograd():
    import torch

    import nnop
    rng = np.random.default_rng(3)
    n, emb = 64, 4096
    x, r = (to_dev(rng.standard_normal((n, emb)), "bf16").requires_grad_(True) for _ in range(2))
    w = to_dev(1 + 0.1 * rng.standard_normal(emb), "bf16").requires_grad_(True)
    y, h = nnop.add_rms_norm(x, r, w)
    (y.float().sum() + 0.5 * h.float().sum()).backward()
    torch.cuda.synchronize()
    y2, h2, rstd = nnop._add_rms_norm(x.detach(), r.detach(), w.detach())
    dx, dw = nnop.grad_add_rms_norm(torch.ones_like(y2), torch.full_like(h2, 0.5), h2, w.detach(), rstd)
    assert torch.equal(x.grad, dx) and torch.equal(r.grad, dx)
    assert torch.allclose(w.grad.float(), dw.to(torch.bfloat16).float())
