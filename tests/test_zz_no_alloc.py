"""The allocation-free RMSNorm backward (nnop_rms_norm_bwd_noalloc).

Callers that cannot allocate device memory at the call site (a memory pool's
own callbacks, runtimes that plan every byte in advance) use this entry point
instead of nnop_rms_norm_bwd: it needs no workspace because its scratch lives
in a fixed 8 MiB array inside the library.  These tests call it through the C
ABI and compare it with the workspace entry point on two calls in a row (the
second call sees the scratch the first one left behind).  The file is named
so that pytest collects it last."""
import ctypes as C
import gc

import numpy as np
import pytest

from _util import isapprox

pytestmark = pytest.mark.gpu


def _call_both(lib, dy, x, w, rstd, offset, dtype_id):
    import torch
    n, emb = x.shape
    stream = torch.cuda.current_stream().cuda_stream
    dx_ref = torch.empty_like(x)
    dw_ref = torch.empty(emb, dtype=torch.float32, device="cuda")
    ws_bytes = lib.nnop_rms_norm_bwd_workspace_size(emb, n)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    assert lib.nnop_rms_norm_bwd(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx_ref.data_ptr(),
                                 dw_ref.data_ptr(), ws.data_ptr(), ws_bytes, emb, n, offset, dtype_id, stream) == 0
    dx = torch.full_like(x, float("nan"))
    dw = torch.full((emb,), float("nan"), dtype=torch.float32, device="cuda")
    st = lib.nnop_rms_norm_bwd_noalloc(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(),
                                       dw.data_ptr(), emb, n, offset, dtype_id, stream)
    assert st == 0, lib.nnop_last_error()
    torch.cuda.synchronize()
    return dx, dw, dx_ref, dw_ref


@pytest.mark.parametrize("dtype,emb,n", [("f32", 4096, 3000), ("bf16", 4096, 5000), ("f32", 513, 25),
                                         ("f16", 8192, 700), ("f32", 100000, 9)])
def test_noalloc_matches_workspace_entry_point_twice(dtype, emb, n):
    import torch
    import nnop
    from nnop._lib import lib
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[dtype]
    dtype_id = {"f32": 0, "f16": 1, "bf16": 2}[dtype]
    tol = dict(atol=1e-6, rtol=1e-6) if dtype == "f32" else dict(atol=0.0, rtol=2e-2)
    for call in range(2):   # the second call runs on the scratch the first left behind
        g = torch.Generator(device="cuda").manual_seed(100 * call + emb)
        x = torch.randn(n, emb, device="cuda", generator=g).to(tdt)
        w = (1 + 0.1 * torch.randn(emb, device="cuda", generator=g)).to(tdt)
        dy = torch.randn(n, emb, device="cuda", generator=g).to(tdt)
        _, rstd = nnop._rms_norm(x, w, offset=0.25 * call)
        dx, dw, dx_ref, dw_ref = _call_both(lib, dy, x, w, rstd, 0.25 * call, dtype_id)
        assert not torch.isnan(dx).any() and not torch.isnan(dw).any()
        assert isapprox(dx.double().cpu().numpy(), dx_ref.double().cpu().numpy(), **tol)
        assert isapprox(dw.double().cpu().numpy(), dw_ref.double().cpu().numpy(), **tol)


def test_noalloc_largest_emb_matches_workspace_entry_point():
    """emb = 2^21, the largest the built-in scratch takes: one partial row fits,
    so the whole dw comes from one CTA walking every row."""
    import torch
    import nnop
    from nnop._lib import lib
    emb, n = 1 << 21, 3
    g = torch.Generator(device="cuda").manual_seed(21)
    x = torch.randn(n, emb, device="cuda", generator=g)
    w = 1 + 0.1 * torch.randn(emb, device="cuda", generator=g)
    dy = torch.randn(n, emb, device="cuda", generator=g)
    _, rstd = nnop._rms_norm(x, w)
    for _ in range(2):
        dx, dw, dx_ref, dw_ref = _call_both(lib, dy, x, w, rstd, 0.0, 0)
        assert isapprox(dx.double().cpu().numpy(), dx_ref.double().cpu().numpy(), atol=1e-6, rtol=1e-6)
        assert isapprox(dw.double().cpu().numpy(), dw_ref.double().cpu().numpy(), atol=1e-6, rtol=1e-6)


def test_noalloc_allocates_no_device_memory():
    """Around a warmed-up call, neither torch's allocator nor the device's free
    memory (cudaMemGetInfo) changes: the entry point takes no memory."""
    import torch
    import nnop
    from nnop._lib import lib
    n, emb = 2000, 4096
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(n, emb, device="cuda", generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(emb, device="cuda", generator=g)).bfloat16()
    dy = torch.randn(n, emb, device="cuda", generator=g).bfloat16()
    _, rstd = nnop._rms_norm(x, w)
    dx = torch.empty_like(x)
    dw = torch.empty(emb, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def call():
        st = lib.nnop_rms_norm_bwd_noalloc(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(),
                                           dx.data_ptr(), dw.data_ptr(), emb, n, 0.0, 2, stream)
        assert st == 0, lib.nnop_last_error()

    call()                                   # first call on the device: address lookup
    torch.cuda.synchronize()
    gc.collect()                             # tensors of earlier tests freed now, not during the calls
    torch_before = torch.cuda.memory_allocated()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() <= torch_before
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before


def test_noalloc_rejects_emb_beyond_the_scratch():
    from nnop._lib import lib
    d = C.c_void_p(256)   # never dereferenced: the size check fails first
    st = lib.nnop_rms_norm_bwd_noalloc(d, d, d, d, d, d, (1 << 21) + 1, 4, 0.0, 0, None)
    assert st == -1
    assert b"exceeds the maximum" in lib.nnop_last_error()
