"""CPU checks of the C-ABI library: it loads without a GPU, exports every entry
point declared in include/nnop_b200.h, and rejects invalid shapes before any
launch with the reference's error text (src/attention.jl:153-156)."""
import ctypes as C
import os
import pathlib
import re
import subprocess

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "nnop_b200.h"


def header_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nnop_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = header_functions()
    for n in ("nnop_flash_attention_fwd", "nnop_flash_attention_bwd", "nnop_online_softmax_fwd",
              "nnop_online_softmax_bwd", "nnop_rms_norm_fwd", "nnop_rms_norm_bwd", "nnop_layer_norm_fwd",
              "nnop_layer_norm_bwd", "nnop_llama_rope", "nnop_llama_rope_cos_sin"):
        assert n in names


def test_library_exports_every_header_symbol():
    from nnop import _lib
    lib = C.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in header_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding declares a signature for each of them
    assert set(header_functions()) == set(_lib.SIGNATURES)


def test_exported_symbols_are_c_abi():
    from nnop import _lib
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (nnop_[a-z0-9_]+)\b", out))
    assert set(header_functions()) <= exported


def test_abi_version_and_status_strings():
    from nnop._lib import lib
    assert lib.nnop_abi_version() == 1
    assert lib.nnop_status_string(0) == b"ok"
    assert lib.nnop_status_string(-1) == b"invalid or unsupported shape"


def _fwd(lib, E=64, QL=8, KL=8, QH=2, KH=2, B=1, dtype=2):
    dummy = C.c_void_p(256)   # never dereferenced: validation fails first
    return lib.nnop_flash_attention_fwd(dummy, dummy, dummy, None, None, dummy, dummy, None, 0, E, QL, KL, QH, KH, B,
                                        0, dtype, None)


def test_shape_errors_before_launch():
    from nnop._lib import lib
    assert _fwd(lib, E=48) == -1
    assert b"Only power-of-2 embedding dims are supported." == lib.nnop_last_error()
    assert _fwd(lib, QH=3, KH=2) == -1
    assert lib.nnop_last_error() == b"Number of query heads `3` must be divisible by number of KV heads `2`."
    assert _fwd(lib, E=256) == -1
    assert _fwd(lib, dtype=7) == -2
    assert _fwd(lib, QL=0) == 0          # empty query range: nothing to do
    assert _fwd(lib, B=0) == 0


def test_norm_rope_errors_before_launch():
    from nnop._lib import lib
    d = C.c_void_p(256)
    assert lib.nnop_rms_norm_fwd(d, d, d, d, 0, 4, 1e-6, 0.0, 0, None) == -1
    assert lib.nnop_rms_norm_fwd(d, d, d, d, 16, 0, 1e-6, 0.0, 0, None) == 0
    assert lib.nnop_online_softmax_fwd(d, d, 0, 4, 0, None) == -1
    assert lib.nnop_online_softmax_fwd(d, d, 16, 0, 0, None) == 0
    assert lib.nnop_llama_rope(d, d, d, d, d, d, 15, 4, 1, 1, 1, 1, 1.0, 0, None) == -1
    assert lib.nnop_llama_rope(d, d, d, d, d, d, 16, 4, 1, 1, 2, 3, 1.0, 0, None) == -1
    assert lib.nnop_layer_norm_bwd(d, d, d, d, d, d, d, d, None, 0, 16, 4, 0, None) == -4


def test_workspace_sizes():
    from nnop._lib import lib
    ws = lib.nnop_flash_attention_bwd_workspace_size(64, 4096, 4096, 16, 16, 8, 0, 2)
    assert ws >= 8 * 16 * 4096 * 64 * 4 + 8 * 16 * 4096 * 4
    assert lib.nnop_flash_attention_bwd_workspace_size(64, 4096, 4096, 16, 16, 8, 0, 0) < ws
    tiles = 8 * 16 * 4096 * 4096 * 2
    assert lib.nnop_flash_attention_bwd_workspace_size(64, 4096, 4096, 16, 16, 8, 1, 2) >= ws + 2 * tiles
    assert lib.nnop_flash_attention_fwd_workspace_size(64, 4096, 4096, 16, 16, 8, 1, 2) >= tiles
    assert lib.nnop_flash_attention_fwd_workspace_size(64, 4096, 4096, 16, 16, 8, 0, 2) == 0
    assert lib.nnop_flash_attention_fwd_workspace_size(64, 4096, 4096, 16, 16, 8, 1, 0) == 0
    assert lib.nnop_rms_norm_bwd_workspace_size(4096, 65536) >= 4096 * 4
    assert lib.nnop_layer_norm_bwd_workspace_size(4096, 3) == 3 * 2 * 4096 * 4


def test_no_cpu_fallback():
    """The product path refuses CPU tensors instead of computing on the host."""
    import torch
    import nnop
    x = torch.ones(4, 8)
    with pytest.raises(nnop.NNopError, match="CUDA tensors only"):
        nnop.online_softmax(x)
    with pytest.raises(nnop.NNopError, match="CUDA tensors only"):
        nnop.flash_attention(torch.ones(1, 1, 4, 16), torch.ones(1, 1, 4, 16), torch.ones(1, 1, 4, 16), causal=False)


def test_missing_library_fails_loudly(tmp_path):
    """Without the compiled library the package does not import (no host path to fall back to)."""
    import sys
    code = "import nnop"
    env = dict(os.environ, NNOP_B200_LIB=str(tmp_path / "absent.so"), PYTHONPATH=str(ROOT / "onionop.jl_b200"))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode != 0 and "absent.so" in r.stderr


def test_product_does_not_import_oracle():
    pkg = ROOT / "onionop.jl_b200"
    for f in pkg.rglob("*.py"):
        assert "oracle" not in f.read_text().replace("# oracle", ""), f


def test_bwd_reuse_workspace_sizes():
    """With the forward's pair tiles reused, the backward needs one tile buffer
    less; without a pair, or with no (or too small) forward workspace, the
    reuse size is the full backward size."""
    from nnop._lib import lib
    E, L, H, B, bf16 = 64, 4096, 16, 8, 2
    fw = lib.nnop_flash_attention_fwd_workspace_size(E, L, L, H, H, B, 1, bf16)
    full = lib.nnop_flash_attention_bwd_workspace_size(E, L, L, H, H, B, 1, bf16)
    reuse = lib.nnop_flash_attention_bwd_workspace_size_reuse(E, L, L, H, H, B, 1, fw, bf16)
    tiles = B * H * L * L * 2
    assert fw == tiles
    assert full - reuse == tiles
    assert lib.nnop_flash_attention_bwd_workspace_size_reuse(E, L, L, H, H, B, 1, 0, bf16) == full
    assert lib.nnop_flash_attention_bwd_workspace_size_reuse(E, L, L, H, H, B, 1, fw - 256, bf16) == full
    assert (lib.nnop_flash_attention_bwd_workspace_size_reuse(E, L, L, H, H, B, 0, fw, bf16)
            == lib.nnop_flash_attention_bwd_workspace_size(E, L, L, H, H, B, 0, bf16))
    # fp32 and E != 64 keep no tiles
    assert lib.nnop_flash_attention_fwd_workspace_size(E, L, L, H, H, B, 1, 0) == 0
    assert lib.nnop_flash_attention_fwd_workspace_size(128, L, L, H, H, B, 1, bf16) == 0


def test_kernel_timing_read_arguments():
    from nnop._lib import lib
    ms, n = C.c_double(1.0), C.c_int(5)
    assert lib.nnop_kernel_timing_read(2, C.byref(ms), C.byref(n)) == -3
    assert lib.nnop_kernel_timing_read(0, None, C.byref(n)) == -3
    lib.nnop_kernel_timing(0)
    # nothing recorded: zero launches, zero time (needs no device)
    assert lib.nnop_kernel_timing_read(1, C.byref(ms), C.byref(n)) == 0
    assert (ms.value, n.value) == (0.0, 0)


def _bwd(lib, *, pair=None, dpair=None, ws=None, ws_bytes=0, E=64, L=256, H=2, B=1, dtype=2, align=256):
    d = C.c_void_p(align)   # never dereferenced: validation fails first
    return lib.nnop_flash_attention_bwd(d, d, d, d, d, d, pair, None, d, d, d, dpair, ws, ws_bytes,
                                        E, L, L, H, H, B, 1, dtype, None)


def test_backward_argument_errors_before_launch():
    from nnop._lib import lib
    d = C.c_void_p(256)
    # dpair given exactly when pair is given
    assert _bwd(lib, pair=d, dpair=None) == -3
    assert _bwd(lib, pair=None, dpair=d) == -3
    # dense tensors must be 16-byte aligned
    assert _bwd(lib, align=8) == -6
    # workspace missing, too small, or not 256-byte aligned
    need = lib.nnop_flash_attention_bwd_workspace_size(64, 256, 256, 2, 2, 1, 0, 2)
    assert need > 0
    assert _bwd(lib, ws=None, ws_bytes=0) == -4
    assert b"workspace too small" in lib.nnop_last_error()
    assert _bwd(lib, ws=C.c_void_p(4096), ws_bytes=need - 1) == -4
    assert _bwd(lib, ws=C.c_void_p(4096 + 16), ws_bytes=need) == -6
    # the reuse variant: a forward workspace that holds no tiles changes nothing
    full = lib.nnop_flash_attention_bwd_workspace_size_reuse(64, 256, 256, 2, 2, 1, 0, 0, 2)
    assert full == need
