"""Helpers shared by the tests: seeded inputs, dtype round-trips and Julia's
norm-based ``isapprox``."""
from __future__ import annotations

import numpy as np

DTYPES = {"f32": "float32", "f16": "float16", "bf16": "bfloat16"}


def isapprox(a, b, *, atol, rtol) -> bool:
    """Julia ``isapprox`` on arrays: ‖a−b‖ ≤ max(atol, rtol·max(‖a‖, ‖b‖))
    (the criterion of every reference test, e.g. test/attention_tests.jl:41)."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    d = np.linalg.norm(a - b)
    return bool(d <= max(atol, rtol * max(np.linalg.norm(a), np.linalg.norm(b))))


def torch_dtype(name: str):
    import torch
    return {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[name]


def to_dev(x: np.ndarray, dtype: str):
    """numpy -> CUDA tensor of the given dtype (rounded there)."""
    import torch
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to("cuda").to(torch_dtype(dtype))


def to_np(t) -> np.ndarray:
    """CUDA tensor -> float64 numpy (exact values of the stored dtype)."""
    import torch
    return t.detach().to(torch.float64).cpu().numpy()
