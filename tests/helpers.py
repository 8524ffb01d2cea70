"""Shared helpers of the GPU parity tests."""

from __future__ import annotations

import numpy as np

TORCH_DTYPES = {}


def torch_dtype(name):
    import torch

    return {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}[name]


def small_experts(seed=181, hidden=256, intermediate=384, experts=3, k=4):
    """Random trellis experts like the reference's fixture (test_fast_decode.py:119-129)."""
    rng = np.random.default_rng(seed)
    packed, scales = {}, {}
    for projection in ("gate", "up", "down"):
        a, b = (intermediate, hidden) if projection == "down" else (hidden, intermediate)
        packed[projection] = rng.integers(0, 256, experts * a * b * k // 8, dtype=np.uint8)
        scales[projection] = (
            rng.uniform(-0.08, 0.08, (experts, a)).astype(np.float16),
            rng.uniform(-0.5, 0.5, (experts, b)).astype(np.float16),
        )
    return packed, scales


def to_device(packed, scales, device="cuda"):
    import torch

    p = {k: torch.from_numpy(v).to(device) for k, v in packed.items()}
    s = {k: tuple(torch.from_numpy(np.ascontiguousarray(a)).to(device) for a in v) for k, v in scales.items()}
    return p, s


def host(t):
    import torch

    return t.detach().to(torch.float32).cpu().numpy()


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def assert_bf16_close(actual, expected, rtol=1e-2, rel=7e-3):
    """Layer-output tolerance for 16-bit outputs: elementwise rtol 1e-2 with an
    absolute floor of 1e-2 of the largest magnitude, and relative L2 < 7e-3."""
    scale = float(np.max(np.abs(expected))) if expected.size else 1.0
    np.testing.assert_allclose(actual, expected, rtol=rtol, atol=1e-2 * scale)
    assert rel_l2(actual, expected) < rel
