"""The C oracle (fast checker and CPU baseline) agrees with the NumPy oracle."""

import numpy as np
import pytest

from helpers import small_experts
from oracle import c_oracle
from oracle import trellis_oracle as ref


@pytest.mark.parametrize("k", [2, 3, 4])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_expert_mlp_rows_matches_numpy(k, dtype):
    packed, scales = small_experts(k=k, experts=3)
    x = ref.rounder(dtype)(np.random.default_rng(5).normal(size=(3, 256)).astype(np.float32))
    for e in range(3):
        got = c_oracle.expert_mlp_rows(x, e, packed, scales, k, 256, 384, dtype)
        ids = np.full((3, 1), e)
        want = ref.expert_mlp_fused(x, ids, packed, scales, k, 256, 384, dtype)[:, 0]
        np.testing.assert_allclose(got, want, rtol=2e-2 if dtype == "bfloat16" else 5e-5, atol=1e-6)


def test_moe_layer_matches_numpy():
    rng = np.random.default_rng(9)
    hidden, inter, experts = 256, 128, 256
    packed = {p: rng.integers(0, 256, experts * hidden * inter // 2, dtype=np.uint8) for p in ("gate", "up", "down")}
    scales = {
        "gate": (rng.uniform(-0.1, 0.1, (experts, hidden)).astype(np.float16), rng.uniform(-1, 1, (experts, inter)).astype(np.float16)),
        "up": (rng.uniform(-0.1, 0.1, (experts, hidden)).astype(np.float16), rng.uniform(-1, 1, (experts, inter)).astype(np.float16)),
        "down": (rng.uniform(-0.1, 0.1, (experts, inter)).astype(np.float16), rng.uniform(-1, 1, (experts, hidden)).astype(np.float16)),
    }
    shared = tuple(ref.round_bf16(0.02 * rng.normal(size=s).astype(np.float32)) for s in ((inter, hidden), (inter, hidden), (hidden, inter)))
    shared_bits = tuple(ref.bf16_bits(s) for s in shared)
    wg = (0.02 * rng.normal(size=(256, hidden))).astype(np.float32)
    bias = (0.01 * rng.normal(size=256)).astype(np.float32)
    x = ref.round_bf16(rng.normal(size=(3, hidden)).astype(np.float32))
    res = ref.round_bf16(rng.normal(size=(3, hidden)).astype(np.float32))
    out, ids, scores = c_oracle.moe_layer(x, res, wg, bias, packed, scales, 4, hidden, inter, shared_bits)
    logits = ref.router_logits(x, wg)
    e_out, e_ids, e_scores = ref.moe_layer(x, res, wg, bias, packed, scales, 4, hidden, inter, shared=shared,
                                           logits=logits)
    np.testing.assert_array_equal(ids, e_ids)
    np.testing.assert_allclose(scores, e_scores, rtol=1e-5)
    scale = np.abs(e_out).max()
    np.testing.assert_allclose(out, e_out, rtol=1e-2, atol=1e-2 * scale)
