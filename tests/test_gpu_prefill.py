"""Trellis prefill (more than 16 token rows, experts.py:171-174): grouped
tcgen05 GEMMs whose decoder warps expand the trellis codes, against the CPU
oracle of the reference operators (fast_prefill.py:188-211,
tests/test_fast_prefill.py).

The GEMM feeds activations as two E4M3 planes with shared E8M0 block scales
(about eight significant bits against each block's maximum), so these tests
use the layer-output bar: max |a - b| <= 1e-2 of the largest reference
magnitude and relative L2 below 5e-3.  The GEMM serves 16-bit activations;
the expert operators keep float32 activations on the float32-accurate
streaming path at every row count (the reference's float32 tolerance,
test_experts.py:147: rtol 5e-4).
"""

import numpy as np
import pytest

from helpers import host, rel_l2, small_experts, to_device
from oracle import trellis_oracle as ref

pytestmark = pytest.mark.gpu


def gemm_ok(workspace, tokens, slots, intermediate, experts):
    """The grouped GEMMs of the last prefill call finished without a timed-out wait."""
    from mlxlr8_b200 import _lib

    header = _lib.prefill_status(workspace, tokens, slots, intermediate, experts)
    assert header[4] == 0, header
    return header


def assert_prefill_close(actual, expected, tol=1e-2, rel=5e-3):
    scale = max(float(np.max(np.abs(expected))), 1e-30)
    err = float(np.max(np.abs(actual - expected)))
    assert err <= tol * scale, (err, scale)
    assert rel_l2(actual, expected) < rel, rel_l2(actual, expected)


@pytest.mark.parametrize("k", [3, 4])
@pytest.mark.parametrize("per_slot", [False, True])
@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_prefill_expert_mlp_matches_oracle(k, per_slot, dtype):
    import torch

    from mlxlr8_b200.fast_decode import fast_expert_mlp
    from helpers import torch_dtype

    packed, scales = small_experts(k=k, experts=5)
    rng = np.random.default_rng(53)
    tokens, slots = 40, 3
    ids = rng.integers(0, 5, (tokens, slots)).astype(np.int32)
    x = ref.rounder(dtype)(rng.normal(size=(tokens, slots, 256) if per_slot else (tokens, 256)).astype(np.float32))
    expected = ref.expert_mlp_fused(x, ids, packed, scales, k, 256, 384, dtype)
    dp, ds = to_device(packed, scales)
    ws = torch.zeros(64 << 20, dtype=torch.uint8, device="cuda")
    actual = host(fast_expert_mlp(torch.from_numpy(x).to(torch_dtype(dtype)).cuda(), torch.from_numpy(ids).cuda(),
                                  dp, ds, k, 256, 384, workspace=ws))
    assert actual.shape == (tokens, slots, 256)
    if dtype == "float32":
        # streaming path: float32 accumulation, the decode tests' tolerance
        scale = float(np.max(np.abs(expected)))
        np.testing.assert_allclose(actual, expected, rtol=1e-4, atol=1e-6 * scale)
        return
    gemm_ok(ws, tokens, slots, 384, 5)
    assert_prefill_close(actual, expected)


def test_prefill_ragged_chunks():
    """Experts with 0, 1, 127, 128, 160, 161 and 300 rows (empty segments,
    partial MMA columns, the 160-row chunk limit, 128-row chunks), and an
    intermediate size that leaves a half weight block (out 128)."""
    import torch

    from mlxlr8_b200.fast_decode import fast_expert_mlp

    counts = [0, 1, 127, 128, 160, 161, 300]
    packed, scales = small_experts(hidden=256, intermediate=128, experts=len(counts))
    ids = np.concatenate([np.full(c, e, dtype=np.int32) for e, c in enumerate(counts)])
    np.random.default_rng(2).shuffle(ids)
    ids = ids.reshape(-1, 1)
    x = ref.round_bf16(np.random.default_rng(3).normal(size=(ids.shape[0], 256)).astype(np.float32))
    expected = ref.expert_mlp_fused(x, ids, packed, scales, 4, 256, 128, "bfloat16")
    dp, ds = to_device(packed, scales)
    ws = torch.empty(64 << 20, dtype=torch.uint8, device="cuda")
    actual = host(fast_expert_mlp(torch.from_numpy(x).to(torch.bfloat16).cuda(), torch.from_numpy(ids).cuda(), dp,
                                  ds, 4, 256, 128, workspace=ws))
    header = gemm_ok(ws, ids.shape[0], 1, 128, len(counts))
    assert header[0] == 1 + 1 + 1 + 1 + 2 + 3  # 1, 127, 128, 160 rows: one chunk; 161: 128 + 33; 300: 128 + 128 + 44
    assert_prefill_close(actual, expected)
    for e, c in enumerate(counts):
        if c:
            sel = ids[:, 0] == e
            assert_prefill_close(actual[sel], expected[sel])


@pytest.mark.parametrize("tokens", [24, 40, 130, 600])
@pytest.mark.parametrize("shared", ["bf16", "trellis"])
def test_prefill_layer_matches_oracle(tokens, shared):
    """600 tokens (5,400 slots) takes the multi-CTA dispatch plan."""
    import torch

    from mlxlr8_b200.fast_router import router, router_logits
    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.synthetic import host_copy, make_layer

    layer = make_layer(seed=17, hidden=256, intermediate=128, shared=shared)
    x, residual = layer.tokens(tokens)
    moe = MoELayer(layer.gate_weight, layer.bias, layer.experts)
    out, ids, scores = moe(x, residual, return_routing=True)
    torch.cuda.synchronize()
    gemm_ok(moe._workspace, tokens, 9, 128, layer.experts.experts)
    if tokens >= 64:
        logits = router_logits(x, layer.gate_weight)
    else:
        logits, _, _ = router(x, layer.gate_weight, layer.bias)
    ids_np = ids.cpu().numpy()
    hc = host_copy(layer, np.unique(ids_np[:, :8] if shared == "bf16" else ids_np))
    e_out, e_ids, e_scores = ref.moe_layer(host(x), host(residual), hc["gate_weight"], hc["bias"], hc["packed"],
                                           hc["scales"], 4, 256, 128, shared=hc["shared"], dtype="bfloat16",
                                           logits=host(logits))
    np.testing.assert_array_equal(ids_np, e_ids)
    np.testing.assert_allclose(scores.cpu().numpy(), e_scores, rtol=1e-6, atol=1e-7)
    assert_prefill_close(host(out) - host(residual), e_out - host(residual))


@pytest.mark.parametrize("skew", ["uniform", "zipf"])
@pytest.mark.parametrize("k", [4, 3])
def test_glm_prefill_sampled_tokens(k, skew):
    """GLM shape at the speculative-verify size (128 tokens; K3 is the
    layer-78 width), with the router's own bias or the calibrated Zipf(1.1)
    skew (the popular experts then get many rows): the layer runs on the
    GPU, the C oracle checks the routed experts of sampled tokens (each
    token's output depends only on its own slots)."""
    import torch

    from mlxlr8_b200.fast_router import router_logits
    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.synthetic import host_copy, make_layer, zipf_bias
    from oracle import c_oracle

    layer = make_layer(seed=23, k=k)
    bias = zipf_bias(303) if skew == "zipf" else layer.bias
    tokens = 128
    x, residual = layer.tokens(tokens)
    moe = MoELayer(layer.gate_weight, bias, layer.experts)
    out, ids, scores = moe(x, residual, return_routing=True)
    logits = router_logits(x, layer.gate_weight)
    torch.cuda.synchronize()
    gemm_ok(moe._workspace, tokens, 9, 2048, layer.experts.experts)
    e_ids, e_scores = ref.route(host(logits), bias.cpu().numpy())
    np.testing.assert_array_equal(ids.cpu().numpy(), e_ids)
    if skew == "zipf":
        counts = np.bincount(e_ids[:, :8].ravel(), minlength=256)
        assert counts.max() >= 20  # the head experts carry many rows (~0.24 x 128 for the first)
    sample = np.array([0, 77, 101])
    hc = host_copy(layer, np.unique(e_ids[sample, :8]))
    xs = host(x)[sample]
    values = np.zeros((sample.size, 9, 6144), np.float32)
    for i, t in enumerate(sample):
        for r in range(8):
            values[i, r] = c_oracle.expert_mlp_rows(xs[i:i + 1], int(e_ids[t, r]), hc["packed"], hc["scales"], k,
                                                    6144, 2048, "bfloat16")[0]
    values[:, 8] = ref.shared_bf16(xs, *hc["shared"])
    expected = ref.combine(values, e_scores[sample], host(residual)[sample], "bfloat16")
    got = host(out)[sample]
    assert_prefill_close(got - host(residual)[sample], expected - host(residual)[sample])
