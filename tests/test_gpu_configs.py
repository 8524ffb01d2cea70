"""Parity at the benchmark workloads, full GLM-5 shape (hidden 6144,
intermediate 2048, 256 K4 experts + the bf16 shared expert).

* Router indices end to end: the layer's own routing against the oracle's
  routing of the oracle's OWN float32 gate product (model.py:111-132 with
  model.py:366-371), not of the kernel's logits.  The two float32 gate
  products differ in summation order, so a token whose 8th and 9th choice
  values lie closer than the measured logit error can legitimately flip;
  every other token must select exactly the oracle's experts.  Near ties
  are counted and printed.
* Layer outputs at T = 4 (the CPU-baseline configuration), 8 and 32 tokens
  against the C oracle of the whole layer (pinned to the NumPy oracle),
  routed from the logits the layer used so both sides take the same experts.
"""

import numpy as np
import pytest

from helpers import assert_bf16_close, host, rel_l2
from oracle import trellis_oracle as ref

pytestmark = pytest.mark.gpu

# |d sigmoid / d logit| <= 1/4; choice values lie in (-0.1, 1.1), where a
# float32 ulp is at most 2^-23.
SIGMOID_SLOPE = 0.25
CHOICE_ULP = 2.0 ** -23


@pytest.fixture(scope="module")
def glm_layer():
    from mlxlr8_b200.synthetic import make_layer

    return make_layer(seed=11)


def _exact_logits(x, weight):
    return np.asarray(x, np.float64) @ np.asarray(weight, np.float64).T


def _gpu_logits(x, layer):
    """The gate products the layer path uses: the float32 GEMV below 64 tokens,
    the tensor-core product from 64 tokens (both deterministic)."""
    from mlxlr8_b200.fast_router import router, router_logits

    if x.shape[0] >= 64:
        return router_logits(x, layer.gate_weight)
    return router(x, layer.gate_weight, layer.bias)[0]


def check_routing_against_oracle(x, weight, bias, ids_gpu, scores_gpu, logits_gpu, what):
    """Exact expert sets for every token outside the near-tie band; returns
    the number of near-tie tokens."""
    xs = host(x)
    w = np.asarray(weight, np.float32)
    b = np.asarray(bias, np.float32)
    exact = _exact_logits(xs, w)
    oracle_logits = ref.router_logits(xs, w)
    bound = float(np.abs(logits_gpu - exact).max() + np.abs(oracle_logits - exact).max())
    choice_bound = SIGMOID_SLOPE * bound + 2 * CHOICE_ULP
    e_ids, e_scores = ref.route(oracle_logits, b)
    choice = ref.sigmoid_f32(oracle_logits).astype(np.float64) + b[None, :]
    ordered = -np.sort(-choice, axis=1)
    margin = ordered[:, 7] - ordered[:, 8]
    clear = margin > choice_bound
    np.testing.assert_array_equal(ids_gpu[:, 8], 256)
    got_sets = np.sort(ids_gpu[:, :8], axis=1)
    want_sets = np.sort(e_ids[:, :8].astype(np.int64), axis=1)
    wrong = np.nonzero(clear & np.any(got_sets != want_sets, axis=1))[0]
    assert wrong.size == 0, f"{what}: tokens {wrong[:8]} select other experts than the oracle"
    # Scores of the clear tokens, matched by expert id.
    for t in np.nonzero(clear)[0][:256]:
        g = dict(zip(ids_gpu[t, :8].tolist(), scores_gpu[t].tolist()))
        e = dict(zip(e_ids[t, :8].tolist(), e_scores[t].tolist()))
        for k, v in e.items():
            assert abs(g[int(k)] - v) <= 2e-5 * abs(v) + 1e-6, (what, t, k)
    near = int((~clear).sum())
    print(f"{what}: {x.shape[0]} tokens, logit error bound {bound:.3g}, choice bound {choice_bound:.3g}, "
          f"near ties {near}")
    assert near <= max(2, x.shape[0] // 100), f"{what}: {near} near-tie tokens"
    return near


@pytest.mark.parametrize("tokens", [1, 4, 8, 32, 128])
def test_router_indices_end_to_end_trellis(glm_layer, tokens):
    """The parity size T = 4, the decode sizes T = 1, 8, 32 and the 128-token
    verify size: the indices the whole layer returns."""
    import torch

    from mlxlr8_b200.moe import MoELayer

    x, residual = glm_layer.tokens(tokens, seed_offset=tokens)
    moe = MoELayer(glm_layer.gate_weight, glm_layer.bias, glm_layer.experts)
    _, ids, scores = moe(x, residual, return_routing=True)
    logits = _gpu_logits(x, glm_layer)
    torch.cuda.synchronize()
    check_routing_against_oracle(x, glm_layer.gate_weight.cpu().numpy(), glm_layer.bias.cpu().numpy(),
                                 ids.cpu().numpy().astype(np.int64), scores.cpu().numpy(), host(logits),
                                 f"trellis T={tokens}")


def test_router_indices_end_to_end_zipf(glm_layer):
    """The speculative-verify size (128 tokens) with the calibrated Zipf(1.1)
    router bias."""
    import torch

    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.synthetic import zipf_bias

    bias = zipf_bias(301)
    x, residual = glm_layer.tokens(128, seed_offset=7)
    moe = MoELayer(glm_layer.gate_weight, bias, glm_layer.experts)
    _, ids, scores = moe(x, residual, return_routing=True)
    logits = _gpu_logits(x, glm_layer)
    torch.cuda.synchronize()
    check_routing_against_oracle(x, glm_layer.gate_weight.cpu().numpy(), bias.cpu().numpy(),
                                 ids.cpu().numpy().astype(np.int64), scores.cpu().numpy(), host(logits),
                                 "trellis T=128 zipf")


def test_router_indices_end_to_end_joined_prefill():
    """The prefill size: 4096 tokens through the joined MXFP4 layer
    (tensor-core gate product)."""
    import torch

    from mlxlr8_b200.fast_router import router_logits
    from mlxlr8_b200.joined_mxfp4 import JoinedMoELayer, JoinedMXFP4
    from mlxlr8_b200.synthetic import make_joined

    j = make_joined(seed=13)
    layer = JoinedMoELayer(j.gate_weight, j.bias, JoinedMXFP4(j.unit, j.weights, j.scales, j.hidden, j.intermediate))
    x, residual = j.tokens(4096)
    _, ids, scores = layer(x, residual, return_routing=True)
    logits = router_logits(x, j.gate_weight)
    torch.cuda.synchronize()
    check_routing_against_oracle(x, j.gate_weight.cpu().numpy(), j.bias.cpu().numpy(),
                                 ids.cpu().numpy().astype(np.int64), scores.cpu().numpy(), host(logits),
                                 "joined T=4096")


def _bf16_bits(a):
    return (np.ascontiguousarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16)


@pytest.mark.parametrize("tokens", [4, 8, 32])
def test_glm_layer_full_shape(glm_layer, tokens):
    """The whole layer at full shape against the C oracle of the layer:
    T = 4 is the parity size (the reference's fused-finish decode bound,
    model.py:389), T = 8 decode, T = 32 the grouped prefill GEMM."""
    import torch

    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.synthetic import host_copy
    from oracle import c_oracle

    x, residual = glm_layer.tokens(tokens, seed_offset=100 + tokens)
    moe = MoELayer(glm_layer.gate_weight, glm_layer.bias, glm_layer.experts)
    out, ids, scores = moe(x, residual, return_routing=True)
    logits = _gpu_logits(x, glm_layer)
    torch.cuda.synchronize()
    ids_np = ids.cpu().numpy()
    hc = host_copy(glm_layer, np.unique(ids_np[:, :8]))
    shared_bits = [_bf16_bits(t) for t in hc["shared"]]
    expected, e_ids, e_scores = c_oracle.moe_layer(host(x), host(residual), hc["gate_weight"], hc["bias"],
                                                   hc["packed"], hc["scales"], 4, 6144, 2048, shared_bits,
                                                   "bfloat16", logits=host(logits))
    np.testing.assert_array_equal(ids_np, e_ids.astype(np.int64))
    np.testing.assert_allclose(scores.cpu().numpy(), e_scores, rtol=1e-6, atol=1e-7)
    got, res = host(out), host(residual)
    if tokens <= 16:
        # Streaming decode path: float16 hi/lo activation pieces, float32 sums.
        assert_bf16_close(got, expected)
        assert rel_l2(got - res, expected - res) < 1e-2
    else:
        # Grouped tcgen05 GEMM: E4M3 hi/lo activation planes.
        from test_gpu_prefill import assert_prefill_close, gemm_ok

        gemm_ok(moe._workspace, tokens, 9, 2048, glm_layer.experts.experts)
        assert_prefill_close(got - res, expected - res)


def test_zipf_bias_skews_gpu_routing(glm_layer):
    """The calibrated bias on the GPU router with a layer's own gate weight:
    the top-8 selection frequencies of 10^5 seeded tokens fit Zipf(1.1)
    (least-squares log-log slope against the popularity rank)."""
    import torch

    from mlxlr8_b200.fast_router import route, router_logits
    from mlxlr8_b200.synthetic import ZIPF_S, zipf_bias, zipf_ranks

    bias = zipf_bias(305)
    rank = zipf_ranks(305).cpu().numpy()
    g = torch.Generator(device="cuda")
    g.manual_seed(99)
    counts = torch.zeros(256, dtype=torch.int64, device="cuda")
    tokens = 0
    for _ in range(13):
        x = torch.randn(8192, 6144, generator=g, device="cuda").to(torch.bfloat16)
        ids, _ = route(router_logits(x, glm_layer.gate_weight), bias)
        counts += torch.bincount(ids[:, :8].reshape(-1).long(), minlength=256)
        tokens += 8192
    freq = counts.cpu().numpy() / tokens
    keep = freq > 0
    slope = np.polyfit(np.log(rank[keep] + 1.0), np.log(freq[keep]), 1)[0]
    print(f"GPU routing with the Zipf bias: slope {slope:.4f} over {tokens} tokens")
    assert abs(slope + ZIPF_S) < 0.08, slope
