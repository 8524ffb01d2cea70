"""Joined MXFP4 experts (JoinedMXFP4.slots / .finish and the prefill layer) on
the grouped block-scaled tcgen05 GEMM, against the CPU oracle of the
reference's joined path (joined_mxfp4.py:90-165).

Tolerance (the MXFP4 bar of the layer outputs): max |a - b| <= 2e-2 of the
largest reference magnitude, and relative L2 below 1e-2.  The GEMM feeds the
activations as two E4M3 planes with shared E8M0 block scales; the observed
error is about 1e-3 relative.
"""

import numpy as np
import pytest

from helpers import host, rel_l2
from oracle import trellis_oracle as ref

pytestmark = pytest.mark.gpu

MXFP4_TOL = 2e-2


def assert_mxfp4_close(actual, expected, tol=MXFP4_TOL, rel=1e-2):
    scale = max(float(np.max(np.abs(expected))), 1e-30)
    err = float(np.max(np.abs(actual - expected)))
    assert err <= tol * scale, (err, scale)
    assert rel_l2(actual, expected) < rel, rel_l2(actual, expected)


def _joined(seed, h, m, experts, scale_lo=118, scale_hi=127):
    from mlxlr8_b200.joined_mxfp4 import JoinedMXFP4
    from mlxlr8_b200.synthetic import make_joined

    j = make_joined(seed=seed, hidden=h, intermediate=m, experts=experts, scale_lo=scale_lo, scale_hi=scale_hi)
    return j, JoinedMXFP4(j.unit, j.weights, j.scales, h, m)


def _oracle_slots(j, x, ids, dtype="bfloat16"):
    from mlxlr8_b200.synthetic import joined_host_copy

    ids = np.asarray(ids)
    hc = joined_host_copy(j, np.unique(ids[(ids >= 0) & (ids < j.experts)]))
    return ref.joined_slots(host(x), ids, hc["unit"], hc["gate_up"], hc["down"], hc["scales"], j.hidden,
                            j.intermediate, dtype)


def _chunks(rows):
    if rows <= 0:
        return 0
    if rows <= 160:
        return 1
    return (rows - 160 + 127) // 128 + 1


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
def test_slots_match_oracle(dtype):
    import torch

    from helpers import torch_dtype

    j, joined = _joined(seed=3, h=512, m=256, experts=9)
    tokens, slots = 24, 9
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    ids = torch.randint(0, 9, (tokens, slots), generator=g, device="cuda", dtype=torch.int32)
    x, _ = j.tokens(tokens, dtype=torch_dtype(dtype))
    out = joined.slots(x, ids)
    torch.cuda.synchronize()
    assert out.shape == (tokens, slots, 512) and out.dtype == x.dtype
    assert joined.dispatch_header(tokens, slots)[4] == 0
    expected = _oracle_slots(j, x, ids.cpu().numpy(), dtype)
    assert_mxfp4_close(host(out), expected)


def test_finish_matches_oracle():
    import torch

    j, joined = _joined(seed=4, h=512, m=256, experts=17)
    tokens = 40
    g = torch.Generator(device="cuda")
    g.manual_seed(9)
    routed = torch.stack([torch.randperm(16, generator=g, device="cuda")[:8] for _ in range(tokens)]).int()
    ids = torch.cat([routed, torch.full((tokens, 1), 16, dtype=torch.int32, device="cuda")], dim=1)
    scores = torch.rand(tokens, 8, generator=g, device="cuda") * 0.5
    x, residual = j.tokens(tokens)
    out = joined.finish(x, ids, scores, residual)
    torch.cuda.synchronize()
    values = _oracle_slots(j, x, ids.cpu().numpy())
    expected = ref.combine(values, scores.cpu().numpy(), host(residual), "bfloat16")
    assert_mxfp4_close(host(out) - host(residual), expected - host(residual))
    assert_mxfp4_close(host(out), expected)


def test_ragged_segments_and_chunk_boundaries():
    """Experts with 0, 1, 127, 128, 160, 161, 300 and 520 rows: empty
    segments, partial MMA columns, the one-chunk limit (160 rows) and the
    128-row chunking of larger segments (fast_prefill.py:19-46 ragged
    segments)."""
    import torch

    counts = [0, 1, 127, 128, 160, 161, 300, 520]
    j, joined = _joined(seed=5, h=256, m=128, experts=len(counts))
    ids_np = np.concatenate([np.full(c, e, dtype=np.int32) for e, c in enumerate(counts)])
    rng = np.random.default_rng(0)
    rng.shuffle(ids_np)
    tokens = ids_np.size
    ids = torch.from_numpy(ids_np.reshape(tokens, 1)).cuda()
    x, _ = j.tokens(tokens)
    out = joined.slots(x, ids)
    torch.cuda.synchronize()
    header = joined.dispatch_header(tokens, 1)
    assert header[0] == sum(_chunks(c) for c in counts)
    assert header[1] == sum((c + 127) // 128 * 128 for c in counts)
    assert header[4] == 0
    expected = _oracle_slots(j, x, ids_np.reshape(tokens, 1))
    assert_mxfp4_close(host(out), expected)
    for e, c in enumerate(counts):  # every expert's rows, not just the bulk
        sel = ids_np == e
        if c:
            assert_mxfp4_close(host(out)[sel], expected[sel])


def test_out_of_range_ids_give_zero_slots():
    import torch

    j, joined = _joined(seed=6, h=256, m=128, experts=4)
    ids = torch.tensor([[0, 4, 1], [7, 2, 3]], dtype=torch.int32, device="cuda")
    x, _ = j.tokens(2)
    out = host(joined.slots(x, ids))
    torch.cuda.synchronize()
    assert np.all(out[0, 1] == 0) and np.all(out[1, 0] == 0)
    expected = _oracle_slots(j, x, ids.cpu().numpy())
    assert_mxfp4_close(out, expected)


def test_prepared_scale_layout():
    import torch

    from mlxlr8_b200.joined_mxfp4 import _prepare

    rows, k = 256, 512
    src = torch.randint(0, 255, (rows, k // 32), dtype=torch.uint8, device="cuda")
    got = _prepare(src, rows, k, torch.device("cuda")).cpu().numpy()
    s = src.cpu().numpy()
    r = np.arange(rows)[:, None]
    kb = np.arange(k // 32)[None, :]
    offset = ((r // 128) * (k // 128) + kb // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + kb % 4
    np.testing.assert_array_equal(got[offset], s)


def test_wide_scale_range():
    """E8M0 codes over [100, 150] (products spanning 2^-27 .. 2^23)."""
    import torch

    j, joined = _joined(seed=8, h=256, m=128, experts=3, scale_lo=100, scale_hi=150)
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    ids = torch.randint(0, 3, (16, 2), generator=g, device="cuda", dtype=torch.int32)
    x, _ = j.tokens(16, dtype=torch.float32)
    out = joined.slots(x, ids)
    torch.cuda.synchronize()
    expected = _oracle_slots(j, x, ids.cpu().numpy(), "float32")
    assert_mxfp4_close(host(out), expected)


def test_joined_layer_routes_and_matches_oracle():
    import torch

    from mlxlr8_b200.fast_router import router
    from mlxlr8_b200.joined_mxfp4 import JoinedMoELayer

    j, joined = _joined(seed=9, h=256, m=128, experts=257)
    layer = JoinedMoELayer(j.gate_weight, j.bias, joined)
    tokens = 48
    x, residual = j.tokens(tokens)
    out, ids, scores = layer(x, residual, return_routing=True)
    torch.cuda.synchronize()
    assert layer.dispatch_header(tokens)[4] == 0
    logits, ids2, scores2 = router(x, j.gate_weight, j.bias)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids2.cpu().numpy())
    e_ids, e_scores = ref.route(host(logits), j.bias.cpu().numpy())
    np.testing.assert_array_equal(ids.cpu().numpy(), e_ids)
    np.testing.assert_allclose(scores.cpu().numpy(), e_scores, rtol=1e-6, atol=1e-7)
    values = _oracle_slots(j, x, e_ids)
    expected = ref.combine(values, e_scores, host(residual), "bfloat16")
    assert_mxfp4_close(host(out) - host(residual), expected - host(residual))


def test_joined_layer_tensor_core_router():
    """From 64 tokens the layer's gate product runs on the tensor cores; its
    routing equals the oracle's routing of those logits."""
    import torch

    from mlxlr8_b200.fast_router import router_logits
    from mlxlr8_b200.joined_mxfp4 import JoinedMoELayer

    j, joined = _joined(seed=10, h=256, m=128, experts=257)
    layer = JoinedMoELayer(j.gate_weight, j.bias, joined)
    tokens = 300
    x, residual = j.tokens(tokens)
    out, ids, scores = layer(x, residual, return_routing=True)
    logits = router_logits(x, j.gate_weight)
    torch.cuda.synchronize()
    assert layer.dispatch_header(tokens)[4] == 0
    e_ids, e_scores = ref.route(host(logits), j.bias.cpu().numpy())
    np.testing.assert_array_equal(ids.cpu().numpy(), e_ids)
    np.testing.assert_allclose(scores.cpu().numpy(), e_scores, rtol=1e-6, atol=1e-7)
    sample = np.arange(0, tokens, 7)
    values = _oracle_slots(j, x[sample], e_ids[sample])
    expected = ref.combine(values, e_scores[sample], host(residual)[sample], "bfloat16")
    assert_mxfp4_close(host(out)[sample] - host(residual)[sample], expected - host(residual)[sample])


def test_glm_prefill_shape_sampled_tokens():
    """Config-3 shape (hidden 6144, intermediate 2048, 257 experts, 4096
    tokens): the whole layer runs on the GPU; the oracle checks a sample of
    tokens (each token's output depends only on its own nine slots)."""
    import torch

    from mlxlr8_b200.joined_mxfp4 import JoinedMoELayer

    j, joined = _joined(seed=0, h=6144, m=2048, experts=257)
    layer = JoinedMoELayer(j.gate_weight, j.bias, joined)
    tokens = 4096
    x, residual = j.tokens(tokens)
    out, ids, scores = layer(x, residual, return_routing=True)
    torch.cuda.synchronize()
    header = layer.dispatch_header(tokens)
    assert header[4] == 0
    assert header[0] >= 257 and header[1] >= tokens * 9
    sample = np.array([0, 1777, 4095])
    ids_s = ids.cpu().numpy()[sample]
    values = _oracle_slots(j, x[sample], ids_s)
    expected = ref.combine(values, scores.cpu().numpy()[sample], host(residual)[sample], "bfloat16")
    got = host(out)[sample]
    assert_mxfp4_close(got - host(residual)[sample], expected - host(residual)[sample])


@pytest.mark.parametrize("tokens", [700, 4096])
def test_pair_and_single_sm_gemms_agree(tokens):
    """The SM-pair GEMM (two-CTA clusters, M = 256 tcgen05 MMAs with the
    activation tile split between the SMs) issues, per accumulator, the MMAs
    of the one-SM GEMM in the same order: the layer's outputs are identical
    bit for bit, neither form records a pipeline error, and the pair result
    matches the oracle on sampled tokens.  700 tokens give chunks of 16-48
    rows (odd half tiles of 8-row boxes), 4096 tokens full 160-row chunks."""
    import torch

    from mlxlr8_b200 import _lib
    from mlxlr8_b200.joined_mxfp4 import JoinedMoELayer

    lib = _lib.lib()
    j, joined = _joined(seed=21, h=512, m=256, experts=257)
    layer = JoinedMoELayer(j.gate_weight, j.bias, joined)
    x, residual = j.tokens(tokens)
    previous = lib.exlr8_gemm_pair(1)
    try:
        pair, ids, scores = layer(x, residual, return_routing=True)
        pair = pair.clone()
        torch.cuda.synchronize()
        assert layer.dispatch_header(tokens)[4] == 0
        lib.exlr8_gemm_pair(0)
        single = layer(x, residual).clone()
        torch.cuda.synchronize()
        assert layer.dispatch_header(tokens)[4] == 0
    finally:
        lib.exlr8_gemm_pair(previous)
    assert torch.equal(pair, single)
    sample = np.arange(0, tokens, 97)
    values = _oracle_slots(j, x[sample], ids.cpu().numpy()[sample])
    expected = ref.combine(values, scores.cpu().numpy()[sample], host(residual)[sample], "bfloat16")
    assert_mxfp4_close(host(pair)[sample] - host(residual)[sample], expected - host(residual)[sample])


# ---- decode batches (<= 16 tokens): the MXFP4 streaming GEMV ----------------

@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
@pytest.mark.parametrize("tokens, slots", [(1, 9), (2, 3), (5, 9), (16, 9), (3, 20)])
def test_decode_slots_match_oracle(dtype, tokens, slots):
    """Up to 16 token rows the joined products stream through the MXFP4 GEMV
    (groups of up to eight slots per expert, split K)."""
    import torch

    from helpers import torch_dtype

    j, joined = _joined(seed=21 + tokens, h=512, m=256, experts=9)
    g = torch.Generator(device="cuda")
    g.manual_seed(100 + tokens)
    ids = torch.randint(0, 9, (tokens, slots), generator=g, device="cuda", dtype=torch.int32)
    x, _ = j.tokens(tokens, dtype=torch_dtype(dtype))
    out = joined.slots(x, ids)
    torch.cuda.synchronize()
    assert joined.dispatch_header(tokens, slots)[4] == 0
    expected = _oracle_slots(j, x, ids.cpu().numpy(), dtype)
    assert_mxfp4_close(host(out), expected)


@pytest.mark.parametrize("tokens", [1, 4, 16])
def test_decode_finish_and_layer_match_oracle(tokens):
    import torch

    from mlxlr8_b200.fast_router import router
    from mlxlr8_b200.joined_mxfp4 import JoinedMoELayer

    j, joined = _joined(seed=40 + tokens, h=256, m=128, experts=257)
    layer = JoinedMoELayer(j.gate_weight, j.bias, joined)
    x, residual = j.tokens(tokens)
    out, ids, scores = layer(x, residual, return_routing=True)
    torch.cuda.synchronize()
    assert layer.dispatch_header(tokens)[4] == 0
    logits, _, _ = router(x, j.gate_weight, j.bias)
    e_ids, e_scores = ref.route(host(logits), j.bias.cpu().numpy())
    np.testing.assert_array_equal(ids.cpu().numpy(), e_ids)
    np.testing.assert_allclose(scores.cpu().numpy(), e_scores, rtol=1e-6, atol=1e-7)
    values = _oracle_slots(j, x, e_ids)
    expected = ref.combine(values, e_scores, host(residual), "bfloat16")
    assert_mxfp4_close(host(out) - host(residual), expected - host(residual))
    fin = joined.finish(x, ids, scores, residual)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(fin), host(out))


def test_decode_glm_shape_one_token():
    """GLM-5 shape (6144 x 2048, 257 experts) at T = 1, the single-token decode
    size on the joined path."""
    import torch

    from mlxlr8_b200.joined_mxfp4 import JoinedMoELayer

    j, joined = _joined(seed=12, h=6144, m=2048, experts=257)
    layer = JoinedMoELayer(j.gate_weight, j.bias, joined)
    x, residual = j.tokens(1)
    out, ids, scores = layer(x, residual, return_routing=True)
    torch.cuda.synchronize()
    assert layer.dispatch_header(1)[4] == 0
    values = _oracle_slots(j, x, ids.cpu().numpy())
    expected = ref.combine(values, scores.cpu().numpy(), host(residual), "bfloat16")
    assert_mxfp4_close(host(out) - host(residual), expected - host(residual))
