"""Static hot-expert cache on the GPU: the expansion kernel against the
reference's own bytes and the oracle, and the cache's decode (bit-equal with
the layer's, as test_static_cache.py requires)."""

import numpy as np
import pytest

from helpers import host
from oracle import trellis_oracle as ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("k", [2, 3, 4])
@pytest.mark.parametrize("side", [1, 2])
def test_expansion_matches_reference_bytes(golden, k, side):
    import torch

    from mlxlr8_b200.static_cache import expand_static_trellis

    a, b = (128, 256) if side == 1 else (256, 128)
    packed = torch.from_numpy(golden[f"static_k{k}_s{side}_packed"]).cuda()
    out = expand_static_trellis(packed, k, a, b, side)
    torch.cuda.synchronize()
    assert out.dtype == torch.uint8 and out.numel() == 2 * a * b
    np.testing.assert_array_equal(out.cpu().numpy(), golden[f"static_k{k}_s{side}_bytes"])


@pytest.mark.parametrize("k", [3, 4])
def test_expansion_full_glm_matrix(k):
    """One expert's gate (side 1, 6144 x 2048) and down (side 2, 2048 x 6144)
    matrices at full size against the oracle."""
    import torch

    from mlxlr8_b200.static_cache import expand_static_trellis

    rng = np.random.default_rng(70 + k)
    for a, b, side in ((6144, 2048, 1), (2048, 6144, 2)):
        raw = rng.integers(0, 256, a * b * k // 8, np.uint8)
        out = expand_static_trellis(torch.from_numpy(raw).cuda(), k, a, b, side)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), ref.expand_static(raw, k, a, b, side))


@pytest.mark.parametrize("k", [3, 4])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("hot", [[10], [0, 1, 2, 10]])
def test_static_decode_is_bit_equal_with_cached_and_uncached_experts(k, dtype, hot):
    import torch

    from helpers import torch_dtype
    from mlxlr8_b200.fast_decode import fast_expert_mlp
    from mlxlr8_b200.static_cache import StaticExpertCache
    from mlxlr8_b200.synthetic import make_layer

    layer = make_layer(seed=9, k=k, hidden=256, intermediate=384, routed=12, shared="none").experts
    cache = StaticExpertCache(layer, hot)
    size = 256 * 384
    for p in ("gate", "up", "down"):
        a, b, side = (384, 256, 2) if p == "down" else (256, 384, 1)
        src = layer.packed[p].cpu().numpy()
        want = np.concatenate([ref.expand_static(src[e * size * k // 8:(e + 1) * size * k // 8], k, a, b, side)
                               for e in hot])
        np.testing.assert_array_equal(cache.fp8[p].cpu().numpy(), want)
    slot_map = cache.expert_to_slot.cpu().numpy().view(np.uint32)
    assert cache.expert_to_slot.dtype == torch.int32 and slot_map.size == 12
    np.testing.assert_array_equal(slot_map[hot], np.arange(len(hot)))
    assert np.all(np.delete(slot_map, hot) == 0xFFFFFFFF)
    assert cache.stats()["weight_bytes"] == 3 * size * len(hot)
    ids = torch.tensor([[2, 0, 10], [1, 7, 10]], dtype=torch.int32, device="cuda")
    g = torch.Generator(device="cuda")
    g.manual_seed(15)
    x = torch.randn(2, 256, generator=g, device="cuda").to(torch_dtype(dtype))
    expected = fast_expert_mlp(x, ids, layer.packed, layer.scales, k, 256, 384)
    actual = cache(x, ids)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(actual).view(np.uint32), host(expected).view(np.uint32))


def test_static_cache_needs_resident_codes():
    from mlxlr8_b200.static_cache import StaticExpertCache
    from mlxlr8_b200.synthetic import make_layer

    layer = make_layer(seed=9, hidden=256, intermediate=384, routed=4, shared="none").experts
    layer.packed = None
    with pytest.raises(ValueError, match="resident packed weights"):
        StaticExpertCache(layer, [1])


def _bit_equal_cached(layer, hot, ids, x):
    import torch

    from mlxlr8_b200.fast_decode import fast_expert_mlp
    from mlxlr8_b200.static_cache import StaticExpertCache

    cache = StaticExpertCache(layer, hot)
    expected = fast_expert_mlp(x, ids, layer.packed, layer.scales, layer.k, layer.hidden, layer.intermediate)
    actual = cache(x, ids)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(actual).view(np.uint32), host(expected).view(np.uint32))


def test_static_decode_k2_and_shared_rows():
    """K2 (two K tiles per hot stage) with eight rows on one cached expert,
    which fills both fragment column groups of a unit."""
    import torch

    from mlxlr8_b200.synthetic import make_layer

    layer = make_layer(seed=12, k=2, hidden=256, intermediate=384, routed=12, shared="none").experts
    ids = torch.tensor([[10, 3, 5]] * 8, dtype=torch.int32, device="cuda")
    g = torch.Generator(device="cuda")
    g.manual_seed(16)
    x = torch.randn(8, 256, generator=g, device="cuda").to(torch.bfloat16)
    _bit_equal_cached(layer, [10, 3], ids, x)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_static_decode_full_glm_dimensions(dtype):
    """GLM-5 size (6144 x 2048, K4) with one cached expert among the eight of
    a token (fast_decode tests' full-size case)."""
    import torch

    from helpers import torch_dtype
    from mlxlr8_b200.synthetic import make_layer

    layer = make_layer(seed=13, routed=24, shared="none").experts
    ids = torch.tensor([[8, 1, 2, 3, 4, 5, 6, 7, 23]], dtype=torch.int32, device="cuda")
    g = torch.Generator(device="cuda")
    g.manual_seed(17)
    x = torch.randn(1, 6144, generator=g, device="cuda").to(torch_dtype(dtype))
    _bit_equal_cached(layer, [8, 23], ids, x)
