"""Static hot-expert cache host logic and the oracle's tile bytes
(test_static_cache.py of the reference, without Metal)."""

import numpy as np
import pytest

from oracle import trellis_oracle as ref


def test_hot_slots_keep_the_given_order():
    from mlxlr8_b200.static_cache import _hot_slots

    assert _hot_slots([256, 17, 3], 257) == (256, 17, 3)
    assert _hot_slots(np.array([5, 0], np.uint32), 257) == (5, 0)


@pytest.mark.parametrize("ids", [[], [1.5], [-1], [257], [3, 3], [[3]], [True]])
def test_invalid_hot_ids(ids):
    from mlxlr8_b200.static_cache import _hot_slots

    with pytest.raises(ValueError):
        _hot_slots(ids, 257)


def test_static_memory_budget():
    from mlxlr8_b200.static_cache import static_cache_bytes

    assert static_cache_bytes(6144, 2048, 1) == 37749764
    assert 75 * static_cache_bytes(6144, 2048, 18) < 48 * 1024**3
    assert 75 * static_cache_bytes(6144, 2048, 19) > 48 * 1024**3


@pytest.mark.parametrize("k", [2, 3, 4])
@pytest.mark.parametrize("side", [1, 2])
def test_static_tile_bytes_match_the_decoded_matrix(k, side):
    """Byte 8*lane+j of each stored tile is the E4M3 code of the decoded
    weight at that lane's fragment position, tiles in storage order."""
    h, m = 256, 384
    raw = np.random.default_rng(53).integers(0, 256, h * m * k // 8, np.uint8)
    matrix = ref.decode_trellis(raw, k, h, m, side)
    tiles = matrix.reshape(h // 16, 16, m // 16, 16).transpose(0, 2, 1, 3)
    lane, j = np.arange(256) // 8, np.arange(256) % 8
    position = ((lane & 3) * 2 + (j & 1) + (j & 2) * 4) * 16 + (lane >> 2) + (j & 4) * 2
    tiles = tiles.reshape(h // 16, m // 16, 256)[..., position]
    if side == 2:
        tiles = tiles.reshape(h // 128, 8, m // 128, 8, 256).transpose(0, 2, 1, 3, 4)
    else:
        tiles = tiles.reshape(h // 16, m // 128, 8, 256).transpose(1, 0, 2, 3)
    np.testing.assert_array_equal(ref.expand_static(raw, k, h, m, side), ref.e4m3_code(tiles).reshape(-1))


def test_fast_expert_mlp_takes_cache_bytes_and_map_together():
    import torch

    from mlxlr8_b200.fast_decode import fast_expert_mlp

    x, ids = torch.zeros(1, 256), torch.zeros(1, 3, dtype=torch.int32)
    with pytest.raises(ValueError, match="go together"):
        fast_expert_mlp(x, ids, {}, {}, 4, 256, 384, fp8={"gate": x, "up": x, "down": x})
    with pytest.raises(ValueError, match="gate, up and down"):
        fast_expert_mlp(x, ids, {}, {}, 4, 256, 384, fp8={"gate": x}, expert_to_slot=ids)
