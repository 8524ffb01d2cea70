"""Static hot-expert cache host logic and the oracle's tile bytes
(test_static_cache.py of the reference, without Metal)."""

import numpy as np
import pytest

from oracle import trellis_oracle as ref


def test_map_keeps_the_given_slot_order_and_miss_sentinel():
    from mlxlr8_b200.static_cache import _expert_map

    ids, mapping = _expert_map([256, 17, 3], 257)
    assert ids == (256, 17, 3)
    assert mapping.dtype == np.uint32
    np.testing.assert_array_equal(mapping[[256, 17, 3]], [0, 1, 2])
    assert np.all(mapping[np.setdiff1d(np.arange(257), [256, 17, 3])] == 0xFFFFFFFF)


@pytest.mark.parametrize("ids", [[], [1.5], [-1], [257], [3, 3], [[3]]])
def test_invalid_hot_ids(ids):
    from mlxlr8_b200.static_cache import _expert_map

    with pytest.raises(ValueError):
        _expert_map(ids, 257)


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


def test_hot_lists_use_train_routes_only_and_break_ties_by_id():
    """tools/static_cache_routes.py via test_static_cache.py's trace."""
    from mlxlr8_b200.static_cache import fixed_hot_lists

    trace = {"layers": {"3": {"routes": [[8, 4, 256], [4, 8, 256], [17, 8, 256], [17, 4, 256]]}}}
    result = fixed_hot_lists(trace, split=2, capacities=(1, 2, 3))
    assert result["layers"]["3"]["2"]["expert_ids"] == [256, 4]
    assert result["layers"]["3"]["3"]["expert_ids"] == [256, 4, 8]
    assert result["totals"]["heldout"]["3"]["hit_rate"] == 4 / 6
    assert result["totals"]["heldout"]["3"]["routed_hit_rate"] == 2 / 4
    assert result["totals"]["heldout"]["1"]["all_selected_hit_token_rate"] == 0
    assert result["totals"]["train"]["3"]["all_selected_hit_token_rate"] == 1


def test_hot_lists_require_a_complete_split():
    from mlxlr8_b200.static_cache import fixed_hot_lists

    with pytest.raises(ValueError, match="needs 2 routes"):
        fixed_hot_lists({"layers": {"3": {"routes": [[0, 256]]}}}, split=1)


def test_hot_list_command_writes_the_lists(tmp_path, capsys):
    import json

    from mlxlr8_b200.static_cache import main

    routes = [[e % 5, (e + 1) % 5, 256] for e in range(512)]
    (tmp_path / "trace.json").write_text(json.dumps({"layers": {"5": {"routes": routes}}}))
    main([str(tmp_path / "trace.json"), "--output", str(tmp_path / "hot.json")])
    result = json.loads((tmp_path / "hot.json").read_text())
    assert result["layers"]["5"]["9"]["expert_ids"][:1] == [256]
    assert len(result["layers"]["5"]["9"]["expert_ids"]) == 6  # five routed ids in the trace
    assert result["source"].endswith("trace.json")
    assert "heldout" in capsys.readouterr().out
