"""EXLR8 checkpoints into device memory (experts.py:16-188), mirroring
test_experts.py: the bounded LRU cache and exact expert byte ranges, resident
buffers and side vectors, bounded-vs-resident parity, the compact routing with
the shared expert against the trellis oracle, optimize on/off agreement, and
the GLM-5-size re-encode to joined MXFP4 at load (experts.py:134-148)."""

import json

import numpy as np
import pytest
from safetensors.numpy import save_file

from helpers import host
from oracle import trellis_oracle as ref

pytestmark = pytest.mark.gpu


@pytest.fixture
def expert_checkpoint(tmp_path):
    """The checkpoint of test_experts.py:13-48 (128 x 128, 256 experts + shared)."""
    directory = tmp_path / "experts"
    directory.mkdir()
    manifests = tmp_path / "manifests"
    manifests.mkdir()
    plan = {"gate": [[4]] * 256, "up": [[4]] * 256, "down": [4] * 256,
            "shared": {"gate": [4], "up": [4], "down": 4}}
    (manifests / "exlr8-manifest-up1.json").write_text(json.dumps({"name": "up1", "layers": {"3": plan}}))
    rng = np.random.default_rng(17)
    raw = {}
    index = {"signs.in": rng.choice([-1, 1], 128).astype(np.int8),
             "signs.out": rng.choice([-1, 1], 128).astype(np.int8)}
    for projection in ("gate", "up", "down"):
        raw["trellis." + projection] = rng.integers(0, 256, 256 * 8192, dtype=np.uint8)
        raw["shared.trellis." + projection] = rng.integers(0, 256, 8192, dtype=np.uint8)
        block_name = "sv_block" if projection == "down" else "su_block"
        channel_name = "suh" if projection == "down" else "svh"
        for prefix, count in (("k4", 256), ("shared.k4", 1)):
            index[f"{prefix}.{projection}.{block_name}"] = rng.uniform(0.01, 0.02, (count, 1)).astype(np.float16)
            index[f"{prefix}.{projection}.{channel_name}"] = rng.uniform(-1, 1, (count, 128)).astype(np.float16)
    save_file(raw, str(directory / "exlr8-layer-003.k4.safetensors"))
    save_file(index, str(directory / "exlr8-layer-003.index.safetensors"))
    return tmp_path, raw


def _oracle_slots(layer, raw, x, ids, dtype):
    packed = {p: np.concatenate([raw["trellis." + p], raw["shared.trellis." + p]]) for p in ("gate", "up", "down")}
    scales = {p: tuple(host(s) for s in layer.scales[p]) for p in ("gate", "up", "down")}
    return ref.expert_mlp(host(x), ids.cpu().numpy(), packed, scales, 4, 128, 128, dtype=dtype)


@pytest.mark.parametrize("optimize", [False, True])
def test_compact_routing_shared_expert_and_side_scales(expert_checkpoint, optimize):
    import torch

    from mlxlr8_b200.experts import ExpertStore

    path, raw = expert_checkpoint
    store = ExpertStore(path, cache_gib=1, optimize=optimize)
    layer = store.layer(3)
    x = torch.from_numpy(np.random.default_rng(20).normal(size=(2, 128)).astype(np.float32)).cuda()
    ids = torch.tensor([[256, 9, 2], [2, 9, 2]], dtype=torch.int32, device="cuda")
    actual = layer(x, ids)
    torch.cuda.synchronize()
    expected = _oracle_slots(layer, raw, x, ids, "float32")
    np.testing.assert_allclose(host(actual), expected, rtol=2e-4, atol=1e-6)


def test_cache_limit_and_exact_expert_range(expert_checkpoint):
    from mlxlr8_b200.experts import ExpertStore

    path, raw = expert_checkpoint
    size = 3 * 8192
    store = ExpertStore(path, cache_gib=size * 2 / 1024**3)
    layer = store.layer(3)
    for expert in (4, 8, 4, 12):
        values = store._get(layer, expert)
        np.testing.assert_array_equal(values[0].cpu().numpy(), raw["trellis.gate"][expert * 8192:(expert + 1) * 8192])
    assert set(store.cache) == {(3, 4), (3, 12)}
    assert store.cache_bytes == 2 * size
    assert store.stats()["hits"] == 1
    assert store.stats()["misses"] == 3
    shared = store._get(layer, 256)
    np.testing.assert_array_equal(shared[0].cpu().numpy(), raw["shared.trellis.gate"])
    np.testing.assert_array_equal(shared[2].cpu().numpy(), raw["shared.trellis.down"])


def test_resident_weights_scales_and_two_token_parity(expert_checkpoint):
    import torch

    from mlxlr8_b200.experts import ExpertStore

    path, raw = expert_checkpoint
    bounded = ExpertStore(path, cache_gib=1)
    resident = ExpertStore(path, resident=True)
    layer = resident.layer(3)
    x = torch.from_numpy(np.random.default_rng(30).normal(size=(2, 128)).astype(np.float32)).cuda().to(torch.bfloat16)
    ids = torch.tensor([[256, 9, 2], [2, 255, 256]], dtype=torch.int32, device="cuda")
    expected = bounded.layer(3)(x, ids)
    actual = layer(x, ids)
    np.testing.assert_array_equal(host(actual), host(expected))
    for projection in ("gate", "up", "down"):
        np.testing.assert_array_equal(layer.packed[projection].cpu().numpy(),
                                      np.concatenate([raw["trellis." + projection], raw["shared.trellis." + projection]]))
        for a, b in zip(layer.scales[projection], bounded.layer(3).scales[projection]):
            np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy())
    assert resident.stats()["resident_bytes"] == 3 * 257 * (8192 + 2 * 128 * 2)
    assert resident.cache_bytes == resident.hits == resident.misses == 0
    assert resident.layer(3) is layer


def test_bounded_rejects_out_of_range_ids(expert_checkpoint):
    import torch

    from mlxlr8_b200.experts import ExpertStore

    path, _ = expert_checkpoint
    layer = ExpertStore(path, cache_gib=1).layer(3)
    x = torch.ones(1, 128, device="cuda")
    with pytest.raises(ValueError, match="Expert IDs must be in 0..256"):
        layer(x, torch.tensor([[257, 1]], dtype=torch.int32, device="cuda"))


def test_grouped_prefill_routing_matches_reference(expert_checkpoint):
    import torch

    from mlxlr8_b200.experts import ExpertStore

    path, _ = expert_checkpoint
    rng = np.random.default_rng(31)
    x = torch.from_numpy(rng.normal(size=(17, 128)).astype(np.float32)).cuda()
    ids = torch.from_numpy(np.column_stack([rng.integers(0, 256, (17, 2)), np.full(17, 256)]).astype(np.int32)).cuda()
    reference = ExpertStore(path, resident=True, optimize=False).layer(3)(x, ids)
    actual = ExpertStore(path, resident=True).layer(3)(x, ids)
    np.testing.assert_allclose(host(actual), host(reference), rtol=5e-4, atol=2e-7)


def test_glm5_layer_reencodes_to_joined_mxfp4(tmp_path):
    """A K4 layer of GLM-5 size (6144 x 2048; 8 routed experts + shared here)
    is re-encoded on load: trellis codes and gate/up in-scales released, the
    joined weights equal to the oracle encode of the file's bytes, and the
    store's MoE layer (router from the dense file) is the joined one."""
    import torch

    from mlxlr8_b200.experts import ExpertStore
    from mlxlr8_b200.joined_mxfp4 import JoinedMoELayer
    from mlxlr8_b200.synthetic import write_checkpoint
    from mlxlr8_b200.weights import SafeTensorFile

    h, m, routed = 6144, 2048, 8
    write_checkpoint(tmp_path, layers=(3,), hidden=h, intermediate=m, routed=routed, seed=4)
    store = ExpertStore(tmp_path, resident=True)
    layer = store.layer(3)
    assert layer.affine is not None and layer.packed is None
    assert layer.scales["gate"][0] is None and layer.scales["up"][0] is None
    torch.cuda.synchronize()
    f = SafeTensorFile(tmp_path / "experts" / "exlr8-layer-003.k4.safetensors")
    packed = {p: np.concatenate([f.raw("trellis." + p), f.raw("shared.trellis." + p)]) for p in ("gate", "up", "down")}
    plain = ExpertStore(tmp_path, resident=True, optimize=False).layer(3)
    scales16 = {p: tuple(s.cpu().numpy() for s in plain.scales[p]) for p in ("gate", "up", "down")}
    check = (1, routed)  # a routed expert and the shared one
    _, expected = ref.encode_joined(packed, scales16, 4, h, m, experts=check)
    for name in ("gate_up", "down"):
        for i in check:
            np.testing.assert_array_equal(layer.affine.weights[name][0][i].cpu().numpy().view(np.uint32),
                                          expected[name][0][i])
            np.testing.assert_array_equal(layer.affine.weights[name][1][i].cpu().numpy(), expected[name][1][i])
    matrices = routed + 1
    mx_bytes = matrices * (3 * h * m // 2 + 3 * h * m // 32)
    side = matrices * (2 * m + m + h) * 2  # gate/up out-scales, down in/out-scales (fp16)
    assert store.stats()["resident_bytes"] == mx_bytes + side + h * 2
    moe = store.moe_layer(3)
    assert isinstance(moe, JoinedMoELayer)
    gate_weight, bias = store.router(3)
    assert gate_weight.dtype == torch.float32 and tuple(gate_weight.shape) == (256, h)


def test_expert_parallel_layer_from_checkpoint_shards(tmp_path):
    """ExpertStore.ep_layer at one rank (the whole routed set as its shard, the
    trellis shared expert replicated) against the resident single-device
    layer built from the same checkpoint."""
    import torch

    from helpers import assert_bf16_close
    from mlxlr8_b200.experts import ExpertStore
    from mlxlr8_b200.synthetic import write_checkpoint

    write_checkpoint(tmp_path, layers=(3,), hidden=256, intermediate=128, routed=256, seed=8)
    store = ExpertStore(tmp_path, resident=True, optimize=False)
    single = store.moe_layer(3)
    ep = store.ep_layer(3, 0, 1)
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    x = torch.randn(4, 256, generator=g, device="cuda").to(torch.bfloat16)
    r = torch.randn(4, 256, generator=g, device="cuda").to(torch.bfloat16)
    out, ids, _ = single(x, r, return_routing=True)
    out_ep, ids_ep, _ = ep(x, r, return_routing=True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_ep.cpu().numpy())
    assert_bf16_close(host(out_ep) - host(r), host(out) - host(r))
