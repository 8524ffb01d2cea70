"""EXLR8 checkpoint reading without a GPU: the safetensors reader
(weights.py:20-69), the up1 manifest checks and the signed side vectors of
``ExpertStore.layer`` (experts.py:16-33, 77-115), the router record
(dense.py:174-191), on the reference's own fixture layout
(test_experts.py:13-48, written with ``safetensors.numpy.save_file``) and on
``synthetic.write_checkpoint`` directories."""

import json

import numpy as np
import pytest
from safetensors.numpy import save_file

from mlxlr8_b200.experts import ExpertStore, load_router
from mlxlr8_b200.synthetic import write_checkpoint
from mlxlr8_b200.weights import SafeTensorFile


@pytest.fixture
def reference_checkpoint(tmp_path):
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
    return tmp_path, raw, index


def test_safetensor_reader_matches_writer(reference_checkpoint):
    path, raw, index = reference_checkpoint
    f = SafeTensorFile(path / "experts" / "exlr8-layer-003.index.safetensors")
    assert set(f.tensors) == set(index)
    for name, value in index.items():
        got = f.raw(name)
        assert got.dtype == value.dtype and got.shape == value.shape
        np.testing.assert_array_equal(got, value)
    w = SafeTensorFile(path / "experts" / "exlr8-layer-003.k4.safetensors")
    np.testing.assert_array_equal(w.raw("trellis.up", 9 * 8192, 8192), raw["trellis.up"][9 * 8192:10 * 8192])
    np.testing.assert_array_equal(f.raw("k4.gate.svh", 2 * 128 * 2, 4), index["k4.gate.svh"].reshape(-1)[256:258])


@pytest.mark.parametrize("start, count", [(-2, 2), (0, 10 ** 9), (1, 2), (2, 3)])
def test_invalid_byte_ranges(reference_checkpoint, start, count):
    path, _, _ = reference_checkpoint
    f = SafeTensorFile(path / "experts" / "exlr8-layer-003.index.safetensors")
    with pytest.raises(ValueError, match="invalid byte range for k4.gate.svh"):
        f.raw("k4.gate.svh", start, count)


def test_truncated_file(reference_checkpoint, tmp_path):
    path, _, _ = reference_checkpoint
    source = path / "experts" / "exlr8-layer-003.k4.safetensors"
    cut = tmp_path / "cut.safetensors"
    cut.write_bytes(source.read_bytes()[:-100])
    f = SafeTensorFile(cut)
    last = max(f.tensors, key=lambda name: f.tensors[name]["data_offsets"][1])
    with pytest.raises(ValueError, match=f"truncated tensor {last}"):
        f.raw(last)


def test_signed_side_vectors(reference_checkpoint):
    """experts.py:97-115: hidden side = repeat(block, 128) * signs, shared expert last."""
    path, _, index = reference_checkpoint
    layer = ExpertStore(path, device="cpu").layer(3)
    assert (layer.k, layer.hidden, layer.intermediate, layer.expert_bytes) == (4, 128, 128, 8192)
    assert layer.experts == 257
    for projection in ("gate", "up", "down"):
        block_name = "sv_block" if projection == "down" else "su_block"
        channel_name = "suh" if projection == "down" else "svh"
        signs = index["signs.out" if projection == "down" else "signs.in"].astype(np.float16)
        block = np.concatenate([index[f"k4.{projection}.{block_name}"], index[f"shared.k4.{projection}.{block_name}"]])
        hidden = np.repeat(block, 128, axis=-1) * signs
        channel = np.concatenate([index[f"k4.{projection}.{channel_name}"],
                                  index[f"shared.k4.{projection}.{channel_name}"]])
        want = (channel, hidden) if projection == "down" else (hidden, channel)
        for got, expected in zip(layer.scales[projection], want):
            assert got.dtype.is_floating_point and got.element_size() == 2
            np.testing.assert_array_equal(got.numpy(), expected)


def test_manifest_and_width_checks(reference_checkpoint):
    path, _, _ = reference_checkpoint
    manifest = path / "manifests" / "exlr8-manifest-up1.json"
    with pytest.raises(ValueError, match="cache_gib must be nonnegative"):
        ExpertStore(path, cache_gib=-1)
    data = json.loads(manifest.read_text())
    data["layers"]["3"]["down"][7] = 3
    manifest.write_text(json.dumps(data))
    with pytest.raises(ValueError, match="Layer 3 is not uniform K4"):
        ExpertStore(path, device="cpu").layer(3)
    data["name"] = "up2"
    manifest.write_text(json.dumps(data))
    with pytest.raises(ValueError, match="This loader requires the up1 manifest"):
        ExpertStore(path)


def test_synthetic_checkpoint_layers_and_router(tmp_path):
    write_checkpoint(tmp_path, layers=(3, 78), hidden=256, intermediate=128, routed=4, seed=2)
    store = ExpertStore(tmp_path, device="cpu")
    assert store.layer(3).k == 4 and store.layer(78).k == 3
    assert store.layer(3) is store.layer(3)
    assert store.layer(78).expert_bytes == 256 * 128 * 3 // 8
    weight, bias = load_router(tmp_path, 3, "cpu")
    assert tuple(weight.shape) == (256, 256) and str(weight.dtype) == "torch.float32"
    bits = SafeTensorFile(tmp_path / "dense" / "exlr8-dense-003.safetensors").raw("mlp.gate.bf16")
    np.testing.assert_array_equal(weight.numpy(), (bits.astype(np.uint32) << 16).view(np.float32))
    assert tuple(bias.shape) == (256,)
    write_checkpoint(tmp_path / "f32", layers=(5,), hidden=128, intermediate=128, routed=2, router_format=7)
    weight, _ = load_router(tmp_path / "f32", 5, "cpu")
    np.testing.assert_array_equal(
        weight.numpy(), SafeTensorFile(tmp_path / "f32" / "dense" / "exlr8-dense-005.safetensors").raw("mlp.gate.fp32"))


def test_shard_reads_only_the_rank_experts(reference_checkpoint):
    """Expert-parallel shards: rank r of 4 holds experts [64 r, 64 r + 64)
    and the shared expert, with the matching signed side vectors."""
    path, raw, _ = reference_checkpoint
    store = ExpertStore(path, device="cpu")
    full = store.layer(3)
    for rank in (0, 3):
        local, shared = store.shard(3, rank, 4)
        assert local.experts == 64 and shared.experts == 1
        lo = 64 * rank
        for projection in ("gate", "up", "down"):
            np.testing.assert_array_equal(local.packed[projection].numpy(),
                                          raw["trellis." + projection][lo * 8192:(lo + 64) * 8192])
            np.testing.assert_array_equal(shared.packed[projection].numpy(), raw["shared.trellis." + projection])
            for a, b in zip(local.scales[projection], full.scales[projection]):
                np.testing.assert_array_equal(a.numpy(), b[lo:lo + 64].numpy())
            for a, b in zip(shared.scales[projection], full.scales[projection]):
                np.testing.assert_array_equal(a.numpy(), b[256:257].numpy())
    with pytest.raises(ValueError, match="divide evenly"):
        store.shard(3, 0, 3)
