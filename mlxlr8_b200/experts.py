"""Expert store and expert layers (``exlr8/experts.py``).

``ExpertStore(path, cache_gib, resident, optimize)`` reads an EXLR8
checkpoint directory (``manifests/exlr8-manifest-up1.json``,
``experts/exlr8-layer-NNN.k{3,4}.safetensors`` and
``experts/exlr8-layer-NNN.index.safetensors``) straight into device memory:

* ``store.layer(n)`` builds the layer once (experts.py:35-38, 77-148): the
  uniform-K check of the manifest, the signed side vectors
  ``repeat(block, 128) * signs`` from the index (experts.py:97-115), and in
  resident mode the packed codes of the 256 routed experts followed by the
  shared expert as one device buffer per projection (experts.py:116-124).
  With ``optimize`` a K4 layer of GLM-5 size is re-encoded to joined MXFP4 on
  the GPU (experts.py:134-148) and its trellis codes and gate/up in-scales
  are released.
* ``store.shard(n, rank, world)`` reads one rank's contiguous block of routed
  experts plus the shared expert (expert parallelism; ``store.ep_layer``
  builds the sharded MoE layer).
* Without ``resident``, ``store._get(layer, expert)`` reads one expert's
  three matrices into a byte-bounded LRU cache on the device
  (experts.py:40-64), and the layer gathers the selected experts per call
  (experts.py:155-169).

``ExpertLayer(x, ids)`` returns ``[*ids.shape, hidden]`` per-slot outputs in
the activation dtype (experts.py:150-188).  A layer can also be built from
device tensors: ``packed[p]`` (uint8 grouped128 bytes of all experts, the
shared expert last when it is a trellis matrix) and ``scales[p] = (in, out)``;
an optional dense bf16 shared expert (``shared = (gate, up, down)``) is then
used by the layer finish instead of trellis matrix 256.
"""

from __future__ import annotations

import json
from collections import OrderedDict
from pathlib import Path

import torch

from .fast_decode import compiled_expert_mlp_finish, fast_expert_mlp


class ExpertStore:
    def __init__(self, path, cache_gib=32, resident=False, optimize=True, device=None):
        self.path = Path(path)
        self.resident = resident
        self.optimize = optimize
        self.manifest = json.loads((self.path / "manifests/exlr8-manifest-up1.json").read_text())
        if self.manifest["name"] != "up1":
            raise ValueError("This loader requires the up1 manifest")
        self.limit = int(cache_gib * 1024**3)
        if self.limit < 0:
            raise ValueError("cache_gib must be nonnegative")
        self._device = None if device is None else torch.device(device)
        self.cache = OrderedDict()
        self.cache_bytes = 0
        self.resident_bytes = 0
        self.hits = 0
        self.misses = 0
        self._layers = {}

    @property
    def device(self):
        if self._device is None:
            self._device = torch.device("cuda", torch.cuda.current_device())
        return self._device

    def layer(self, number):
        if number not in self._layers:
            self._layers[number] = _load_layer(self, number)
        return self._layers[number]

    def _get(self, layer, expert):
        """(gate, up, down) packed bytes of one expert (256 = shared) on the device."""
        key = (layer.number, expert)
        if key in self.cache:
            self.hits += 1
            self.cache.move_to_end(key)
            return self.cache[key]
        self.misses += 1
        shared = expert == 256
        prefix = "shared." if shared else ""
        start = 0 if shared else expert * layer.expert_bytes
        arrays = tuple(layer.weights.load_slice(prefix + "trellis." + projection, start, layer.expert_bytes,
                                                self.device)
                       for projection in ("gate", "up", "down"))
        size = 3 * layer.expert_bytes
        if size <= self.limit:
            while self.cache_bytes + size > self.limit:
                _, old = self.cache.popitem(last=False)
                self.cache_bytes -= sum(a.numel() for a in old)
            self.cache[key] = arrays
            self.cache_bytes += size
        return arrays

    def shard(self, number, rank, world, routed=256):
        """(routed shard, shared expert) of layer ``number`` for expert
        parallelism over ``world`` ranks: this rank's contiguous block of
        routed / world experts and the shared expert (matrix 256), read from
        the checkpoint by their byte ranges only, so a rank holds 1 / world
        of the routed codes."""
        return _load_shard(self, number, rank, world, routed)

    def ep_layer(self, number, rank, world, group=None, routed=256):
        """The MoE branch of layer ``number`` sharded over ``world`` ranks
        (``ep.ExpertParallelMoE``, NCCL exchange, the trellis shared expert
        replicated on every rank)."""
        from .ep import ExpertParallelMoE

        gate_weight, bias = self.router(number)
        local, shared = self.shard(number, rank, world, routed)
        return ExpertParallelMoE(gate_weight, bias, local, rank, world, group=group, shared_layer=shared,
                                 routed=routed, exchange="nccl")

    def router(self, number):
        """(gate weight float32 [256, hidden], bias float32 [256]) of layer
        ``number`` from ``dense/exlr8-dense-NNN.safetensors`` (model.py:361-371)."""
        return load_router(self.path, number, self.device)

    def moe_layer(self, number):
        """The MoE branch of decoder layer ``number`` (model.py:385-418): router
        plus this store's experts, joined MXFP4 when the layer was re-encoded."""
        from .joined_mxfp4 import JoinedMoELayer
        from .moe import MoELayer

        gate_weight, bias = self.router(number)
        experts = self.layer(number)
        if experts.affine is not None:
            return JoinedMoELayer(gate_weight, bias, experts.affine)
        if not self.resident:
            raise ValueError("the fused MoE layer needs resident experts")
        return MoELayer(gate_weight, bias, experts)

    def stats(self):
        return {
            "cache_bytes": self.cache_bytes,
            "cache_limit_bytes": self.limit,
            "resident_bytes": self.resident_bytes,
            "hits": self.hits,
            "misses": self.misses,
        }


def load_router(path, number, device=None):
    """Router of decoder layer ``number``: the ``mlp.gate`` matrix record of
    the dense file (dense.py:174-191; format 6 = bf16, 7 = float32, [256,
    hidden]) widened to float32 as model.py:366-370 does, and
    ``mlp.gate.e_score_correction_bias`` as float32."""
    from .weights import SafeTensorFile

    file = SafeTensorFile(Path(path) / "dense" / f"exlr8-dense-{number:03d}.safetensors")
    record = tuple(int(v) for v in file.raw("mlp.gate.record").reshape(-1).tolist())
    if record[0] not in (6, 7):
        raise ValueError(f"unsupported EXLR8 dense format {record[0]} for the router gate")
    weight = file.load("mlp.gate." + ("bf16" if record[0] == 6 else "fp32"), device).to(torch.float32)
    if tuple(weight.shape) != (record[1], record[2]):
        raise ValueError("router gate shape does not match its record")
    bias = file.load("mlp.gate.e_score_correction_bias", device).to(torch.float32)
    return weight.contiguous(), bias.contiguous()


def _layer_scales(index, k, device):
    """Signed side vectors of the 256 routed experts and the shared expert
    (experts.py:97-115): the hidden side is ``repeat(block, 128) * signs``
    (signs.in for gate/up, signs.out for down), the other side the stored
    channel vector; fp16 as stored."""
    import numpy as np

    signs_in = index.raw("signs.in").astype(np.float16)
    signs_out = index.raw("signs.out").astype(np.float16)
    scales = {}
    for projection in ("gate", "up", "down"):
        block_name = "sv_block" if projection == "down" else "su_block"
        channel_name = "suh" if projection == "down" else "svh"
        block = np.concatenate([index.raw(f"k{k}.{projection}.{block_name}"),
                                index.raw(f"shared.k{k}.{projection}.{block_name}")])
        channel = np.concatenate([index.raw(f"k{k}.{projection}.{channel_name}"),
                                  index.raw(f"shared.k{k}.{projection}.{channel_name}")])
        hidden_scale = np.repeat(block, 128, axis=-1)
        hidden_scale *= signs_out if projection == "down" else signs_in
        pair = (channel, hidden_scale) if projection == "down" else (hidden_scale, channel)
        scales[projection] = tuple(torch.from_numpy(np.ascontiguousarray(a)).to(device) for a in pair)
    return scales


def _layer_files(store, number):
    """(k, weights file, index file, hidden, intermediate) of layer ``number``
    after the manifest's uniform-K check (experts.py:80-94)."""
    from .weights import SafeTensorFile

    plan = store.manifest["layers"][str(number)]
    widths = {v for rows in (plan["gate"], plan["up"]) for row in rows for v in row}
    widths.update(plan["down"])
    widths.update(plan["shared"]["gate"])
    widths.update(plan["shared"]["up"])
    widths.add(plan["shared"]["down"])
    k = 3 if number == 78 else 4
    if widths != {k}:
        raise ValueError(f"Layer {number} is not uniform K{k}")
    directory = store.path / "experts"
    weights = SafeTensorFile(directory / f"exlr8-layer-{number:03d}.k{k}.safetensors")
    index = SafeTensorFile(directory / f"exlr8-layer-{number:03d}.index.safetensors")
    hidden = index.header["signs.in"]["shape"][0]
    intermediate = index.header[f"k{k}.gate.svh"]["shape"][-1]
    return k, weights, index, hidden, intermediate


def _load_shard(store, number, rank, world, routed):
    """Routed experts [rank * routed / world, (rank + 1) * routed / world) and
    the shared expert of layer ``number`` as two resident layers, reading only
    those experts' byte ranges of the weights file."""
    if routed % world or not 0 <= rank < world:
        raise ValueError("routed experts must divide evenly over the ranks")
    k, weights, index, hidden, intermediate = _layer_files(store, number)
    scales = _layer_scales(index, k, store.device)
    per = routed // world
    lo, hi = rank * per, (rank + 1) * per
    nbytes = hidden * intermediate * k // 8
    local, shared = {}, {}
    for projection in ("gate", "up", "down"):
        buf = torch.empty(per * nbytes, dtype=torch.uint8, device=store.device)
        weights.read_into("trellis." + projection, buf, lo * nbytes, per * nbytes)
        local[projection] = buf
        one = torch.empty(nbytes, dtype=torch.uint8, device=store.device)
        weights.read_into("shared.trellis." + projection, one)
        shared[projection] = one
    local_scales = {p: tuple(v[lo:hi].contiguous() for v in pair) for p, pair in scales.items()}
    shared_scales = {p: tuple(v[-1:].contiguous() for v in pair) for p, pair in scales.items()}
    return (ExpertLayer(local, local_scales, k, hidden, intermediate, number=number),
            ExpertLayer(shared, shared_scales, k, hidden, intermediate, number=number))


def _load_layer(store, number):
    """``ExpertLayer(store, number)`` of experts.py:77-148."""
    k, weights, index, hidden, intermediate = _layer_files(store, number)
    scales = _layer_scales(index, k, store.device)
    packed = None
    if store.resident:
        packed = {}
        for projection in ("gate", "up", "down"):
            routed = weights.tensors["trellis." + projection]["data_offsets"]
            shared = weights.tensors["shared.trellis." + projection]["data_offsets"]
            n_routed, n_shared = routed[1] - routed[0], shared[1] - shared[0]
            buf = torch.empty(n_routed + n_shared, dtype=torch.uint8, device=store.device)
            weights.read_into("trellis." + projection, buf[:n_routed])
            weights.read_into("shared.trellis." + projection, buf[n_routed:])
            packed[projection] = buf
    layer = ExpertLayer(packed, scales, k, hidden, intermediate, number=number, store=store, weights=weights)
    if store.resident:
        store.resident_bytes += sum(t.numel() for t in packed.values())
        store.resident_bytes += sum(s.numel() * s.element_size() for pair in scales.values() for s in pair)
        if store.optimize and k == 4 and (hidden, intermediate) == (6144, 2048):
            from .joined_mxfp4 import JoinedMXFP4

            layer.affine = JoinedMXFP4(layer)
            store.resident_bytes += (
                sum(a.numel() * a.element_size() for values in layer.affine.weights.values()
                    for a in values if a is not None)
                - sum(t.numel() for t in layer.packed.values())
                + layer.affine.unit.numel() * layer.affine.unit.element_size())
            for projection in ("gate", "up"):
                incoming, outgoing = layer.scales[projection]
                store.resident_bytes -= incoming.numel() * incoming.element_size()
                layer.scales[projection] = (None, outgoing)
            layer.packed = None
    return layer


class ExpertLayer:
    def __init__(self, packed, scales, k, hidden, intermediate, shared=None, number=None, store=None,
                 weights=None):
        if k not in (2, 3, 4):
            raise ValueError("EXLR8 trellis width must be 2, 3, or 4")
        self.packed = None if packed is None else {p: packed[p].contiguous() for p in ("gate", "up", "down")}
        self.scales = {p: tuple(s.contiguous() for s in scales[p]) for p in ("gate", "up", "down")}
        self.k, self.hidden, self.intermediate = k, hidden, intermediate
        self.shared = None if shared is None else tuple(t.contiguous() for t in shared)
        self.number = number
        self.store = store
        self.weights = weights
        self.affine = None
        self.experts = self.scales["gate"][0].shape[0]
        self.expert_bytes = hidden * intermediate * k // 8
        self._finish = None

    def _selected(self, ids):
        """Bounded-cache form (experts.py:155-169): the distinct experts of the
        call, their packed bytes and side vectors, ids renumbered to them."""
        selected, inverse = torch.unique(ids.reshape(-1).to(torch.int64), return_inverse=True)
        chosen = selected.tolist()
        if chosen[0] < 0 or chosen[-1] > 256:
            raise ValueError("Expert IDs must be in 0..256")
        remapped = inverse.reshape(ids.shape).to(torch.int32)
        weights = [self.store._get(self, int(expert)) for expert in chosen]
        packed = {projection: torch.cat([w[p] for w in weights])
                  for p, projection in enumerate(("gate", "up", "down"))}
        rows = selected.to(self.scales["down"][0].device)
        scales = {projection: tuple(s[rows] for s in values) for projection, values in self.scales.items()}
        return remapped, packed, scales

    def __call__(self, x, ids):
        if self.affine is not None:
            return self.affine.slots(x, ids)
        if self.store is not None and not self.store.resident:
            remapped, packed, scales = self._selected(ids)
        else:
            remapped, packed, scales = ids, self.packed, self.scales
        if self.store is None or self.store.optimize:
            return fast_expert_mlp(x, remapped, packed, scales, self.k, self.hidden, self.intermediate)
        from .trellis import expert_linear

        outputs = []
        for projection in ("gate", "up"):
            in_scale, out_scale = scales[projection]
            outputs.append(expert_linear(x, remapped, packed[projection], in_scale, out_scale, self.k, self.hidden,
                                         self.intermediate, sharded_side=1))
        hidden = torch.nn.functional.silu(outputs[0]) * outputs[1]  # mlx-lm swiglu in the activation dtype
        in_scale, out_scale = scales["down"]
        return expert_linear(hidden, remapped, packed["down"], in_scale, out_scale, self.k, self.intermediate,
                             self.hidden, sharded_side=2)

    def finish(self, x, ids, scores, residual):
        """residual + routed + shared for nine-slot ids (compiled_expert_mlp_finish)."""
        if self.affine is not None:
            return self.affine.finish(x, ids, scores, residual)
        if self._finish is None:
            self._finish = compiled_expert_mlp_finish(self)
        return self._finish(x, ids, scores, residual)

    @property
    def resident_bytes(self):
        total = sum(t.numel() for t in self.packed.values()) if self.packed is not None else 0
        total += sum(s.numel() * s.element_size() for pair in self.scales.values() for s in pair if s is not None)
        if self.shared is not None:
            total += sum(t.numel() * t.element_size() for t in self.shared)
        return total
