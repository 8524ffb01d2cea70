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
from pathlib import Path

import torch

from .fast_decode import compiled_expert_mlp_finish, fast_expert_mlp

_PROJECTIONS = ("gate", "up", "down")


class _Up1Manifest:
    """``manifests/exlr8-manifest-up1.json``: per decoder layer the trellis
    width of every routed and shared matrix."""

    def __init__(self, root: Path):
        data = json.loads((root / "manifests" / "exlr8-manifest-up1.json").read_text())
        if data.get("name") != "up1":
            raise ValueError("This loader requires the up1 manifest")
        self.data = data

    def __getitem__(self, key):
        return self.data[key]

    @staticmethod
    def _widths(node):
        if isinstance(node, dict):
            for value in node.values():
                yield from _Up1Manifest._widths(value)
        elif isinstance(node, (list, tuple)):
            for value in node:
                yield from _Up1Manifest._widths(value)
        else:
            yield int(node)

    def width(self, number: int) -> int:
        """The layer's single trellis width: K3 for the MTP layer 78, K4 for the
        others; any other width in the layer's plan is refused."""
        want = 3 if number == 78 else 4
        plan = self.data["layers"][str(number)]
        found = set(self._widths({name: plan[name] for name in (*_PROJECTIONS, "shared")}))
        if found != {want}:
            raise ValueError(f"Layer {number} is not uniform K{want}")
        return want


class _DeviceLRU:
    """Byte-bounded least-recently-used map of per-expert device tensors
    (the bounded expert cache of the non-resident store).  An entry larger
    than the whole budget is returned but never kept."""

    def __init__(self, limit: int):
        self.limit = limit
        self.entries = {}  # insertion order = recency order, oldest first
        self.bytes = 0
        self.hits = 0
        self.misses = 0

    def fetch(self, key, load, nbytes: int):
        entry = self.entries.pop(key, None)
        if entry is not None:
            self.hits += 1
            self.entries[key] = entry  # now the most recent
            return entry
        self.misses += 1
        entry = load()
        if nbytes <= self.limit:
            while self.entries and self.bytes + nbytes > self.limit:
                oldest = next(iter(self.entries))
                self.bytes -= sum(t.numel() * t.element_size() for t in self.entries.pop(oldest))
            self.entries[key] = entry
            self.bytes += nbytes
        return entry


class ExpertStore:
    """Experts of an EXLR8 checkpoint on the GPU (experts.py:16-73): resident
    layers, or per-expert reads through a byte-bounded cache."""

    def __init__(self, path, cache_gib=32, resident=False, optimize=True, device=None):
        self.path = Path(path)
        self.resident = resident
        self.optimize = optimize
        self.manifest = _Up1Manifest(self.path)
        limit = int(cache_gib * 1024**3)
        if limit < 0:
            raise ValueError("cache_gib must be nonnegative")
        self._lru = _DeviceLRU(limit)
        self._device = None if device is None else torch.device(device)
        self.resident_bytes = 0
        self._layers = {}

    # The cache's state under the reference's attribute names.
    @property
    def limit(self):
        return self._lru.limit

    @property
    def cache(self):
        return self._lru.entries

    @property
    def cache_bytes(self):
        return self._lru.bytes

    @property
    def hits(self):
        return self._lru.hits

    @property
    def misses(self):
        return self._lru.misses

    @property
    def device(self):
        if self._device is None:
            self._device = torch.device("cuda", torch.cuda.current_device())
        return self._device

    def layer(self, number):
        layer = self._layers.get(number)
        if layer is None:
            layer = self._layers[number] = _load_layer(self, number)
        return layer

    def _get(self, layer, expert):
        """(gate, up, down) packed bytes of one expert (256 = the shared
        expert, stored in its own tensors) read into device memory."""
        name = "shared.trellis." if expert == 256 else "trellis."
        offset = 0 if expert == 256 else expert * layer.expert_bytes

        def read():
            return tuple(layer.weights.load_slice(name + projection, offset, layer.expert_bytes, self.device)
                         for projection in _PROJECTIONS)

        return self._lru.fetch((layer.number, expert), read, 3 * layer.expert_bytes)

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
        return {"cache_bytes": self.cache_bytes, "cache_limit_bytes": self.limit,
                "resident_bytes": self.resident_bytes, "hits": self.hits, "misses": self.misses}


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


# Index-file tensor names per projection: (block scale over the hidden side,
# channel scale over the intermediate side, sign vector of the hidden side).
_SIDE_NAMES = {"gate": ("su_block", "svh", "signs.in"), "up": ("su_block", "svh", "signs.in"),
               "down": ("sv_block", "suh", "signs.out")}


def _layer_scales(index, k, device):
    """Signed side vectors of the routed experts followed by the shared expert
    (experts.py:97-115).  The hidden side of each matrix is its per-128-channel
    block scale spread over the block's channels times the layer's sign
    vector; the intermediate side is the stored channel scale.  Built on the
    device in float16, the stored type; returned as (in, out) per projection
    (gate/up: hidden in, down: hidden out)."""
    out = {}
    for projection in _PROJECTIONS:
        block_name, channel_name, sign_name = _SIDE_NAMES[projection]
        signs = torch.from_numpy(index.raw(sign_name)).to(device=device, dtype=torch.float16)
        parts = [torch.from_numpy(index.raw(f"{prefix}k{k}.{projection}.{block_name}")).to(device)
                 for prefix in ("", "shared.")]
        block = torch.cat(parts).to(torch.float16)
        hidden_side = block.repeat_interleave(128, dim=1) * signs
        channel = torch.cat([torch.from_numpy(index.raw(f"{prefix}k{k}.{projection}.{channel_name}")).to(device)
                             for prefix in ("", "shared.")]).to(torch.float16)
        out[projection] = (channel, hidden_side) if projection == "down" else (hidden_side, channel)
    return out


def _layer_files(store, number):
    """(k, weights file, index file, hidden, intermediate) of layer ``number``
    once the manifest's width check passed (experts.py:80-94)."""
    from .weights import SafeTensorFile

    k = store.manifest.width(number)
    stem = store.path / "experts" / f"exlr8-layer-{number:03d}"
    weights = SafeTensorFile(Path(f"{stem}.k{k}.safetensors"))
    index = SafeTensorFile(Path(f"{stem}.index.safetensors"))
    hidden = int(index.header["signs.in"]["shape"][0])
    intermediate = int(index.header[f"k{k}.gate.svh"]["shape"][-1])
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
        self._staging = None

    def _stage(self, ids):
        """Non-resident layer: the call's distinct experts (sorted) are read
        through the store's cache and copied into this layer's staging
        buffers (grown on demand, reused across calls); returns the ids
        renumbered to staging slots, the staged bytes and the matching
        side-vector rows (the bounded-cache form of experts.py:155-169)."""
        distinct, slots = torch.unique(ids.reshape(-1).to(torch.int64), return_inverse=True)
        chosen = distinct.tolist()
        if chosen[0] < 0 or chosen[-1] > 256:
            raise ValueError("Expert IDs must be in 0..256")
        count, size = len(chosen), self.expert_bytes
        device = self.store.device
        if self._staging is None or self._staging["gate"].numel() < count * size:
            self._staging = {name: torch.empty(count * size, dtype=torch.uint8, device=device)
                             for name in ("gate", "up", "down")}
        for slot, expert in enumerate(chosen):
            for name, part in zip(("gate", "up", "down"), self.store._get(self, int(expert))):
                self._staging[name][slot * size:(slot + 1) * size].copy_(part, non_blocking=True)
        packed = {name: buf[:count * size] for name, buf in self._staging.items()}
        rows = distinct.to(self.scales["down"][0].device)
        scales = {name: tuple(v.index_select(0, rows) for v in pair) for name, pair in self.scales.items()}
        return slots.reshape(ids.shape).to(torch.int32), packed, scales

    def __call__(self, x, ids):
        """Per-slot outputs ``[*ids.shape, hidden]`` in x's dtype (experts.py:150-188)."""
        if self.affine is not None:
            return self.affine.slots(x, ids)
        staged = self.store is not None and not self.store.resident
        which, packed, scales = self._stage(ids) if staged else (ids, self.packed, self.scales)
        if self.store is None or self.store.optimize:
            return fast_expert_mlp(x, which, packed, scales, self.k, self.hidden, self.intermediate)
        return reference_operator_mlp(x, which, packed, scales, self.k, self.hidden, self.intermediate)

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


def reference_operator_mlp(x, ids, packed, scales, k, hidden, intermediate):
    """The ``--no-optimize`` expert MLP (experts.py:176-188): gate and up
    through the reference operator ``expert_linear`` (side 1), the mlx-lm
    SwiGLU ``silu(gate) * up`` in the activation dtype, down through
    ``expert_linear`` (side 2).  Every product is the CUDA operator."""
    from .trellis import expert_linear

    def project(v, name, n_in, n_out, side):
        in_scale, out_scale = scales[name]
        return expert_linear(v, ids, packed[name], in_scale, out_scale, k, n_in, n_out, sharded_side=side)

    gate = project(x, "gate", hidden, intermediate, 1)
    up = project(x, "up", hidden, intermediate, 1)
    return project(torch.nn.functional.silu(gate) * up, "down", intermediate, hidden, 2)
