"""Static hot-expert cache: fixed experts expanded to their exact E4M3 bytes
(``exlr8/static_cache.py``).

``expand_static_trellis`` turns a packed trellis buffer into one E4M3 byte
per weight in the stored tile order (``static_cache.py:61-75``): tile ``t``
becomes bytes ``[256 t, 256 t + 256)``, byte ``8 * lane + j`` the exact code
of the lane's codeword ``j``.  The values are the trellis weights themselves,
so a cached expert gives the same products as its codes.

``StaticExpertCache(layer, expert_ids)`` expands the listed experts of a
resident layer once (``static_cache.py:91-134``) and keeps the GPU map
``expert_to_slot`` (0xFFFFFFFF for an uncached expert).  Its decode is the
layer's streaming expert MLP with the cache attached: units of cached experts
stream their bytes (twice the bytes of K4 codes, one conversion per two
weights instead of the trellis codec) in the codec path's MMA order, so the
outputs are bit-equal to the uncached decode, as the reference's test of the
cache requires (``test_static_cache.py``).

``fixed_hot_lists`` picks the cached experts from a routing trace
(``tools/static_cache_routes.py``): the most frequent routed experts of a
training split, scored on a held-out split; ``python -m
mlxlr8_b200.static_cache TRACE --output OUT`` writes the lists.
"""

from __future__ import annotations

import argparse
import json
from collections import Counter
from pathlib import Path

import numpy as np
import torch

from . import _lib
from .trellis import _words, check_format


def expand_static_trellis(packed, k, in_features, out_features, sharded_side=1):
    """Flat exact E4M3 bytes (uint8 CUDA tensor, ``in * out`` per matrix) of
    every matrix in ``packed``, tile order kept (static_cache.py:61-75)."""
    device = _lib.require_cuda(packed)
    raw = _words(packed)
    matrices = check_format(raw, k, in_features, out_features, sharded_side)
    out = torch.empty(matrices * in_features * out_features, dtype=torch.uint8, device=device)
    _lib.check(_lib.lib().exlr8_expand_static_trellis(raw.data_ptr(), raw.numel(), k, in_features, out_features,
                                                      sharded_side, out.data_ptr(), _lib.stream_handle(device)))
    return out


def _expert_map(expert_ids, experts):
    """(ids as a tuple, uint32 [experts] slot map with 0xFFFFFFFF for a miss),
    with the reference's checks (static_cache.py:78-84)."""
    ids = np.asarray(expert_ids)
    if ids.ndim != 1 or ids.size == 0 or ids.dtype.kind not in "iu":
        raise ValueError("hot expert IDs must be a nonempty integer vector")
    if np.any(ids < 0) or np.any(ids >= experts) or np.unique(ids).size != ids.size:
        raise ValueError("hot expert IDs must be unique and within the source layer")
    mapping = np.full(experts, 0xFFFFFFFF, np.uint32)
    mapping[ids] = np.arange(ids.size, dtype=np.uint32)
    return tuple(int(i) for i in ids), mapping


def static_cache_bytes(hidden, intermediate, hot_experts, experts=257):
    """Device bytes of a cache of ``hot_experts`` experts: three E4M3 matrices
    each plus the uint32 map (static_cache.py:87-88)."""
    return 3 * hidden * intermediate * hot_experts + 4 * experts


class StaticExpertCache:
    """Expand fixed experts once; decode with the source scales and the GPU
    map (static_cache.py:91-134).

    ``fp8[p]`` is the flat uint8 buffer of projection ``p`` with
    ``hidden * intermediate`` bytes per cache slot, in the source tile order;
    ``expert_to_slot`` is the uint32 map (an int32 tensor with the same bits
    on the device).
    """

    def __init__(self, layer, expert_ids=(256,)):
        store = getattr(layer, "store", None)
        if layer.packed is None or (store is not None and not store.resident):
            raise ValueError("static decode requires resident packed weights")
        self.layer = layer
        count = layer.scales["down"][1].shape[0]
        self.expert_ids, mapping = _expert_map(expert_ids, count)
        device = layer.packed["gate"].device
        self.expert_to_slot = torch.from_numpy(mapping.view(np.int32)).to(device)
        size = layer.hidden * layer.intermediate * layer.k // 8
        self.fp8 = {}
        for projection in ("gate", "up", "down"):
            a, b, side = ((layer.intermediate, layer.hidden, 2) if projection == "down"
                          else (layer.hidden, layer.intermediate, 1))
            source = layer.packed[projection].reshape(-1)
            self.fp8[projection] = torch.cat([expand_static_trellis(source[e * size:(e + 1) * size], layer.k, a, b,
                                                                    side) for e in self.expert_ids])

    def __call__(self, x, ids):
        """Per-slot expert MLP outputs ``[*ids.shape, hidden]``, equal bit for
        bit to the layer's own decode (the cached bytes are its weights)."""
        from .fast_decode import fast_expert_mlp

        layer = self.layer
        return fast_expert_mlp(x, ids, layer.packed, layer.scales, layer.k, layer.hidden, layer.intermediate,
                               fp8=self.fp8, expert_to_slot=self.expert_to_slot)

    def stats(self):
        return {"expert_ids": list(self.expert_ids),
                "weight_bytes": sum(t.numel() for t in self.fp8.values()),
                "map_bytes": self.expert_to_slot.numel() * 4}


def _hit_counts(rows, hot, shared):
    """Selections served by the cache in ``rows`` (lists of expert ids)."""
    cached = set(hot)
    hits = routed_hits = full_rows = 0
    for row in rows:
        inside = [e in cached for e in row]
        hits += sum(inside)
        routed_hits += sum(1 for e, hit in zip(row, inside) if hit and e != shared)
        full_rows += all(inside)
    return {"hits": hits, "routed_hits": routed_hits, "all_selected_hit_tokens": full_rows}


def fixed_hot_lists(trace, split=256, shared=256, capacities=(1, 9, 12, 18)):
    """Hot-expert lists per layer and capacity from a routing trace
    (tools/static_cache_routes.py:16-52).

    ``trace["layers"][n]["routes"]`` holds ``2 * split`` rows of selected
    expert ids.  The first ``split`` rows rank the routed experts by
    frequency (ties: lowest id); a capacity-``c`` list is the shared expert
    plus the ``c - 1`` highest ranked.  Each list is scored on both splits
    (hits, routed hits, rows served entirely from the cache), and the totals
    over layers carry the hit rates.
    """
    sections = ("train", "heldout")
    fields = ("tokens", "selections", "routed_selections", "hits", "routed_hits", "all_selected_hit_tokens")
    totals = {name: {str(c): dict.fromkeys(fields, 0) for c in capacities} for name in sections}
    layers = {}
    for number, source in trace["layers"].items():
        routes = source["routes"]
        if len(routes) != 2 * split:
            raise ValueError(f"layer {number} needs {2 * split} routes, got {len(routes)}")
        parts = {"train": routes[:split], "heldout": routes[split:]}
        frequency = Counter(e for row in parts["train"] for e in row if e != shared)
        ranked = sorted(frequency, key=lambda e: (-frequency[e], e))
        layers[number] = {}
        for capacity in capacities:
            hot = [shared] + ranked[:capacity - 1]
            entry = {"expert_ids": hot}
            for name in sections:
                rows = parts[name]
                counts = _hit_counts(rows, hot, shared)
                entry[name] = counts
                total = totals[name][str(capacity)]
                total["tokens"] += len(rows)
                total["selections"] += sum(len(row) for row in rows)
                total["routed_selections"] += sum(1 for row in rows for e in row if e != shared)
                for key, value in counts.items():
                    total[key] += value
            layers[number][str(capacity)] = entry
    for section in totals.values():
        for total in section.values():
            total["hit_rate"] = total["hits"] / total["selections"]
            total["routed_hit_rate"] = total["routed_hits"] / total["routed_selections"]
            total["all_selected_hit_token_rate"] = total["all_selected_hit_tokens"] / total["tokens"]
    return {"train_tokens_per_layer": split, "heldout_tokens_per_layer": split, "shared_expert": shared,
            "tie_break": "lowest expert ID", "totals": totals, "layers": layers}


def main(argv=None):
    parser = argparse.ArgumentParser(description="Choose fixed hot experts from a routing trace.")
    parser.add_argument("trace")
    parser.add_argument("--output", required=True)
    args = parser.parse_args(argv)
    result = fixed_hot_lists(json.loads(Path(args.trace).read_text()))
    result["source"] = args.trace
    Path(args.output).write_text(json.dumps(result, separators=(",", ":")) + "\n")
    print(json.dumps(result["totals"], indent=2))


if __name__ == "__main__":
    main()
