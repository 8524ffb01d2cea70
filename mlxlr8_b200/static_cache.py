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
"""

from __future__ import annotations

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
