"""Static hot-expert cache: fixed experts expanded to their exact E4M3 bytes
(``exlr8/static_cache.py``).

``expand_static_trellis`` turns a packed trellis buffer into one E4M3 byte
per weight in the stored tile order (``static_cache.py:61-75``): tile ``t``
becomes bytes ``[256 t, 256 t + 256)``, byte ``8 * lane + j`` the exact code
of the lane's codeword ``j``.  The values are the trellis weights themselves,
so a cached expert gives the same products as its codes.

``StaticExpertCache(layer, expert_ids)`` (``static_cache.py:91-134``) owns
one device buffer per projection holding the listed experts' bytes in list
order, and the device map ``expert_to_slot`` (int32 bits of the reference's
uint32 map, 0xFFFFFFFF for an uncached expert).  The C structs of the layer
and the cache are prepared once, so a call is one ``exlr8_expert_mlp_cached``
launch chain: units of cached experts stream their bytes (twice the bytes of
K4 codes, one conversion per two weights instead of the trellis codec) in the
codec path's MMA order, so the outputs are bit-equal to the uncached decode,
as the reference's test of the cache requires (``test_static_cache.py``).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .trellis import _ids, _words, check_format


def _expand_into(raw, k, in_features, out_features, sharded_side, out):
    _lib.check(_lib.lib().exlr8_expand_static_trellis(raw.data_ptr(), raw.numel(), k, in_features, out_features,
                                                      sharded_side, out.data_ptr(),
                                                      _lib.stream_handle(raw.device)))


def expand_static_trellis(packed, k, in_features, out_features, sharded_side=1):
    """Flat exact E4M3 bytes (uint8 CUDA tensor, ``in * out`` per matrix) of
    every matrix in ``packed``, tile order kept (static_cache.py:61-75)."""
    _lib.require_cuda(packed)
    raw = _words(packed)
    matrices = check_format(raw, k, in_features, out_features, sharded_side)
    out = torch.empty(matrices * in_features * out_features, dtype=torch.uint8, device=raw.device)
    _expand_into(raw, k, in_features, out_features, sharded_side, out)
    return out


def _hot_slots(expert_ids, experts):
    """Validated hot expert ids as a tuple, in slot order.  Accepts a 1-D
    sequence or tensor of integers; the reference's ValueError texts
    (static_cache.py:78-84)."""
    values = torch.as_tensor(expert_ids)
    if values.dim() != 1 or values.numel() == 0 or values.dtype.is_floating_point or values.dtype.is_complex \
            or values.dtype == torch.bool:
        raise ValueError("hot expert IDs must be a nonempty integer vector")
    ids = tuple(int(v) for v in values.tolist())
    if len(set(ids)) != len(ids) or min(ids) < 0 or max(ids) >= experts:
        raise ValueError("hot expert IDs must be unique and within the source layer")
    return ids


def _slot_map(ids, experts, device):
    """int32 [experts] device map: the slot of each cached expert, -1 (the bits
    of uint32 0xFFFFFFFF) elsewhere."""
    table = torch.full((experts,), -1, dtype=torch.int32, device=device)
    table[torch.tensor(ids, dtype=torch.long, device=device)] = torch.arange(len(ids), dtype=torch.int32,
                                                                             device=device)
    return table


def static_cache_bytes(hidden, intermediate, hot_experts, experts=257):
    """Device bytes of a cache of ``hot_experts`` experts: one E4M3 byte per
    weight of the three matrices, plus the 4-byte map entry of every expert."""
    return 3 * hidden * intermediate * hot_experts + 4 * experts


class StaticExpertCache:
    """Fixed experts of a resident layer as exact E4M3 bytes (static_cache.py:91-134).

    ``fp8[p]`` is the uint8 buffer of projection ``p``: ``hidden *
    intermediate`` bytes per cache slot, slots in the order of
    ``expert_ids``, each in the source tile order.  ``expert_to_slot`` is the
    device map.
    """

    def __init__(self, layer, expert_ids=(256,)):
        from .fast_decode import trellis_experts

        store = getattr(layer, "store", None)
        if layer.packed is None or (store is not None and not store.resident):
            raise ValueError("static decode requires resident packed weights")
        self.layer = layer
        experts = layer.scales["down"][1].shape[0]
        self.expert_ids = _hot_slots(expert_ids, experts)
        device = layer.packed["gate"].device
        self.expert_to_slot = _slot_map(self.expert_ids, experts, device)
        h, m, k = layer.hidden, layer.intermediate, layer.k
        per_slot = h * m
        code_bytes = per_slot * k // 8
        self.fp8 = {}
        for projection in ("gate", "up", "down"):
            a, b, side = (m, h, 2) if projection == "down" else (h, m, 1)
            source = _words(layer.packed[projection]).reshape(-1)
            bytes_out = torch.empty(len(self.expert_ids) * per_slot, dtype=torch.uint8, device=device)
            for slot, e in enumerate(self.expert_ids):
                _expand_into(source[e * code_bytes:(e + 1) * code_bytes], k, a, b, side,
                             bytes_out[slot * per_slot:(slot + 1) * per_slot])
            self.fp8[projection] = bytes_out
        self._experts, self._count = trellis_experts(layer.packed, layer.scales, k, h, m)
        self._cache = _lib.StaticCache()
        for i, projection in enumerate(("gate", "up", "down")):
            self._cache.fp8[i] = self.fp8[projection].data_ptr()
        self._cache.expert_to_slot = self.expert_to_slot.data_ptr()
        self._cache.slots = len(self.expert_ids)
        self._workspace = None

    def __call__(self, x, ids):
        """Per-slot expert MLP outputs ``[*ids.shape, hidden]``, bit-equal to
        the layer's own decode (the cached bytes are its weights)."""
        layer = self.layer
        device = _lib.require_cuda(x, ids)
        if x.shape[-1] != layer.hidden:
            raise ValueError("activation width does not match in_features")
        if x.shape[:-1] == ids.shape:
            per_slot = 1
        elif x.shape[:-1] == ids.shape[:-1]:
            per_slot = 0
        else:
            raise ValueError("activation rows do not match the expert indices")
        indices = _ids(ids)
        slots = ids.shape[-1]
        tokens = indices.numel() // slots
        xs = x.contiguous()
        out = torch.empty(tuple(ids.shape) + (layer.hidden,), dtype=x.dtype, device=device)
        lib = _lib.lib()
        need = lib.exlr8_expert_mlp_workspace(tokens, slots, layer.hidden, layer.intermediate, self._count)
        if self._workspace is None or self._workspace.numel() < need or self._workspace.device != device:
            self._workspace = _lib.workspace(need, device)
        _lib.check(lib.exlr8_expert_mlp_cached(xs.data_ptr(), _lib.act_code(xs), per_slot, indices.data_ptr(),
                                               tokens, slots, self._experts, ctypes.byref(self._cache),
                                               out.data_ptr(), self._workspace.data_ptr(),
                                               self._workspace.numel(), _lib.stream_handle(device)))
        return out

    def stats(self):
        per_slot = self.layer.hidden * self.layer.intermediate
        return {"expert_ids": list(self.expert_ids),
                "weight_bytes": 3 * per_slot * len(self.expert_ids),
                "map_bytes": 4 * self.expert_to_slot.numel()}
