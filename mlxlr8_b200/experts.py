"""Resident expert layer (mirror of the resident branch of ``exlr8/experts.py``).

``ExpertLayer(x, ids)`` returns ``[*ids.shape, hidden]`` per-slot outputs in
the activation dtype (experts.py:150-188).  Weights are resident device
tensors: ``packed[p]`` (uint8 grouped128 bytes of all experts, the shared
expert last when it is a trellis matrix) and ``scales[p] = (in, out)``.  An
optional dense bf16 shared expert (``shared = (gate, up, down)``) is used by
the layer finish instead of trellis matrix 256.
"""

from __future__ import annotations

from .fast_decode import compiled_expert_mlp_finish, fast_expert_mlp


class ExpertLayer:
    def __init__(self, packed, scales, k, hidden, intermediate, shared=None, number=None):
        if k not in (2, 3, 4):
            raise ValueError("EXLR8 trellis width must be 2, 3, or 4")
        self.packed = {p: packed[p].contiguous() for p in ("gate", "up", "down")}
        self.scales = {p: tuple(s.contiguous() for s in scales[p]) for p in ("gate", "up", "down")}
        self.k, self.hidden, self.intermediate = k, hidden, intermediate
        self.shared = None if shared is None else tuple(t.contiguous() for t in shared)
        self.number = number
        self.affine = None
        self.experts = self.scales["gate"][0].shape[0]
        self.expert_bytes = hidden * intermediate * k // 8
        self._finish = None

    def __call__(self, x, ids):
        return fast_expert_mlp(x, ids, self.packed, self.scales, self.k, self.hidden, self.intermediate)

    def finish(self, x, ids, scores, residual):
        """residual + routed + shared for nine-slot ids (compiled_expert_mlp_finish)."""
        if self._finish is None:
            self._finish = compiled_expert_mlp_finish(self)
        return self._finish(x, ids, scores, residual)

    @property
    def resident_bytes(self):
        total = sum(t.numel() for t in self.packed.values())
        total += sum(s.numel() * s.element_size() for pair in self.scales.values() for s in pair)
        if self.shared is not None:
            total += sum(t.numel() * t.element_size() for t in self.shared)
        return total
