"""Seeded synthetic MoE layers with the GLM-5 shape (no checkpoints are available).

One seed per tensor family, derived from a layer seed, so that every run and
every rank regenerates identical tensors:

  x, residual   bf16 ~ N(0, 1)                         seed + 1, seed + 2
  gate weight   fp32 ~ N(0, 0.02) [256, hidden]        seed + 3
  bias          fp32 ~ N(0, 0.01) [256]                seed + 4
  packed        uniform bytes (every byte stream is a valid trellis code)
                gate/up/down                           seed + 10, 11, 12
  side scales   fp16 +-|N(1, 0.1)|; the gate/up input scales share one sign
                vector across experts                  seed + 20 .. 25
  shared expert bf16 ~ N(0, 0.02), [out, in]           seed + 30, 31, 32

``make_layer`` builds the tensors directly on the GPU (a full layer is about
4.9 GB); ``host_copy`` brings selected pieces back for CPU checks.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .experts import ExpertLayer


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


@dataclass
class SyntheticLayer:
    experts: ExpertLayer
    gate_weight: torch.Tensor
    bias: torch.Tensor
    seed: int

    def tokens(self, count: int, seed_offset: int = 0, dtype=torch.bfloat16):
        """Seeded activations and residual, bf16 ~ N(0, 1), on the layer's device."""
        device = self.gate_weight.device
        h = self.experts.hidden
        x = torch.randn(count, h, generator=_gen(self.seed + 1 + 1000 * seed_offset, device), device=device)
        r = torch.randn(count, h, generator=_gen(self.seed + 2 + 1000 * seed_offset, device), device=device)
        return x.to(dtype), r.to(dtype)


def make_layer(seed: int = 0, k: int = 4, hidden: int = 6144, intermediate: int = 2048, routed: int = 256,
               shared: str = "bf16", device="cuda", scale_sigma: float = 0.1) -> SyntheticLayer:
    """A routed-MoE layer: ``routed`` trellis experts (+ trellis matrix 256 when
    ``shared == "trellis"``), a bf16 shared expert when ``shared == "bf16"``."""
    device = torch.device(device)
    matrices = routed + (1 if shared == "trellis" else 0)
    nbytes = hidden * intermediate * k // 8
    packed = {}
    for i, p in enumerate(("gate", "up", "down")):
        packed[p] = torch.randint(0, 256, (matrices * nbytes,), dtype=torch.uint8,
                                  generator=_gen(seed + 10 + i, device), device=device)
    signs_in = torch.where(torch.rand(hidden, generator=_gen(seed + 20, device), device=device) < 0.5, -1.0, 1.0)

    def mag(rows, cols, s):
        return (1.0 + scale_sigma * torch.randn(rows, cols, generator=_gen(s, device), device=device)).abs()

    def signs(rows, cols, s):
        return torch.where(torch.rand(rows, cols, generator=_gen(s, device), device=device) < 0.5, -1.0, 1.0)

    scales = {}
    for i, p in enumerate(("gate", "up")):
        inn = (mag(matrices, hidden, seed + 21 + i) * signs_in).to(torch.float16)
        out = (mag(matrices, intermediate, seed + 23 + i) * signs(matrices, intermediate, seed + 40 + i)).to(torch.float16)
        scales[p] = (inn, out)
    down_in = (mag(matrices, intermediate, seed + 25) * signs(matrices, intermediate, seed + 42)).to(torch.float16)
    down_out = (mag(matrices, hidden, seed + 26) * signs(matrices, hidden, seed + 43)).to(torch.float16)
    scales["down"] = (down_in, down_out)
    dense = None
    if shared == "bf16":
        dense = (
            (0.02 * torch.randn(intermediate, hidden, generator=_gen(seed + 30, device), device=device)).to(torch.bfloat16),
            (0.02 * torch.randn(intermediate, hidden, generator=_gen(seed + 31, device), device=device)).to(torch.bfloat16),
            (0.02 * torch.randn(hidden, intermediate, generator=_gen(seed + 32, device), device=device)).to(torch.bfloat16),
        )
    gate_weight = 0.02 * torch.randn(256, hidden, generator=_gen(seed + 3, device), device=device)
    bias = 0.01 * torch.randn(256, generator=_gen(seed + 4, device), device=device)
    layer = ExpertLayer(packed, scales, k, hidden, intermediate, shared=dense)
    return SyntheticLayer(layer, gate_weight.float(), bias.float(), seed)


def host_copy(layer: SyntheticLayer, experts=None):
    """NumPy copies for CPU checks: packed bytes of the listed experts only
    (others zero-filled, so buffer offsets keep their meaning), all scales,
    router and shared weights as float32."""
    import numpy as np

    e = layer.experts
    nbytes = e.expert_bytes
    count = e.experts
    keep = range(count) if experts is None else sorted(set(int(i) for i in experts))
    packed = {}
    for p in ("gate", "up", "down"):
        buf = np.zeros(count * nbytes, dtype=np.uint8)
        src = e.packed[p]
        for i in keep:
            buf[i * nbytes:(i + 1) * nbytes] = src[i * nbytes:(i + 1) * nbytes].cpu().numpy()
        packed[p] = buf
    scales = {p: tuple(s.float().cpu().numpy() for s in e.scales[p]) for p in ("gate", "up", "down")}
    shared = None if e.shared is None else tuple(t.float().cpu().numpy() for t in e.shared)
    return {
        "packed": packed,
        "scales": scales,
        "shared": shared,
        "gate_weight": layer.gate_weight.cpu().numpy(),
        "bias": layer.bias.cpu().numpy(),
    }


# ---------------------------------------------------------------------------
# Joined MXFP4 layer (the prefill configuration).  Codes and E8M0 scales are
# drawn directly from the seed (the reference derives them from trellis
# experts with MLX quantize, which has no published rounding to restate):
#
#   gate_up codes  uniform uint32 (8 E2M1 values each)  seed + 50
#   down codes     uniform uint32                        seed + 51
#   E8M0 scales    uniform in [scale_lo, scale_hi]       seed + 52, 53
#   unit           +-1 fp16                              seed + 54
#   channel scales fp16 +-|N(1, 0.1)|                    seed + 55 .. 58
#   router         as make_layer                         seed + 3, 4
# ---------------------------------------------------------------------------

@dataclass
class SyntheticJoined:
    unit: torch.Tensor
    weights: dict
    scales: dict
    hidden: int
    intermediate: int
    gate_weight: torch.Tensor
    bias: torch.Tensor
    seed: int

    @property
    def experts(self) -> int:
        return self.weights["gate_up"][0].shape[0]

    def tokens(self, count: int, seed_offset: int = 0, dtype=torch.bfloat16):
        device = self.unit.device
        h = self.hidden
        x = torch.randn(count, h, generator=_gen(self.seed + 1 + 1000 * seed_offset, device), device=device)
        r = torch.randn(count, h, generator=_gen(self.seed + 2 + 1000 * seed_offset, device), device=device)
        return x.to(dtype), r.to(dtype)


def make_joined(seed: int = 0, hidden: int = 6144, intermediate: int = 2048, experts: int = 257, device="cuda",
                scale_lo: int = 118, scale_hi: int = 127, scale_sigma: float = 0.1) -> SyntheticJoined:
    """MXFP4 joined experts: ``experts`` matrices (expert 256 = shared when
    experts == 257), gate/up concatenated [E, 2m, h/8] and down [E, h, m/8]."""
    device = torch.device(device)
    h, m = hidden, intermediate

    def codes(shape, s):
        raw = torch.randint(-(2 ** 31), 2 ** 31 - 1, shape, dtype=torch.int64, generator=_gen(s, device),
                            device=device)
        return raw.to(torch.int32)  # the bits of uint32 words

    def e8m0(shape, s):
        return torch.randint(scale_lo, scale_hi + 1, shape, dtype=torch.uint8, generator=_gen(s, device),
                             device=device)

    def mag(rows, cols, s):
        return (1.0 + scale_sigma * torch.randn(rows, cols, generator=_gen(s, device), device=device)).abs()

    def signs(rows, cols, s):
        return torch.where(torch.rand(rows, cols, generator=_gen(s, device), device=device) < 0.5, -1.0, 1.0)

    weights = {
        "gate_up": (codes((experts, 2 * m, h // 8), seed + 50), e8m0((experts, 2 * m, h // 32), seed + 52), None),
        "down": (codes((experts, h, m // 8), seed + 51), e8m0((experts, h, m // 32), seed + 53), None),
    }
    unit = signs(1, h, seed + 54).reshape(h).to(torch.float16)
    scales = {
        "gate": (None, (mag(experts, m, seed + 55) * signs(experts, m, seed + 60)).to(torch.float16)),
        "up": (None, (mag(experts, m, seed + 56) * signs(experts, m, seed + 61)).to(torch.float16)),
        "down": ((mag(experts, m, seed + 57) * signs(experts, m, seed + 62)).to(torch.float16),
                 (mag(experts, h, seed + 58) * signs(experts, h, seed + 63)).to(torch.float16)),
    }
    gate_weight = 0.02 * torch.randn(256, h, generator=_gen(seed + 3, device), device=device)
    bias = 0.01 * torch.randn(256, generator=_gen(seed + 4, device), device=device)
    return SyntheticJoined(unit, weights, scales, h, m, gate_weight.float(), bias.float(), seed)


def joined_host_copy(j: SyntheticJoined, experts=None):
    """NumPy copies of a joined layer for the oracle (codes of the listed
    experts only; the others are zero)."""
    import numpy as np

    count = j.experts
    keep = range(count) if experts is None else sorted(set(int(i) for i in experts))

    def take(t):
        out = np.zeros(tuple(t.shape), dtype=np.uint32 if t.element_size() == 4 else np.uint8)
        for i in keep:
            out[i] = t[i].cpu().numpy().view(out.dtype)
        return out


    return {
        "unit": j.unit.float().cpu().numpy(),
        "gate_up": (take(j.weights["gate_up"][0]), take(j.weights["gate_up"][1])),
        "down": (take(j.weights["down"][0]), take(j.weights["down"][1])),
        "scales": {
            "gate": j.scales["gate"][1].float().cpu().numpy(),
            "up": j.scales["up"][1].float().cpu().numpy(),
            "down": (j.scales["down"][0].float().cpu().numpy(), j.scales["down"][1].float().cpu().numpy()),
        },
        "gate_weight": j.gate_weight.cpu().numpy(),
        "bias": j.bias.cpu().numpy(),
    }


def zipf_bias(seed: int, s: float = 1.1, experts: int = 256, strength: float = 0.2, device="cuda"):
    """Router bias [experts] float32 that skews expert popularity towards a
    Zipf(s) shape (the speculative-verify step): a seeded
    random ranking of the experts and bias = -strength * s * log(rank + 1), so
    the rank-k expert's chance of a top-8 slot falls off roughly as k^-s on
    top of the gate's own spread."""
    device = torch.device(device)
    order = torch.randperm(experts, generator=_gen(seed, device), device=device)
    rank = torch.empty(experts, dtype=torch.float32, device=device)
    rank[order] = torch.arange(experts, dtype=torch.float32, device=device)
    return (-strength * s * torch.log(rank + 1.0)).float()
