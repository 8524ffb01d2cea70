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


@dataclass
class SyntheticShard:
    """One rank's part of a synthetic layer for expert parallelism: the
    routed experts [rank * E / world, (rank + 1) * E / world) and the
    replicated router and bf16 shared expert."""
    experts: ExpertLayer
    gate_weight: torch.Tensor
    bias: torch.Tensor
    shared: tuple
    rank: int
    world: int
    seed: int


def make_shard(seed: int, rank: int = 0, world: int = 1, k: int = 4, hidden: int = 6144, intermediate: int = 2048,
               routed: int = 256, device="cuda", scale_sigma: float = 0.1, placement=None) -> SyntheticShard:
    """Expert-parallel shard of a synthetic layer.  Every routed expert's
    codes come from their own seed (layer seed, expert, projection), so the
    shards of all ranks together are the same layer whatever ``world`` is;
    side scales, router and shared expert are drawn whole and sliced.  With
    ``placement`` (``ep.seeded_placement``) the shard holds the experts
    placed at this rank's positions, in position order."""
    from .ep import _owned

    if routed % world or not 0 <= rank < world:
        raise ValueError("routed experts must divide evenly over the ranks")
    device = torch.device(device)
    per = routed // world
    owned = _owned(rank, world, routed, placement)
    nbytes = hidden * intermediate * k // 8
    packed = {}
    for i, p in enumerate(("gate", "up", "down")):
        buf = torch.empty(per * nbytes, dtype=torch.uint8, device=device)
        for j in range(per):
            e = owned[j]
            buf[j * nbytes:(j + 1) * nbytes] = torch.randint(
                0, 256, (nbytes,), dtype=torch.uint8, generator=_gen(seed * 7919 + e * 3 + i, device), device=device)
        packed[p] = buf
    signs_in = torch.where(torch.rand(hidden, generator=_gen(seed + 20, device), device=device) < 0.5, -1.0, 1.0)

    def mag(rows, cols, sd):
        return (1.0 + scale_sigma * torch.randn(rows, cols, generator=_gen(sd, device), device=device)).abs()

    def signs(rows, cols, sd):
        return torch.where(torch.rand(rows, cols, generator=_gen(sd, device), device=device) < 0.5, -1.0, 1.0)

    owned_idx = torch.tensor(owned, dtype=torch.int64, device=device)

    def rows_of(t):
        return t.index_select(0, owned_idx).contiguous()

    scales = {}
    for i, p in enumerate(("gate", "up")):
        inn = (mag(routed, hidden, seed + 21 + i) * signs_in).to(torch.float16)
        out = (mag(routed, intermediate, seed + 23 + i) * signs(routed, intermediate, seed + 40 + i)).to(torch.float16)
        scales[p] = (rows_of(inn), rows_of(out))
    down_in = (mag(routed, intermediate, seed + 25) * signs(routed, intermediate, seed + 42)).to(torch.float16)
    down_out = (mag(routed, hidden, seed + 26) * signs(routed, hidden, seed + 43)).to(torch.float16)
    scales["down"] = (rows_of(down_in), rows_of(down_out))
    shared = tuple((0.02 * torch.randn(*shape, generator=_gen(seed + 30 + i, device), device=device)).to(torch.bfloat16)
                   for i, shape in enumerate(((intermediate, hidden), (intermediate, hidden), (hidden, intermediate))))
    gate_weight = (0.02 * torch.randn(256, hidden, generator=_gen(seed + 3, device), device=device)).float()
    bias = (0.01 * torch.randn(256, generator=_gen(seed + 4, device), device=device)).float()
    layer = ExpertLayer(packed, scales, k, hidden, intermediate, shared=shared if world == 1 else None)
    return SyntheticShard(layer, gate_weight, bias, shared, rank, world, seed)


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


# ---------------------------------------------------------------------------
# Skewed expert popularity for the speculative-verify workload (128 tokens,
# Zipf(1.1) expert selection).  The router bias of expert e is
#   bias_e = -gamma * s * ln(rank_e + 1)
# over a seeded random ranking of the experts.  gamma is calibrated once by
# bisection (calibrate_zipf_gamma) so that the top-8 selection frequencies of
# 10^5 seeded tokens fit Zipf(s): the least-squares slope of log(frequency)
# against log(rank + 1) over the experts equals -s.  The tokens' logits are
# drawn from the distribution the synthetic layers produce (x ~ N(0, I),
# gate weight ~ N(0, 0.02) of seed ZIPF_SEED: logits ~ N(0, W W^T)).
# ---------------------------------------------------------------------------

ZIPF_S = 1.1
ZIPF_SEED = 4242
ZIPF_TOKENS = 100_000
ZIPF_GAMMA = 0.038376  # calibrate_zipf_gamma() with the defaults above


def _zipf_logits(seed: int, tokens: int, hidden: int = 6144, experts: int = 256):
    import numpy as np

    rng = np.random.default_rng(seed)
    w = 0.02 * rng.standard_normal((experts, hidden))
    chol = np.linalg.cholesky(w @ w.T)
    return (rng.standard_normal((tokens, experts)) @ chol.T).astype(np.float32)


def zipf_selection_slope(logits, bias, rank, top_k: int = 8):
    """(slope, frequencies): per-expert top-k selection frequency of
    ``sigmoid(logits) + bias`` and its least-squares log-log slope against
    ``rank + 1`` (experts never selected left out)."""
    import numpy as np

    choice = 1.0 / (1.0 + np.exp(-np.asarray(logits, np.float64))) + np.asarray(bias, np.float64)[None, :]
    chosen = np.argpartition(-choice, top_k - 1, axis=1)[:, :top_k]
    freq = np.bincount(chosen.ravel(), minlength=choice.shape[1]) / choice.shape[0]
    keep = freq > 0
    slope = np.polyfit(np.log(np.asarray(rank, np.float64)[keep] + 1.0), np.log(freq[keep]), 1)[0]
    return float(slope), freq


def calibrate_zipf_gamma(seed: int = ZIPF_SEED, tokens: int = ZIPF_TOKENS, s: float = ZIPF_S,
                         lo: float = 0.0, hi: float = 0.1, tol: float = 1e-5) -> float:
    """Bisection on gamma in [lo, hi] (the slope falls monotonically there)
    until the selection slope of ``tokens`` seeded tokens equals -s."""
    import numpy as np

    logits = _zipf_logits(seed, tokens)
    rank = np.random.default_rng(seed + 1).permutation(logits.shape[1]).astype(np.float64)
    while hi - lo > tol:
        mid = 0.5 * (lo + hi)
        slope, _ = zipf_selection_slope(logits, -mid * s * np.log(rank + 1.0), rank)
        if slope > -s:
            lo = mid
        else:
            hi = mid
    return 0.5 * (lo + hi)


def zipf_ranks(seed: int, experts: int = 256, device="cuda"):
    """Seeded popularity rank of every expert (0 = most popular), float32."""
    device = torch.device(device)
    order = torch.randperm(experts, generator=_gen(seed, device), device=device)
    rank = torch.empty(experts, dtype=torch.float32, device=device)
    rank[order] = torch.arange(experts, dtype=torch.float32, device=device)
    return rank


def zipf_bias(seed: int, s: float = ZIPF_S, experts: int = 256, gamma: float = ZIPF_GAMMA, device="cuda"):
    """Router bias [experts] float32 giving Zipf(s) expert selection
    (the calibrated gamma above) over the ranking ``zipf_ranks(seed)``."""
    rank = zipf_ranks(seed, experts, device)
    return (-gamma * s * torch.log(rank + 1.0)).float()


# ---------------------------------------------------------------------------
# EXLR8 checkpoint directories on disk (the loader's input format,
# experts.py:16-33,77-124, dense.py:174-191, README.md:60-74).  Contents are
# seeded from numpy's default_rng(seed + layer):
#
#   packed codes   uniform bytes, routed experts then the shared expert
#   signs.in/out   +-1 int8 [hidden]
#   block scales   fp16 U(0.5, 1.5), one per 128 hidden channels, random sign
#   channel scales fp16 +-U(0.5, 1.5)
#   router         bf16 N(0, 0.02) [256, hidden]; bias float32 N(0, 0.01)
# ---------------------------------------------------------------------------

_SAFETENSORS_DTYPES = {"uint8": "U8", "int8": "I8", "int32": "I32", "float16": "F16", "float32": "F32"}


def _write_safetensors(path, entries, chunk=64 << 20):
    """Write a safetensors file from (name, dtype, shape, source) entries
    without holding big tensors in memory: ``source`` is a numpy array, or a
    callable ``source(n) -> bytes`` streamed in chunks for uint8 tensors.
    bf16 tensors are passed as uint16 bit patterns with dtype ``"BF16"``."""
    import json
    import struct

    import numpy as np

    header, offset = {}, 0
    for name, dtype, shape, _ in entries:
        itemsize = {"U8": 1, "I8": 1, "F16": 2, "BF16": 2, "I32": 4, "F32": 4}[dtype]
        size = int(np.prod(shape, dtype=np.int64)) * itemsize
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [offset, offset + size]}
        offset += size
    blob = json.dumps(header, separators=(",", ":")).encode()
    blob += b" " * (-len(blob) % 8)
    with open(path, "wb") as out:
        out.write(struct.pack("<Q", len(blob)))
        out.write(blob)
        for name, dtype, shape, source in entries:
            begin, end = header[name]["data_offsets"]
            if callable(source):
                left = end - begin
                while left:
                    n = min(chunk, left)
                    out.write(source(n))
                    left -= n
            else:
                out.write(np.ascontiguousarray(source).tobytes())


def write_checkpoint(path, layers=(3,), hidden: int = 6144, intermediate: int = 2048, routed: int = 256,
                     seed: int = 0, router_format: int = 6):
    """Write an EXLR8 checkpoint directory holding the expert and router
    files of ``layers`` (K3 for layer 78, K4 otherwise, as the up1 manifest
    selects) and return its path.  A full-size layer is 4.85 GB of codes."""
    import json
    from pathlib import Path

    import numpy as np

    root = Path(path)
    for sub in ("manifests", "experts", "dense"):
        (root / sub).mkdir(parents=True, exist_ok=True)
    plans = {}
    h, m = hidden, intermediate
    for number in layers:
        k = 3 if number == 78 else 4
        plans[str(number)] = {"gate": [[k]] * routed, "up": [[k]] * routed, "down": [k] * routed,
                              "shared": {"gate": [k], "up": [k], "down": k}}
        rng = np.random.default_rng(seed + number)
        nbytes = h * m * k // 8
        entries = []
        for projection in ("gate", "up", "down"):
            entries.append((f"trellis.{projection}", "U8", (routed * nbytes,), rng.bytes))
            entries.append((f"shared.trellis.{projection}", "U8", (nbytes,), rng.bytes))
        _write_safetensors(root / "experts" / f"exlr8-layer-{number:03d}.k{k}.safetensors", entries)

        def signed(shape):
            return (rng.uniform(0.5, 1.5, shape) * rng.choice([-1.0, 1.0], shape)).astype(np.float16)

        index = [("signs.in", "I8", (h,), rng.choice([-1, 1], h).astype(np.int8)),
                 ("signs.out", "I8", (h,), rng.choice([-1, 1], h).astype(np.int8))]
        for projection in ("gate", "up", "down"):
            block_name = "sv_block" if projection == "down" else "su_block"
            channel_name = "suh" if projection == "down" else "svh"
            other = m
            for prefix, count in ((f"k{k}", routed), (f"shared.k{k}", 1)):
                index.append((f"{prefix}.{projection}.{block_name}", "F16", (count, h // 128),
                              signed((count, h // 128))))
                index.append((f"{prefix}.{projection}.{channel_name}", "F16", (count, other), signed((count, other))))
        _write_safetensors(root / "experts" / f"exlr8-layer-{number:03d}.index.safetensors", index)

        gate = (rng.standard_normal((256, h)) * 0.02).astype(np.float32)
        dense = [("mlp.gate.record", "I32", (5,), np.array([router_format, 256, h, 0, 0], np.int32))]
        if router_format == 6:
            bits = gate.view(np.uint32)
            bf16 = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)
            dense.append(("mlp.gate.bf16", "BF16", (256, h), bf16))
        else:
            dense.append(("mlp.gate.fp32", "F32", (256, h), gate))
        dense.append(("mlp.gate.e_score_correction_bias", "F32", (256,),
                      (rng.standard_normal(256) * 0.01).astype(np.float32)))
        _write_safetensors(root / "dense" / f"exlr8-dense-{number:03d}.safetensors", dense)
    (root / "manifests" / "exlr8-manifest-up1.json").write_text(json.dumps({"name": "up1", "layers": plans}))
    return root
