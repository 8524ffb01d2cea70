"""Load-time trellis -> MXFP4 re-encode (joined_mxfp4.py:12-47) and the MLX
``quantize(mode="mxfp4")`` rule on the GPU, bit-exact against the CPU oracle.

Mirrors test_joined_mxfp4.py:18-58: the reference fixture (rng 817, h 256,
m 128, 257 matrices, gate/up in-scales with per-block signs times a shared
sign vector) and the check that ``weights[i, offset:offset + out]`` equals
the quantisation of the folded, transposed decode for matrices 0, 1, 255
and 256.  Codes and scales are integers: the bar is equality.
"""

import numpy as np
import pytest

from helpers import host, rel_l2, to_device
from oracle import trellis_oracle as ref

pytestmark = pytest.mark.gpu

F32 = np.float32


def _u32(t):
    return t.cpu().numpy().view(np.uint32)


def _reference_fixture(count=257, h=256, m=128, scale_dtype=np.float16):
    rng = np.random.default_rng(817)
    signs = rng.choice([-1, 1], h).astype(np.float16)
    packed, scales = {}, {}
    for projection in ("gate", "up", "down"):
        incoming, outgoing = (m, h) if projection == "down" else (h, m)
        packed[projection] = rng.integers(0, 256, count * h * m // 2, dtype=np.uint8)
        inc = rng.uniform(.01, .04, (count, incoming)).astype(np.float16)
        if projection != "down":
            block = rng.uniform(.01, .04, (count, h // 128)).astype(np.float16)
            block *= rng.choice([-1, 1], block.shape).astype(np.float16)
            inc = np.repeat(block, 128, axis=-1) * signs
        out = rng.uniform(-.5, .5, (count, outgoing)).astype(np.float16)
        scales[projection] = (inc.astype(scale_dtype), out.astype(scale_dtype))
    return packed, scales


def _expert(packed, scales, h, m, k=4):
    from mlxlr8_b200.experts import ExpertLayer

    p, s = to_device(packed, scales)
    return ExpertLayer(p, s, k, h, m)


def _edge_rows():
    """Rows of 64 values (two blocks each) covering the rounding rules."""
    rng = np.random.default_rng(21)
    rows = []
    levels = ref.e2m1_value(np.arange(16))
    for exp in (-30, -4, 0, 9):
        r = rng.choice(levels, 64).astype(F32) * F32(2.0 ** exp)
        r[0] = r[32] = F32(6.0 * 2.0 ** exp)
        rows.append(r)
    ties = np.array([6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, -0.0],
                    F32)
    rows.append(np.concatenate([ties, ties * 0.5, ties * 4, ties * 0.125]).astype(F32))
    for n in (-5, -1, 0, 3):
        centre = F32(6.0 * np.sqrt(2.0) * 2.0 ** n)
        sweep = centre + np.arange(-64, 64, dtype=F32) * np.spacing(centre)
        for i in range(0, 128, 2):
            r = (rng.uniform(-1, 1, 64) * float(centre)).astype(F32)
            r[5], r[40] = sweep[i], -sweep[i + 1]
            rows.append(r)
    z = np.zeros(64, F32)
    rows.append(z.copy())
    nz = np.full(64, -0.0, F32)
    nz[40] = 1e-3
    rows.append(nz)
    tiny = (rng.uniform(-1, 1, 64) * 1e-40).astype(F32)
    rows.append(tiny)
    huge = (rng.uniform(-1, 1, 64) * 3e38).astype(F32)
    rows.append(huge)
    wide = (rng.standard_normal((512, 64)) * np.exp(rng.uniform(-20, 20, (512, 1)))).astype(F32)
    return np.concatenate([np.stack(rows), wide])


def test_quantize_rows_bit_exact():
    import torch

    from mlxlr8_b200.joined_mxfp4 import quantize

    w = _edge_rows()
    codes, scales = quantize(torch.from_numpy(w).cuda())
    torch.cuda.synchronize()
    e_codes, e_scales = ref.mxfp4_quantize(w)
    np.testing.assert_array_equal(scales.cpu().numpy(), e_scales)
    np.testing.assert_array_equal(_u32(codes), e_codes)


def test_quantize_batched_shape_and_empty():
    import torch

    from mlxlr8_b200.joined_mxfp4 import quantize

    g = torch.Generator(device="cuda")
    g.manual_seed(4)
    w = torch.randn(3, 5, 256, generator=g, device="cuda")
    codes, scales = quantize(w)
    assert codes.shape == (3, 5, 32) and scales.shape == (3, 5, 8)
    e_codes, e_scales = ref.mxfp4_quantize(host(w))
    np.testing.assert_array_equal(_u32(codes), e_codes)
    np.testing.assert_array_equal(scales.cpu().numpy(), e_scales)
    codes, scales = quantize(torch.empty(0, 64, device="cuda"))
    assert codes.shape == (0, 8) and scales.shape == (0, 2)


@pytest.mark.parametrize("scale_dtype", [np.float16, np.float32])
def test_encode_matches_reference_fixture(scale_dtype):
    import torch

    from mlxlr8_b200.joined_mxfp4 import encode

    h, m = 256, 128
    packed, scales = _reference_fixture(scale_dtype=scale_dtype)
    unit, weights = encode(_expert(packed, scales, h, m))
    torch.cuda.synchronize()
    check = (0, 1, 255, 256)
    e_unit, e_weights = ref.encode_joined(packed, scales, 4, h, m, experts=check)
    assert tuple(unit.shape) == (1, h)
    np.testing.assert_array_equal(host(unit)[0], e_unit)
    for name in ("gate_up", "down"):
        codes, sc, none = weights[name]
        assert none is None
        for i in check:
            np.testing.assert_array_equal(_u32(codes[i]), e_weights[name][0][i])
            np.testing.assert_array_equal(sc[i].cpu().numpy(), e_weights[name][1][i])


def test_encode_full_size_matrix():
    """GLM-5 expert geometry (6144 x 2048, K4): matrix 1 of a two-matrix buffer."""
    import torch

    from mlxlr8_b200.joined_mxfp4 import encode

    h, m, count = 6144, 2048, 2
    rng = np.random.default_rng(99)
    packed, scales = {}, {}
    signs = rng.choice([-1, 1], h).astype(np.float16)
    for projection in ("gate", "up", "down"):
        incoming, outgoing = (m, h) if projection == "down" else (h, m)
        packed[projection] = rng.integers(0, 256, count * h * m // 2, dtype=np.uint8)
        inc = rng.uniform(.5, 1.5, (count, incoming)).astype(np.float16)
        if projection != "down":
            inc = inc * signs
        scales[projection] = (inc, rng.uniform(-.5, .5, (count, outgoing)).astype(np.float16))
    unit, weights = encode(_expert(packed, scales, h, m))
    torch.cuda.synchronize()
    _, e_weights = ref.encode_joined(packed, scales, 4, h, m, experts=(1,))
    for name in ("gate_up", "down"):
        np.testing.assert_array_equal(_u32(weights[name][0][1]), e_weights[name][0][1])
        np.testing.assert_array_equal(weights[name][1][1].cpu().numpy(), e_weights[name][1][1])


def test_joined_from_trellis_expert_runs_encoded_weights():
    """JoinedMXFP4(expert) (joined_mxfp4.py:137-141): slots over the GPU-encoded
    weights against the joined oracle on the same weights, and the joined
    output against the trellis path within the MXFP4 re-encode error.

    Folding the gate/up in-scale into the Hadamard-domain rows is exact when
    that scale is one magnitude per 128-channel block times a sign vector
    shared by all experts (the checkpoints' folded layout and the reference
    fixture, test_joined_mxfp4.py:25-31), so the fixture is built that way."""
    import torch

    from mlxlr8_b200.joined_mxfp4 import JoinedMXFP4
    from test_gpu_joined import assert_mxfp4_close

    h, m, count = 512, 256, 9
    rng = np.random.default_rng(31)
    packed, scales = {}, {}
    signs = rng.choice([-1, 1], h).astype(np.float16)
    for projection in ("gate", "up", "down"):
        incoming, outgoing = (m, h) if projection == "down" else (h, m)
        packed[projection] = rng.integers(0, 256, count * h * m // 2, dtype=np.uint8)
        inc = rng.uniform(.02, .06, (count, incoming)).astype(np.float16)
        if projection != "down":
            block = rng.uniform(.02, .06, (count, h // 128)).astype(np.float16)
            block *= rng.choice([-1, 1], block.shape).astype(np.float16)
            inc = np.repeat(block, 128, axis=-1) * signs
        scales[projection] = (inc, rng.uniform(-.5, .5, (count, outgoing)).astype(np.float16))
    expert = _expert(packed, scales, h, m)
    joined = JoinedMXFP4(expert)
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    x = torch.randn(6, h, generator=g, device="cuda").to(torch.bfloat16)
    ids = torch.randint(0, count, (6, 9), generator=g, device="cuda", dtype=torch.int32)
    out = joined.slots(x, ids)
    torch.cuda.synchronize()
    gu = tuple(t.cpu().numpy() for t in joined.weights["gate_up"][:2])
    dn = tuple(t.cpu().numpy() for t in joined.weights["down"][:2])
    gu = (gu[0].view(np.uint32), gu[1])
    dn = (dn[0].view(np.uint32), dn[1])
    sc = {"gate": scales["gate"][1].astype(F32), "up": scales["up"][1].astype(F32),
          "down": (scales["down"][0].astype(F32), scales["down"][1].astype(F32))}
    want = ref.joined_slots(host(x), ids.cpu().numpy(), host(joined.unit), gu, dn, sc, h, m, "bfloat16")
    assert_mxfp4_close(host(out), want)
    trellis = expert(x, ids)
    torch.cuda.synchronize()
    # Three chained MXFP4 projections: the CPU restatement of both paths
    # differs by 0.21 relative L2 on this fixture.
    assert rel_l2(host(out), host(trellis)) < 0.3
