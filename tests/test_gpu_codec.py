"""Trellis codec on the GPU: bit-exact against the reference's codebook and decoder."""

import numpy as np
import pytest

from oracle import trellis_oracle as ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("paired", [False, True])
def test_codebook_bit_exact_over_all_states(golden, paired):
    from mlxlr8_b200.trellis import mcg_codebook

    values = mcg_codebook(paired=paired).cpu().numpy()
    np.testing.assert_array_equal(values.view(np.uint16), golden["codebook_bits"])


@pytest.mark.parametrize("k", [2, 3, 4])
@pytest.mark.parametrize("side", [0, 1, 2])
def test_decode_matches_reference_bitstream(golden, k, side):
    import torch
    from mlxlr8_b200.trellis import decode_trellis

    packed = torch.from_numpy(golden[f"decode_k{k}_s{side}_packed"]).cuda()
    inner = decode_trellis(packed, k, 128, 256, side).cpu().numpy()
    expected = golden[f"decode_k{k}_s{side}_inner_bits"].view(np.float16).astype(np.float32)
    np.testing.assert_array_equal(inner.view(np.uint32), expected.view(np.uint32))


@pytest.mark.parametrize("k", [2, 3, 4])
@pytest.mark.parametrize("side", [1, 2])
def test_decode_second_matrix_and_dequantize(golden, k, side):
    import torch
    from mlxlr8_b200.trellis import decode_trellis, dequantize_trellis

    a, b = (128, 256) if side == 1 else (256, 128)
    packed = golden[f"rand_k{k}_s{side}_packed"]
    inner = decode_trellis(torch.from_numpy(packed).cuda(), k, a, b, side, matrix=1).cpu().numpy()
    expected = golden[f"rand_k{k}_s{side}_inner1_bits"].view(np.float16).astype(np.float32)
    np.testing.assert_array_equal(inner, expected)
    second = torch.from_numpy(packed[a * b * k // 8:].copy()).cuda()
    suh = torch.from_numpy(golden[f"rand_k{k}_s{side}_suh"]).cuda()
    svh = torch.from_numpy(golden[f"rand_k{k}_s{side}_svh"]).cuda()
    weight = dequantize_trellis(second, suh, svh, k, a, b, side).cpu().numpy()
    np.testing.assert_allclose(weight, golden[f"rand_k{k}_s{side}_dequant1"], rtol=2e-5, atol=2e-7)


def test_dequantize_rejects_several_matrices(golden):
    import torch
    from mlxlr8_b200.trellis import dequantize_trellis

    packed = torch.from_numpy(golden["rand_k4_s1_packed"]).cuda()
    s = torch.ones(128, dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError, match="one matrix"):
        dequantize_trellis(packed, s, torch.ones(256, dtype=torch.float16, device="cuda"), 4, 128, 256, 1)


def test_hadamard128_bit_exact_against_reference(golden):
    """The device Hadamard-128 (the transform inside every expert kernel) is
    bit-identical to the reference's hadamard_reference (trellis.py:67-75)."""
    import torch

    from mlxlr8_b200.trellis import _hadamard

    x = torch.from_numpy(golden["hadamard_in"]).cuda()
    out = _hadamard(x).cpu().numpy()
    np.testing.assert_array_equal(out.view(np.uint32), golden["hadamard_out"].view(np.uint32))


def test_hadamard128_large_rows_match_oracle():
    """Many rows of 6144 values (the hidden width) against the oracle's
    restatement, bit for bit, and the transform is an involution."""
    import torch

    from mlxlr8_b200.trellis import _hadamard

    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    x = torch.randn(37, 6144, generator=g, device="cuda")
    out = _hadamard(x)
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32),
                                  ref.hadamard128(x.cpu().numpy()).view(np.uint32))
    np.testing.assert_allclose(_hadamard(out).cpu().numpy(), x.cpu().numpy(), atol=3e-6)
