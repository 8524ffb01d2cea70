"""Pin the CPU oracle against vectors produced by the reference's own code."""

import numpy as np
import pytest

from oracle import trellis_oracle as ref


def test_codebook_matches_reference_bits(golden):
    np.testing.assert_array_equal(ref.mcg_codebook().view(np.uint16), golden["codebook_bits"])
    assert ref.mcg_codebook()[0] == 1.875


def test_round_e4m3_ties_saturation_and_sign(golden):
    out = ref.round_e4m3(golden["e4m3_in"])
    np.testing.assert_array_equal(out.view(np.uint32), golden["e4m3_out"].view(np.uint32))
    assert np.signbit(ref.round_e4m3(np.float32(-0.0)))


def test_hadamard_bit_exact(golden):
    out = ref.hadamard128(golden["hadamard_in"])
    np.testing.assert_array_equal(out.view(np.uint32), golden["hadamard_out"].view(np.uint32))


def test_hadamard_is_normalised_and_block_local():
    x = np.zeros((2, 256), np.float32)
    x[0, 0], x[1, 129] = 1, 2
    np.testing.assert_allclose(ref.hadamard128(ref.hadamard128(x)), x, atol=3e-7)
    assert np.all(ref.hadamard128(x)[0, 128:] == 0)


@pytest.mark.parametrize("k", [2, 3, 4])
@pytest.mark.parametrize("side", [0, 1, 2])
def test_bitstream_permutation_and_storage_orders(golden, k, side):
    packed = golden[f"decode_k{k}_s{side}_packed"]
    inner = ref.decode_trellis(packed, k, 128, 256, side)
    np.testing.assert_array_equal(inner.view(np.uint16), golden[f"decode_k{k}_s{side}_inner_bits"])


def test_direct_k4_words_match_reference_unpack(golden):
    canonical = golden["k4_canonical"]
    words = canonical.view(np.uint32)
    np.testing.assert_array_equal(ref.decode_codewords(words, 4), golden["k4_codewords"])


@pytest.mark.parametrize("k", [2, 3, 4])
@pytest.mark.parametrize("side", [1, 2])
def test_random_bytes_decode_and_dequantize(golden, k, side):
    a, b = (128, 256) if side == 1 else (256, 128)
    packed = golden[f"rand_k{k}_s{side}_packed"]
    inner = ref.decode_trellis(packed, k, a, b, side, expert=1)
    np.testing.assert_array_equal(inner.view(np.uint16), golden[f"rand_k{k}_s{side}_inner1_bits"])
    w = ref.dequantize(packed, golden[f"rand_k{k}_s{side}_suh"], golden[f"rand_k{k}_s{side}_svh"], k, a, b, side, 1)
    np.testing.assert_allclose(w, golden[f"rand_k{k}_s{side}_dequant1"], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("side", [1, 2])
@pytest.mark.parametrize("per_slot", [0, 1])
def test_expert_linear_matches_reference_formula(golden, side, per_slot):
    actual = ref.expert_linear(golden[f"linear_s{side}_p{per_slot}_x"], golden["linear_ids"],
                               golden[f"linear_s{side}_packed"], golden[f"linear_s{side}_in_scale"],
                               golden[f"linear_s{side}_out_scale"], 4, 128, 256, side)
    np.testing.assert_allclose(actual, golden[f"linear_s{side}_p{per_slot}_expected"], rtol=4e-5, atol=3e-6)


@pytest.mark.parametrize("case", ["random", "bias", "ties", "saturated", "zero"])
@pytest.mark.parametrize("rows", [1, 2, 3, 4])
def test_router_matches_reference_expectation(golden, case, rows):
    ids, scores = ref.route(golden[f"route_{case}_{rows}_logits"], golden[f"route_{case}_{rows}_bias"])
    np.testing.assert_array_equal(ids[..., 8], 256)
    np.testing.assert_array_equal(ids[..., :8], golden[f"route_{case}_{rows}_ids"])
    np.testing.assert_allclose(scores, golden[f"route_{case}_{rows}_scores"], rtol=1e-6, atol=1e-7)


def test_route_experts_bias_and_groups():
    # test_model.py:391-405: bias changes selection but not probability; groups mask.
    ids, w = ref.route_experts(np.array([[3.0, 2.0, -1.0, -2.0]], np.float32),
                               np.array([0, 0, 2, 3], np.float32), top_k=2)
    np.testing.assert_array_equal(ids[0], [2, 3])
    p = 1 / (1 + np.exp(-np.array([-1.0, -2.0])))
    np.testing.assert_allclose(w[0], p / p.sum() * 2.5, rtol=1e-6)
    ids, _ = ref.route_experts(np.array([[4.0, 3.0, 2.0, 1.0]], np.float32), np.zeros(4, np.float32),
                               top_k=2, n_group=2, topk_group=1)
    np.testing.assert_array_equal(ids[0], [0, 1])


def test_half_bit_round_identity_over_all_codewords():
    # test_fast_decode.py:43-53: the integer half-bit round equals the codebook.
    states = np.arange(65536, dtype=np.uint32)
    product = ((states * np.uint32(0xCBAC1FED)) & np.uint32(0x8FFF8FFF)) ^ np.uint32(0x3B603B60)
    summed = (product & 65535).astype(np.uint16).view(np.float16)
    summed = summed + (product >> 16).astype(np.uint16).view(np.float16)
    bits = summed.view(np.uint16).astype(np.uint32)
    magnitude = bits & 32767
    rounded = (bits + 63 + ((bits >> 7) & 1)) & 65408
    normal = rounded.astype(np.uint16).view(np.float16)
    values = np.where(magnitude < 0x2400, np.rint(summed.astype(np.float32) * 512) / 512, normal)
    np.testing.assert_array_equal(values.astype(np.float16).view(np.uint16), ref.mcg_codebook().view(np.uint16))


def test_invalid_byte_count():
    with pytest.raises(ValueError, match="byte count"):
        ref.decode_trellis(np.zeros(5, np.uint8), 4, 128, 128)


def test_combine_order_and_casts():
    rng = np.random.default_rng(731)
    values = ref.round_bf16(rng.normal(size=(3, 9, 128)).astype(np.float32))
    scores = rng.uniform(0.01, 1, (3, 8)).astype(np.float32)
    residual = ref.round_bf16(rng.normal(size=(3, 128)).astype(np.float32))
    out = ref.combine(values, scores, residual, "bfloat16")
    routed = ref.round_bf16((values[:, :8] * scores[..., None]).sum(axis=1))
    expected = ref.round_bf16(residual + ref.round_bf16(routed + values[:, 8]))
    # Summation order may move a result by at most one bf16 step.
    np.testing.assert_allclose(out, expected, rtol=8e-3, atol=1e-6)
    assert np.array_equal(out, ref.round_bf16(out))


def test_static_codebook_codes_match_reference(golden):
    """E4M3 bytes of all 65,536 codebook values (static_cache.py:11-26):
    decoding each byte as E4M3 gives the codebook value back."""
    codes = ref.e4m3_code(ref.mcg_codebook())
    np.testing.assert_array_equal(codes, golden["static_codebook_codes"])
    levels = np.concatenate([ref.e4m3_levels(), [np.nan]])
    back = np.where(codes & 0x80, -1.0, 1.0) * levels[codes & 0x7F]
    np.testing.assert_array_equal(back.astype(np.float16), ref.mcg_codebook())


@pytest.mark.parametrize("k", [2, 3, 4])
@pytest.mark.parametrize("side", [1, 2])
def test_static_expansion_matches_reference(golden, k, side):
    """Exact E4M3 expansion of two stored matrices in tile order
    (static_cache.py:29-42)."""
    a, b = (128, 256) if side == 1 else (256, 128)
    got = ref.expand_static(golden[f"static_k{k}_s{side}_packed"], k, a, b, side)
    np.testing.assert_array_equal(got, golden[f"static_k{k}_s{side}_bytes"])
