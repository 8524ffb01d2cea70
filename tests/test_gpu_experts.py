"""Trellis expert operators on the GPU against the CPU oracle and the
reference's own test formulas (exlr8 tests/test_trellis.py,
tests/test_fast_decode.py, tests/test_fast_prefill.py)."""

import numpy as np
import pytest

from helpers import assert_bf16_close, host, rel_l2, small_experts, to_device, torch_dtype
from oracle import trellis_oracle as ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("side", [1, 2])
@pytest.mark.parametrize("per_slot", [0, 1])
def test_expert_linear_matches_reference_formula(golden, side, per_slot):
    import torch
    from mlxlr8_b200.trellis import expert_linear

    x = torch.from_numpy(golden[f"linear_s{side}_p{per_slot}_x"]).cuda()
    ids = torch.from_numpy(golden["linear_ids"].astype(np.int32)).cuda()
    packed = torch.from_numpy(golden[f"linear_s{side}_packed"]).cuda()
    suh = torch.from_numpy(golden[f"linear_s{side}_in_scale"]).cuda()
    svh = torch.from_numpy(golden[f"linear_s{side}_out_scale"]).cuda()
    actual = expert_linear(x, ids, packed, suh, svh, 4, 128, 256, side)
    assert actual.shape == (2, 2, 256) and actual.dtype == torch.float32
    np.testing.assert_allclose(host(actual), golden[f"linear_s{side}_p{per_slot}_expected"], rtol=4e-5, atol=3e-6)


@pytest.mark.parametrize("k", [2, 3, 4])
@pytest.mark.parametrize("side", [1, 2])
@pytest.mark.parametrize("per_slot", [False, True])
def test_grouped_linear_matches_oracle(k, side, per_slot):
    # tests/test_fast_prefill.py:31-57 shape: 4 experts, ragged reuse of experts.
    import torch
    from mlxlr8_b200.fast_prefill import grouped_expert_linear

    rng = np.random.default_rng(39)
    experts, width, output = 4, 256, 384
    packed = rng.integers(0, 256, (experts, width * output * k // 8), dtype=np.uint8)
    in_scale = rng.uniform(-0.1, 0.1, (experts, width)).astype(np.float16)
    out_scale = rng.uniform(-0.1, 0.1, (experts, output)).astype(np.float16)
    ids = np.array([[3, 0, 3], [1, 0, 2], [0, 3, 1]], dtype=np.int32)
    x = rng.normal(size=(3, 3, width) if per_slot else (3, width)).astype(np.float32)
    expected = ref.expert_linear(x, ids, packed, in_scale, out_scale, k, width, output, side)
    actual = grouped_expert_linear(torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda(),
                                   torch.from_numpy(packed).cuda(), torch.from_numpy(in_scale).cuda(),
                                   torch.from_numpy(out_scale).cuda(), k, width, output, side)
    np.testing.assert_allclose(host(actual), expected, rtol=5e-5, atol=3e-6)


@pytest.mark.parametrize("tokens", [3, 12, 40, 129])
def test_row_blocks_and_ragged_segments(tokens):
    # tests/test_fast_prefill.py:60-78: expert 1 absent, expert 0 spans many rows.
    import torch
    from mlxlr8_b200.trellis import expert_linear

    rng = np.random.default_rng(41)
    packed = rng.integers(0, 256, (3, 8192), dtype=np.uint8)
    in_scale = rng.uniform(-0.1, 0.1, (3, 128)).astype(np.float16)
    out_scale = rng.uniform(-0.1, 0.1, (3, 128)).astype(np.float16)
    x = rng.normal(size=(tokens, 128)).astype(np.float32)
    ids = np.zeros((tokens, 2), dtype=np.int32)
    ids[::3, 0] = 2
    expected = ref.expert_linear(x, ids, packed, in_scale, out_scale, 4, 128, 128, 1)
    actual = expert_linear(torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda(), torch.from_numpy(packed).cuda(),
                           torch.from_numpy(in_scale).cuda(), torch.from_numpy(out_scale).cuda(), 4, 128, 128)
    np.testing.assert_allclose(host(actual), expected, rtol=5e-5, atol=2e-6)


def test_float32_accumulation_beyond_float16_range():
    # tests/test_fast_prefill.py:207-228: operands fit float16, sums do not.
    import torch
    from mlxlr8_b200.trellis import expert_linear

    width, output = 6144, 128
    x = np.zeros((2, width), dtype=np.float32)
    x[:, ::128] = np.float32(10 * np.sqrt(128))
    actual = host(expert_linear(torch.from_numpy(x).cuda(), torch.zeros(2, 1, dtype=torch.int32, device="cuda"),
                                torch.zeros(width * output // 2, dtype=torch.uint8, device="cuda"),
                                torch.ones(1, width, device="cuda"), torch.ones(1, output, device="cuda"),
                                4, width, output))
    inner_sum = width * 10 * float(ref.mcg_codebook()[0])
    assert inner_sum > float(np.finfo(np.float16).max)
    expected = np.zeros((2, 1, output), dtype=np.float32)
    expected[:, :, 0] = inner_sum * np.sqrt(128)
    assert np.isfinite(actual).all()
    np.testing.assert_allclose(actual, expected, rtol=2e-5, atol=0.01)


def test_large_activations_keep_precision():
    # Activations far outside the float16 range: the per-row power-of-two
    # scale keeps the hi/lo operands finite.
    import torch
    from mlxlr8_b200.trellis import expert_linear

    rng = np.random.default_rng(7)
    packed = rng.integers(0, 256, 2 * 256 * 128 // 2, dtype=np.uint8)
    ins = np.ones((2, 256), np.float32)
    outs = np.ones((2, 128), np.float32)
    ids = np.array([[0], [1]], np.int32)
    for magnitude in (1e-6, 1.0, 1e6):
        x = (magnitude * rng.normal(size=(2, 256))).astype(np.float32)
        expected = ref.expert_linear(x, ids, packed, ins, outs, 4, 256, 128, 1)
        actual = host(expert_linear(torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda(),
                                    torch.from_numpy(packed).cuda(), torch.from_numpy(ins).cuda(),
                                    torch.from_numpy(outs).cuda(), 4, 256, 128, 1))
        assert rel_l2(actual, expected) < 1e-6


@pytest.mark.parametrize("k", [2, 3, 4])
@pytest.mark.parametrize("per_slot", [False, True])
def test_fused_expert_mlp_matches_oracle(k, per_slot):
    # tests/test_fast_decode.py:132-148 (fp32 tolerance of the reference test).
    import torch
    from mlxlr8_b200.fast_decode import fast_expert_mlp

    packed, scales = small_experts(k=k)
    ids = np.array([[2, 0], [1, 2]], dtype=np.int32)
    shape = (2, 2, 256) if per_slot else (2, 256)
    x = np.random.default_rng(29).normal(size=shape).astype(np.float32)
    expected = ref.expert_mlp_fused(x, ids, packed, scales, k, 256, 384, "float32")
    dp, ds = to_device(packed, scales)
    actual = fast_expert_mlp(torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda(), dp, ds, k, 256, 384)
    assert actual.shape == (2, 2, 256)
    np.testing.assert_allclose(host(actual), expected, rtol=7e-5, atol=5e-7)
    # The un-fused reference order (expert_linear, typed SwiGLU, expert_linear).
    unfused = ref.expert_mlp(x, ids, packed, scales, k, 256, 384, "float32")
    np.testing.assert_allclose(host(actual), unfused, rtol=7e-5, atol=5e-7)


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_full_glm_expert_dimensions(dtype):
    # tests/test_fast_decode.py:151-172: nine experts at 6144 x 2048.
    import torch
    from mlxlr8_b200.fast_decode import fast_expert_mlp

    packed, scales = small_experts(hidden=6144, intermediate=2048, experts=9)
    ids = np.arange(9, dtype=np.int32).reshape(1, 9)
    x32 = np.random.default_rng(32).normal(size=(1, 6144)).astype(np.float32)
    xt = torch.from_numpy(x32).to(torch_dtype(dtype)).cuda()
    x_in = host(xt)
    expected = ref.expert_mlp_fused(x_in, ids, packed, scales, 4, 6144, 2048, dtype)
    dp, ds = to_device(packed, scales)
    actual = host(fast_expert_mlp(xt, torch.from_numpy(ids).cuda(), dp, ds, 4, 6144, 2048))
    limit = 3e-6 if dtype == "float32" else 0.001 if dtype == "float16" else 0.007
    assert rel_l2(actual, expected) < limit
    if dtype != "float32":
        assert_bf16_close(actual, expected)


@pytest.mark.parametrize("rows", [2, 3, 4])
@pytest.mark.parametrize("pattern", ["shared", "all", "changing", "duplicates"])
def test_multirow_reuse_keeps_each_output(rows, pattern):
    # tests/test_fast_decode.py:203-225: rows sharing experts give the same
    # result as each row alone.
    import torch
    from mlxlr8_b200.fast_decode import fast_expert_mlp

    packed, scales = small_experts(experts=40)
    if pattern == "shared":
        ids = np.concatenate([np.arange(rows * 8).reshape(rows, 8), np.full((rows, 1), 39)], axis=-1)
    elif pattern == "all":
        ids = np.stack([np.roll(np.arange(9), r) for r in range(rows)])
    elif pattern == "changing":
        ids = np.concatenate([np.stack([np.arange(r * 4, r * 4 + 8) for r in range(rows)]),
                              np.full((rows, 1), 39)], axis=-1)
    else:
        ids = np.tile([0, 0, 1, 1, 2, 2, 0, 1, 2], (rows, 1))
    ids = ids.astype(np.int32)
    x = torch.from_numpy(np.random.default_rng(431).normal(size=(rows, 256)).astype(np.float32)).cuda()
    dp, ds = to_device(packed, scales)
    together = host(fast_expert_mlp(x, torch.from_numpy(ids).cuda(), dp, ds, 4, 256, 384))
    for r in range(rows):
        alone = host(fast_expert_mlp(x[r:r + 1], torch.from_numpy(ids[r:r + 1]).cuda(), dp, ds, 4, 256, 384))
        np.testing.assert_allclose(together[r], alone[0], rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("rows", [1, 2, 3, 4])
def test_finish_keeps_typed_weighted_shared_and_residual_sums(dtype, rows):
    # tests/test_fast_decode.py:456-476 and test_joined_mxfp4.py:87-101.
    import torch
    from mlxlr8_b200.fast_decode import expert_mlp_finish, fast_expert_mlp

    packed, scales = small_experts(experts=9)
    rng = np.random.default_rng(731)
    ids = np.tile([7, 0, 3, 3, 6, 2, 5, 1, 8], (rows, 1)).astype(np.int32)
    scores = rng.uniform(0.01, 1, (rows, 8)).astype(np.float32)
    tdt = torch_dtype(dtype)
    x = torch.from_numpy(rng.normal(size=(rows, 256)).astype(np.float32)).to(tdt).cuda()
    residual = torch.from_numpy(rng.normal(size=(rows, 256)).astype(np.float32)).to(tdt).cuda()
    dp, ds = to_device(packed, scales)
    tid = torch.from_numpy(ids).cuda()
    values = host(fast_expert_mlp(x, tid, dp, ds, 4, 256, 384))
    expected = ref.combine(values, scores, host(residual), dtype)
    actual = host(expert_mlp_finish(x, tid, torch.from_numpy(scores).cuda(), residual, dp, ds, 4, 256, 384))
    np.testing.assert_array_equal(actual.view(np.uint32), expected.view(np.uint32))


def test_out_of_range_ids_are_reported_and_zero():
    import ctypes

    import torch
    from mlxlr8_b200 import _lib
    from mlxlr8_b200.fast_decode import trellis_experts

    packed, scales = small_experts(experts=3)
    dp, ds = to_device(packed, scales)
    st, count = trellis_experts(dp, ds, 4, 256, 384)
    ids = torch.tensor([[0, 5], [1, 2]], dtype=torch.int32, device="cuda")
    x = torch.randn(2, 256, device="cuda")
    out = torch.full((2, 2, 256), 7.0, device="cuda")
    lib = _lib.lib()
    ws = _lib.workspace(lib.exlr8_expert_mlp_workspace(2, 2, 256, 384, count), x.device)
    stream = _lib.stream_handle(x.device)
    _lib.check(lib.exlr8_expert_mlp(x.data_ptr(), 0, 0, ids.data_ptr(), 2, 2, st, out.data_ptr(), ws.data_ptr(),
                                    ws.numel(), stream))
    bad = ctypes.c_int64(-1)
    _lib.check(lib.exlr8_workspace_bad_ids(ws.data_ptr(), ctypes.byref(bad), stream))
    assert bad.value == 1
    assert torch.all(out[0, 1] == 0)
    assert torch.isfinite(out).all()
