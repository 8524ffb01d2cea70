"""Router kernels against the reference's independent NumPy expectation."""

import numpy as np
import pytest

from oracle import trellis_oracle as ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", ["random", "bias", "ties", "saturated", "zero"])
@pytest.mark.parametrize("rows", [1, 2, 3, 4])
def test_route_selection_and_weights(golden, case, rows):
    import torch
    from mlxlr8_b200.fast_router import route

    logits = torch.from_numpy(golden[f"route_{case}_{rows}_logits"]).cuda()
    bias = torch.from_numpy(golden[f"route_{case}_{rows}_bias"]).cuda()
    ids, scores = route(logits, bias)
    ids, scores = ids.cpu().numpy(), scores.cpu().numpy()
    assert ids.shape == (1, rows, 9) and scores.shape == (1, rows, 8)
    np.testing.assert_array_equal(ids[..., 8], 256)
    np.testing.assert_array_equal(ids[..., :8], golden[f"route_{case}_{rows}_ids"])
    np.testing.assert_allclose(scores, golden[f"route_{case}_{rows}_scores"], rtol=1e-6, atol=1e-7)
    assert np.isfinite(scores).all()


def test_route_strided_input(golden):
    import torch
    from mlxlr8_b200.fast_router import route

    logits = torch.from_numpy(golden["route_random_4_logits"]).cuda()
    bias = torch.from_numpy(golden["route_random_4_bias"]).cuda()
    strided = torch.stack([logits, torch.zeros_like(logits)], dim=-1)[..., 0]
    ids, _ = route(strided, torch.stack([bias, torch.zeros_like(bias)], dim=-1)[..., 0])
    np.testing.assert_array_equal(ids.cpu().numpy()[..., :8], golden["route_random_4_ids"])


@pytest.mark.parametrize("tokens", [1, 4, 13, 32])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_gate_gemv_and_route(tokens, dtype):
    import torch
    from helpers import torch_dtype
    from mlxlr8_b200.fast_router import router

    rng = np.random.default_rng(400 + tokens)
    x = torch.from_numpy(rng.normal(size=(tokens, 6144)).astype(np.float32)).to(torch_dtype(dtype)).cuda()
    w = torch.from_numpy((0.02 * rng.normal(size=(256, 6144))).astype(np.float32)).cuda()
    b = torch.from_numpy((0.01 * rng.normal(size=256)).astype(np.float32)).cuda()
    logits, ids, scores = router(x, w, b)
    expected = ref.router_logits(x.float().cpu().numpy(), w.cpu().numpy())
    np.testing.assert_allclose(logits.cpu().numpy(), expected, rtol=1e-4, atol=2e-5)
    # Selection on the kernel's own logits is exact.
    e_ids, e_scores = ref.route(logits.cpu().numpy(), b.cpu().numpy())
    np.testing.assert_array_equal(ids.cpu().numpy(), e_ids)
    np.testing.assert_allclose(scores.cpu().numpy(), e_scores, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("tokens", [64, 300])
def test_tensor_core_gate_product(dtype, tokens):
    """Prefill gate product (bf16 piece products on the tensor cores) against a
    float64 reference: float32-level agreement, and routing from it equals
    the oracle's routing of the same logits."""
    import torch

    from helpers import torch_dtype
    from mlxlr8_b200.fast_router import router_logits

    g = torch.Generator(device="cuda")
    g.manual_seed(tokens)
    x = torch.randn(tokens, 6144, generator=g, device="cuda").to(torch_dtype(dtype))
    w = 0.02 * torch.randn(256, 6144, generator=g, device="cuda")
    logits = router_logits(x, w)
    torch.cuda.synchronize()
    exact = x.double().cpu().numpy() @ w.double().cpu().numpy().T
    got = logits.double().cpu().numpy()
    err = np.abs(got - exact).max() / np.abs(exact).max()
    assert err < 1e-5, err  # float32 accumulation over 6144 terms: ~sqrt(6144) * 2^-24
    np.testing.assert_allclose(got, exact, rtol=1e-4, atol=2e-5)
