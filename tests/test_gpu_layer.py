"""Whole routed-MoE layer (router + experts + shared + combine) on the GPU
against the CPU oracle of the reference's MoE branch (model.py:385-418)."""

import numpy as np
import pytest

from helpers import assert_bf16_close, host
from oracle import trellis_oracle as ref

pytestmark = pytest.mark.gpu


def _check_layer(layer, tokens, shared, seed_offset=0):
    import torch
    from mlxlr8_b200.fast_router import router
    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.synthetic import host_copy

    x, residual = layer.tokens(tokens, seed_offset)
    moe = MoELayer(layer.gate_weight, layer.bias, layer.experts)
    out, ids, scores = moe(x, residual, return_routing=True)
    torch.cuda.synchronize()
    logits, ids2, _ = router(x, layer.gate_weight, layer.bias)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids2.cpu().numpy())
    ids_np = ids.cpu().numpy()
    used = np.unique(ids_np[:, :8] if shared == "bf16" else ids_np)
    hc = host_copy(layer, used)
    xs, rs = host(x), host(residual)
    exp_logits = ref.router_logits(xs, hc["gate_weight"])
    np.testing.assert_allclose(host(logits), exp_logits, rtol=1e-4, atol=2e-5)
    # Routing from the kernel's own logits (an fp32 sum-order tie at rank 8/9
    # would otherwise flip a selection; the oracle is exact given logits).
    e_out, e_ids, e_scores = ref.moe_layer(xs, rs, hc["gate_weight"], hc["bias"], hc["packed"], hc["scales"],
                                           layer.experts.k, layer.experts.hidden, layer.experts.intermediate,
                                           shared=hc["shared"], dtype="bfloat16", logits=host(logits))
    np.testing.assert_array_equal(ids_np, e_ids)
    np.testing.assert_allclose(scores.cpu().numpy(), e_scores, rtol=1e-6, atol=1e-7)
    assert_bf16_close(host(out), e_out)


@pytest.mark.parametrize("tokens", [1, 4, 32])
@pytest.mark.parametrize("shared", ["bf16", "trellis"])
def test_small_layer_matches_oracle(tokens, shared):
    from mlxlr8_b200.synthetic import make_layer

    layer = make_layer(seed=5, hidden=256, intermediate=128, shared=shared, scale_sigma=0.1)
    _check_layer(layer, tokens, shared)


def test_glm_layer_one_token():
    from mlxlr8_b200.synthetic import make_layer

    layer = make_layer(seed=11)
    _check_layer(layer, 1, "bf16")


@pytest.mark.parametrize("tokens", [1, 4, 40])
def test_graph_mode_replays_the_eager_layer(tokens):
    """MoELayer(..., out=, graph=True): the first call captures the kernel
    chain, later calls replay it on whatever the same buffers now hold; every
    result equals the eager call on the same inputs bit for bit, routing
    included (40 tokens take the grouped GEMM path)."""
    import torch

    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.synthetic import make_layer

    layer = make_layer(seed=17, hidden=256, intermediate=128, shared="bf16")
    moe = MoELayer(layer.gate_weight, layer.bias, layer.experts)
    x, residual = layer.tokens(tokens)
    xb, rb = x.clone(), residual.clone()
    out = torch.empty_like(residual)
    for step in range(3):
        x2, r2 = layer.tokens(tokens, seed_offset=50 + step)
        xb.copy_(x2)
        rb.copy_(r2)
        got, ids, scores = moe(xb, rb, out=out, graph=True, return_routing=True)
        want, wids, wscores = moe(x2, r2, return_routing=True)
        torch.cuda.synchronize()
        assert got.data_ptr() == out.data_ptr()
        assert torch.equal(got, want)
        assert torch.equal(ids, wids) and torch.equal(scores, wscores)
    moe.clear_graphs()


def test_graph_mode_with_pinned_host_buffers():
    """graph=True with pinned host x / residual / out: the captured graph
    copies in, runs the layer and copies out; the host result equals the
    eager device call bit for bit on every replay."""
    import torch

    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.synthetic import make_layer

    layer = make_layer(seed=19, hidden=256, intermediate=128, shared="bf16")
    moe = MoELayer(layer.gate_weight, layer.bias, layer.experts)
    x0, r0 = layer.tokens(2)
    xh, rh = x0.cpu().pin_memory(), r0.cpu().pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    for step in range(3):
        x2, r2 = layer.tokens(2, seed_offset=70 + step)
        xh.copy_(x2.cpu())
        rh.copy_(r2.cpu())
        moe(xh, rh, out=oh, graph=True)
        want = moe(x2, r2)
        torch.cuda.synchronize()
        assert torch.equal(oh, want.cpu())
    moe.clear_graphs()


@pytest.mark.parametrize("tokens", [1, 40])
def test_eager_host_buffers_match_the_device_call(tokens):
    """Pinned host x / residual / out without a graph: the staging kernel
    reads the inputs over PCIe and the finishing kernel writes ``out`` on the
    host; equal to the device call bit for bit (40 tokens take the grouped
    GEMM path).  Without ``out`` the result is a new pinned host tensor."""
    import torch

    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.synthetic import make_layer

    layer = make_layer(seed=23, hidden=256, intermediate=128, shared="bf16")
    moe = MoELayer(layer.gate_weight, layer.bias, layer.experts)
    x, r = layer.tokens(tokens, seed_offset=90)
    xh, rh = x.cpu().pin_memory(), r.cpu().pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    got, ids, scores = moe(xh, rh, out=oh, return_routing=True)
    want, wids, wscores = moe(x, r, return_routing=True)
    torch.cuda.synchronize()
    assert got.data_ptr() == oh.data_ptr()
    assert torch.equal(oh, want.cpu())
    assert torch.equal(ids, wids) and torch.equal(scores, wscores)
    fresh = moe(xh, rh)
    torch.cuda.synchronize()
    assert fresh.is_pinned() and torch.equal(fresh, want.cpu())


def test_host_buffers_refuse_pageable_memory():
    """Pageable host tensors are refused on the host (the layer's check, and
    the library's pointer-kind check behind it): no kernel reads them."""
    import ctypes

    import torch

    from mlxlr8_b200 import _lib
    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.synthetic import make_layer

    layer = make_layer(seed=29, hidden=256, intermediate=128, shared="bf16")
    moe = MoELayer(layer.gate_weight, layer.bias, layer.experts)
    x, r = layer.tokens(2)
    with pytest.raises(ValueError):
        moe(x.cpu(), r.cpu())
    lib = _lib.lib()
    pageable = x.cpu()
    dev = torch.empty_like(x)
    ptr = ctypes.c_void_p(0)
    assert lib.exlr8_host_device_pointer(pageable.data_ptr(), ctypes.byref(ptr)) == 11
    nbytes = pageable.numel() * pageable.element_size()
    assert lib.exlr8_stage_in(pageable.data_ptr(), dev.data_ptr(), pageable.data_ptr(), dev.data_ptr(), nbytes,
                              _lib.stream_handle(dev.device)) == 11
    assert lib.exlr8_host_device_pointer(dev.data_ptr(), ctypes.byref(ptr)) == 0 and ptr.value == dev.data_ptr()
