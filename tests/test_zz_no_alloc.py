"""exlr8_moe_layer_noalloc: the MoE layer for callers that cannot allocate.

A host that holds device pointers but owns no device allocator (an FFI caller
fed tensors by another runtime, or a server whose memory pool is fixed at
start-up) cannot pass the workspace that exlr8_moe_layer takes.  The no-alloc
entry point runs the same layer on a fixed scratch array inside the library.
These tests call it through the C ABI and compare it with exlr8_moe_layer on
two calls in a row (the second call finds the first call's data in the shared
scratch), and check that a request larger than the fixed scratch is refused.

This file is collected last on purpose: a run that stops at the first
failure has run every other test before it.  It also passes on its own in a
fresh process.
"""

import ctypes

import numpy as np
import pytest

from helpers import assert_bf16_close, host

pytestmark = pytest.mark.gpu


def _noalloc(lib, moe, x, residual):
    import torch

    tokens = x.numel() // x.shape[-1]
    out = torch.empty_like(residual)
    ids = torch.empty(tokens, 9, dtype=torch.int32, device=x.device)
    scores = torch.empty(tokens, 8, dtype=torch.float32, device=x.device)
    status = lib.exlr8_moe_layer_noalloc(x.data_ptr(), 2, residual.data_ptr(), tokens, moe.gate_weight.data_ptr(),
                                         moe.bias.data_ptr(), moe._struct, moe._shared, out.data_ptr(),
                                         ids.data_ptr(), scores.data_ptr(),
                                         torch.cuda.current_stream(x.device).cuda_stream)
    return status, out, ids, scores


@pytest.mark.parametrize("hidden, intermediate, tokens", [(256, 128, 3), (256, 128, 16), (6144, 2048, 2),
                                                      (6144, 2048, 5)])
def test_noalloc_matches_workspace_entry_point_on_two_calls(hidden, intermediate, tokens):
    import torch
    from mlxlr8_b200 import _lib
    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.synthetic import make_layer

    lib = _lib.load()
    layer = make_layer(seed=21, hidden=hidden, intermediate=intermediate)
    moe = MoELayer(layer.gate_weight, layer.bias, layer.experts)
    for call in range(2):
        x, residual = layer.tokens(tokens, seed_offset=call)
        expected, e_ids, e_scores = moe(x, residual, return_routing=True)
        status, out, ids, scores = _noalloc(lib, moe, x, residual)
        _lib.check(status)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(ids.cpu().numpy(), e_ids.cpu().numpy())
        np.testing.assert_allclose(scores.cpu().numpy(), e_scores.cpu().numpy(), rtol=1e-6, atol=1e-7)
        assert_bf16_close(host(out), host(expected))


@pytest.mark.parametrize("hidden, intermediate, tokens", [(6144, 2048, 6), (6144, 2048, 64), (256, 128, 24)])
def test_noalloc_refuses_requests_beyond_its_fixed_scratch(hidden, intermediate, tokens):
    """Six tokens at GLM-5 width need 16.5 MB; above 16 tokens the layer takes
    the grouped-GEMM path, whose workspace (over 100 MB even at width 256)
    never fits, so that path is never taken through this entry point."""
    import torch
    from mlxlr8_b200 import _lib
    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.synthetic import make_layer

    lib = _lib.load()
    layer = make_layer(seed=22, hidden=hidden, intermediate=intermediate)
    moe = MoELayer(layer.gate_weight, layer.bias, layer.experts)
    assert lib.exlr8_moe_layer_workspace(tokens, hidden, intermediate, 256) > 16 * 1024 * 1024
    x, residual = layer.tokens(tokens)
    status, out, _, _ = _noalloc(lib, moe, x, residual)
    assert status == 15
    with pytest.raises(ValueError, match="fixed no-allocation buffer"):
        _lib.check(status)
    # The refusal happens before any launch; the stream is still healthy.
    torch.cuda.synchronize()
