"""The residual RMS norm in front of each MoE block and a stack of MoE blocks
with the attention stubbed (model.py:373-418), against the CPU oracle.

The norm's float32 sum of squares is reduced in another order than the
oracle's, so its output may differ in the last bit of a few bf16/f16 values
(one rounding of T(h * inv) moved across a rounding boundary) and by a few
ulps in float32; the MoE blocks use the layer tolerance of the decode and
prefill tests.
"""

import numpy as np
import pytest

from helpers import host, rel_l2, torch_dtype
from oracle import trellis_oracle as ref

pytestmark = pytest.mark.gpu


def _ulp(values, dtype):
    mant = {"bfloat16": 7, "float16": 10, "float32": 23}[dtype]
    mag = np.maximum(np.abs(values), 2.0 ** -14)
    return 2.0 ** (np.floor(np.log2(mag)) - mant)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("hidden, rows, with_residual", [(6144, 3, False), (6144, 2, True), (256, 17, True)])
def test_residual_rms_norm_matches_oracle(dtype, hidden, rows, with_residual):
    import torch

    from mlxlr8_b200.stack import residual_rms_norm

    g = torch.Generator(device="cuda")
    g.manual_seed(hidden + rows)
    td = torch_dtype(dtype)
    x = (2.0 * torch.randn(rows, hidden, generator=g, device="cuda")).to(td)
    r = torch.randn(rows, hidden, generator=g, device="cuda").to(td) if with_residual else None
    w = (1.0 + 0.1 * torch.randn(hidden, generator=g, device="cuda")).to(td)
    h, out = residual_rms_norm(x, w, 1e-5, residual=r, return_sum=True)
    torch.cuda.synchronize()
    eh, eo = ref.residual_rms_norm(host(x), host(w), 1e-5, residual=host(r) if r is not None else None, dtype=dtype)
    np.testing.assert_array_equal(host(h), eh)
    diff = np.abs(host(out) - eo)
    if dtype == "float32":
        # No coarser rounding absorbs the last-bit difference of the reduced
        # scale: a few float32 ulps.
        assert np.all(diff <= 4.01 * _ulp(eo, dtype) + 1e-30)
    else:
        assert np.all(diff <= 1.01 * _ulp(eo, dtype) + 1e-30)
        assert np.mean(diff == 0) > 0.97


@pytest.mark.parametrize("tokens", [2, 24])
def test_stack_blocks_match_oracle(tokens):
    """Three MoE blocks (bf16 shared expert) with their post-attention norms:
    every block's normalised input and output against the oracle of that
    block on the block's own input."""
    import torch

    from mlxlr8_b200.fast_router import router
    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.stack import MoEStack
    from mlxlr8_b200.synthetic import host_copy, make_layer

    layers = [make_layer(seed=60 + i, hidden=256, intermediate=128) for i in range(3)]
    g = torch.Generator(device="cuda")
    g.manual_seed(tokens)
    norms = [(1.0 + 0.1 * torch.randn(256, generator=g, device="cuda")).to(torch.bfloat16) for _ in layers]
    stack = MoEStack([(w, MoELayer(l.gate_weight, l.bias, l.experts)) for w, l in zip(norms, layers)])
    h0 = (3.0 * torch.randn(tokens, 256, generator=g, device="cuda")).to(torch.bfloat16)
    h, steps = stack(h0, trace=True)
    torch.cuda.synchronize()
    assert len(steps) == 3 and steps[-1][2] is h
    for (h_in, xn, out), w, layer in zip(steps, norms, layers):
        _, e_xn = ref.residual_rms_norm(host(h_in), host(w), 1e-5)
        assert np.all(np.abs(host(xn) - e_xn) <= 1.01 * _ulp(e_xn, "bfloat16") + 1e-30)
        logits, ids, _ = router(xn, layer.gate_weight, layer.bias)
        ids_np = ids.cpu().numpy()
        hc = host_copy(layer, np.unique(ids_np[:, :8]))
        e_out, e_ids, _ = ref.moe_layer(host(xn), host(h_in), hc["gate_weight"], hc["bias"], hc["packed"],
                                        hc["scales"], 4, 256, 128, shared=hc["shared"], dtype="bfloat16",
                                        logits=host(logits))
        np.testing.assert_array_equal(ids_np, e_ids)
        got, want = host(out) - host(h_in), e_out - host(h_in)
        scale = float(np.max(np.abs(want)))
        assert float(np.max(np.abs(got - want))) <= 1e-2 * scale
        assert rel_l2(got, want) < 5e-3


def _graph_matches_eager(stack, h0, replays=4):
    """The stack captured as one CUDA graph (its kernels launched back to back,
    so chained launches overlap as far as their dependencies allow) gives the
    eager result bit for bit on every replay."""
    import torch

    stream = torch.cuda.Stream()
    torch.cuda.synchronize()  # weights and h0 were made on the default stream
    with torch.cuda.stream(stream):
        want = stack(h0).clone()  # eager; also allocates the workspaces
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            out = stack(h0)
        for _ in range(replays):
            out.zero_()
            graph.replay()
            stream.synchronize()
            np.testing.assert_array_equal(host(out), host(want))
    del graph


@pytest.mark.parametrize("tokens", [1, 3])
def test_stack_graph_matches_eager_trellis(tokens):
    """Four GLM-5-size K4 blocks (bf16 shared expert streamed beside the
    trellis units) in one graph: every block's kernel chain starts only after
    the previous block, including the shared expert's rows that stream
    without waiting for the routing."""
    import torch

    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.stack import MoEStack
    from mlxlr8_b200.synthetic import make_layer

    layers = [make_layer(seed=400 + i) for i in range(4)]
    g = torch.Generator(device="cuda")
    g.manual_seed(41 + tokens)
    norms = [(1.0 + 0.1 * torch.randn(6144, generator=g, device="cuda")).to(torch.bfloat16) for _ in layers]
    stack = MoEStack([(w, MoELayer(l.gate_weight, l.bias, l.experts)) for w, l in zip(norms, layers)])
    h0 = torch.randn(tokens, 6144, generator=g, device="cuda").to(torch.bfloat16)
    _graph_matches_eager(stack, h0)
    del stack, layers
    torch.cuda.empty_cache()


def test_stack_graph_matches_eager_joined():
    """Two GLM-5-size joined MXFP4 blocks at one token in one graph."""
    import torch

    from mlxlr8_b200.joined_mxfp4 import JoinedMoELayer, JoinedMXFP4
    from mlxlr8_b200.stack import MoEStack
    from mlxlr8_b200.synthetic import make_joined

    blocks = []
    g = torch.Generator(device="cuda")
    g.manual_seed(43)
    for i in range(2):
        j = make_joined(seed=500 + i)
        w = (1.0 + 0.1 * torch.randn(6144, generator=g, device="cuda")).to(torch.bfloat16)
        blocks.append((w, JoinedMoELayer(j.gate_weight, j.bias,
                                         JoinedMXFP4(j.unit, j.weights, j.scales, j.hidden, j.intermediate))))
    h0 = torch.randn(1, 6144, generator=g, device="cuda").to(torch.bfloat16)
    _graph_matches_eager(MoEStack(blocks), h0)
    del blocks
    torch.cuda.empty_cache()
