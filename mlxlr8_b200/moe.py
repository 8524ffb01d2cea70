"""One routed-MoE layer on the GPU: the MoE branch of ``DecoderLayer.__call__``.

``MoELayer(x, residual)`` computes ``residual + T(T(sum_r score_r * v_r) +
v_shared)`` where the router is ``route(x.float() @ gate_weight.T, bias)``
(model.py:385-418, fast_router.py:27-37), with one C-ABI call
(``exlr8_moe_layer``) that runs the router, the trellis experts, the shared
expert and the combine on the current stream.
"""

from __future__ import annotations

import torch

from . import _lib
from .fast_decode import dense_expert, trellis_experts


class MoELayer:
    def __init__(self, gate_weight, bias, experts):
        self.gate_weight = gate_weight.to(torch.float32).contiguous()
        self.bias = bias.to(torch.float32).contiguous()
        self.experts = experts
        if tuple(self.gate_weight.shape) != (256, experts.hidden) or self.bias.numel() != 256:
            raise ValueError("gate weight must be [256, hidden] and bias [256]")
        self._struct, self._count = trellis_experts(experts.packed, experts.scales, experts.k, experts.hidden,
                                                    experts.intermediate)
        self._shared, self._keep = dense_expert(experts.shared)
        self._workspace = None

    def workspace_bytes(self, tokens):
        return int(_lib.lib().exlr8_moe_layer_workspace(tokens, self.experts.hidden, self.experts.intermediate,
                                                        self._count))

    def __call__(self, x, residual, return_routing=False, workspace=None):
        device = _lib.require_cuda(x, residual)
        h = self.experts.hidden
        if x.shape[-1] != h or residual.shape != x.shape:
            raise ValueError("activation width does not match in_features")
        tokens = x.numel() // h
        xr = x.contiguous()
        res = residual.to(x.dtype).contiguous()
        out = torch.empty_like(res)
        ids = torch.empty(tokens, 9, dtype=torch.int32, device=device)
        scores = torch.empty(tokens, 8, dtype=torch.float32, device=device)
        need = self.workspace_bytes(tokens)
        if workspace is None:
            if self._workspace is None or self._workspace.numel() < need or self._workspace.device != device:
                self._workspace = _lib.workspace(need, device)
            workspace = self._workspace
        _lib.check(_lib.lib().exlr8_moe_layer(xr.data_ptr(), _lib.act_code(xr), res.data_ptr(), tokens,
                                              self.gate_weight.data_ptr(), self.bias.data_ptr(), self._struct,
                                              self._shared, out.data_ptr(), ids.data_ptr(), scores.data_ptr(),
                                              workspace.data_ptr(), workspace.numel(),
                                              _lib.stream_handle(device)))
        if return_routing:
            return out, ids.reshape(tuple(x.shape[:-1]) + (9,)), scores.reshape(tuple(x.shape[:-1]) + (8,))
        return out
