"""Fused router (mirror of ``exlr8/fast_router.py``).

``route`` is the sigmoid + bias top-8 with renormalisation times 2.5 and the
shared expert id 256 appended (fast_router.metal:1-42); ``combine`` is the
weighted sum of per-slot expert outputs with the shared expert and the
residual (model.py:415-418).  ``router`` adds the
float32 gate GEMV in front (model.py:366-371).  ``compiled_finish`` returns
the whole MoE-layer call ``(x, residual) -> residual + moe(x)``
(fast_router.py:27-37).  Indices are returned as int32 (torch's uint32
support is limited); uint32 and int32 indices are both accepted as inputs.
"""

from __future__ import annotations

import torch

from . import _lib


def route(logits: torch.Tensor, bias: torch.Tensor):
    """``(indices [..., 9] int32, scores [..., 8] float32)`` for 256-wide logits."""
    device = _lib.require_cuda(logits, bias)
    if logits.shape[-1] != 256 or bias.numel() != 256:
        raise ValueError("the fused router takes 256 expert logits")
    rows = logits.numel() // 256
    values = logits.to(torch.float32).contiguous()
    correction = bias.to(torch.float32).contiguous()
    ids = torch.empty(tuple(logits.shape[:-1]) + (9,), dtype=torch.int32, device=device)
    scores = torch.empty(tuple(logits.shape[:-1]) + (8,), dtype=torch.float32, device=device)
    _lib.check(_lib.lib().exlr8_route(values.data_ptr(), correction.data_ptr(), rows, ids.data_ptr(),
                                      scores.data_ptr(), _lib.stream_handle(device)))
    return ids, scores


def combine(values: torch.Tensor, scores: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
    """``residual + T(T(sum_r values[..., r, :] * scores[..., r]) + values[..., 8, :])``
    (model.py:415-418) for per-slot expert outputs ``values [..., 9, h]`` in
    the residual's dtype (slot 8 the shared expert), the routed sum in
    float32 in the order of metal/fast_decode_finish_fused.metal:52-57."""
    device = _lib.require_cuda(values, scores, residual)
    h = residual.shape[-1]
    if values.shape[-2:] != (9, h) or values.dtype != residual.dtype:
        raise ValueError("values must be [..., 9, hidden] in the residual's dtype")
    tokens = residual.numel() // h
    if scores.numel() != tokens * 8:
        raise ValueError("scores must be [..., 8]")
    v = values.contiguous()
    sc = scores.to(torch.float32).contiguous()
    res = residual.contiguous()
    out = torch.empty_like(res)
    _lib.check(_lib.lib().exlr8_combine(v.data_ptr(), sc.data_ptr(), res.data_ptr(), tokens, h, _lib.act_code(res),
                                        out.data_ptr(), _lib.stream_handle(device)))
    return out


def router(x: torch.Tensor, gate_weight: torch.Tensor, bias: torch.Tensor):
    """``(logits, indices, scores)``: ``route(x.float() @ gate_weight.T, bias)`` on the GPU."""
    device = _lib.require_cuda(x, gate_weight, bias)
    hidden = x.shape[-1]
    if tuple(gate_weight.shape) != (256, hidden):
        raise ValueError("gate weight must be [256, hidden]")
    tokens = x.numel() // hidden
    x = x.contiguous()
    w = gate_weight.to(torch.float32).contiguous()
    b = bias.to(torch.float32).contiguous()
    logits = torch.empty(tuple(x.shape[:-1]) + (256,), dtype=torch.float32, device=device)
    ids = torch.empty(tuple(x.shape[:-1]) + (9,), dtype=torch.int32, device=device)
    scores = torch.empty(tuple(x.shape[:-1]) + (8,), dtype=torch.float32, device=device)
    _lib.check(_lib.lib().exlr8_router(x.data_ptr(), _lib.act_code(x), tokens, hidden, w.data_ptr(), b.data_ptr(),
                                       logits.data_ptr(), ids.data_ptr(), scores.data_ptr(),
                                       _lib.stream_handle(device)))
    return logits, ids, scores


def router_logits(x: torch.Tensor, gate_weight: torch.Tensor) -> torch.Tensor:
    """``x.float() @ gate_weight.T`` on the tensor cores (the prefill gate product)."""
    device = _lib.require_cuda(x, gate_weight)
    hidden = x.shape[-1]
    if tuple(gate_weight.shape) != (256, hidden):
        raise ValueError("gate weight must be [256, hidden]")
    tokens = x.numel() // hidden
    x = x.contiguous()
    w = gate_weight.to(torch.float32).contiguous()
    logits = torch.empty(tuple(x.shape[:-1]) + (256,), dtype=torch.float32, device=device)
    ws = _lib.workspace(_lib.lib().exlr8_router_logits_workspace(tokens, hidden, _lib.act_code(x)), device)
    _lib.check(_lib.lib().exlr8_router_logits(x.data_ptr(), _lib.act_code(x), tokens, hidden, w.data_ptr(),
                                              logits.data_ptr(), ws.data_ptr(), ws.numel(),
                                              _lib.stream_handle(device)))
    return logits


def compiled_finish(experts, gate, bias):
    """Return ``call(x, residual) -> residual + routed + shared`` for one layer.

    ``experts`` is a :class:`mlxlr8_b200.experts.ExpertLayer` (its optional
    ``shared`` dense bf16 expert is used when present); ``gate`` is the float32
    gate weight ``[256, hidden]`` or an object with a ``weight`` attribute.
    """
    from .moe import MoELayer

    weight = getattr(gate, "weight", gate)
    layer = MoELayer(weight, bias, experts)

    def call(x, residual):
        return layer(x, residual)

    return call
