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
        self._graphs = {}

    def workspace_bytes(self, tokens):
        return int(_lib.lib().exlr8_moe_layer_workspace(tokens, self.experts.hidden, self.experts.intermediate,
                                                        self._count))

    def _launch(self, xr, res, out, ids, scores, workspace, tokens, device, out_ptr=None):
        # out_ptr: the device-accessible address of a page-locked host `out`,
        # which the finishing kernel then writes over PCIe.
        _lib.check(_lib.lib().exlr8_moe_layer(xr.data_ptr(), _lib.act_code(xr), res.data_ptr(), tokens,
                                              self.gate_weight.data_ptr(), self.bias.data_ptr(), self._struct,
                                              self._shared, out.data_ptr() if out_ptr is None else out_ptr,
                                              ids.data_ptr(), scores.data_ptr(), workspace.data_ptr(),
                                              workspace.numel(), _lib.stream_handle(device)))

    def _stage_in(self, x, residual, xd, rd, device):
        """x and residual (page-locked host) into xd and rd by the library's
        staging kernel, the first launch of the layer's chain."""
        _lib.check(_lib.lib().exlr8_stage_in(x.data_ptr(), xd.data_ptr(), residual.data_ptr(), rd.data_ptr(),
                                             x.numel() * x.element_size(), _lib.stream_handle(device)))

    def _host_operands(self, x, residual, out):
        """Checks of the host-buffer modes; returns (out, tokens)."""
        h = self.experts.hidden
        if x.shape[-1] != h or residual.shape != x.shape or (out is not None and out.shape != x.shape):
            raise ValueError("host buffers take x, residual and out of one shape [..., hidden]")
        if out is None:
            out = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        if not all(t.device.type == "cpu" and t.is_pinned() and t.is_contiguous() and t.dtype == x.dtype
                   for t in (x, residual, out)):
            raise ValueError("host buffers must be contiguous page-locked (pinned) tensors of one dtype")
        _lib.act_code(x)
        return out, x.numel() // h

    def __call__(self, x, residual, return_routing=False, workspace=None, out=None, graph=False):
        """``residual + moe(x)``.  ``out`` (optional) receives the result.

        ``graph=True`` (with ``out``): the layer's kernel chain is captured
        once per (x, residual, out) address triple into a CUDA graph and
        replayed on later calls -- one launch for the seven kernels, the
        B200 counterpart of the reference's ``mx.compile`` of the decode
        finish (fast_decode.py:224-244).  x and residual must then be
        contiguous and of one dtype (their contents may change between
        calls, not their addresses); the routing ids and scores live in
        buffers of the captured call, overwritten by every replay.  In this
        mode x, residual and out may also be pinned host tensors.

        Pinned host x and residual (both modes): the layer's first kernel
        reads them over PCIe into device buffers and its finishing kernel
        writes the result straight into ``out`` (a pinned host tensor, made
        here when not given), so no copy-engine transfer sits between the
        launches.  ``out`` is written asynchronously on the current stream:
        synchronise it before reading the result on the host.  The routing
        ids and scores are device tensors."""
        if x.device.type == "cpu":
            if graph:
                return self._graph_call_host(x, residual, out, return_routing)
            return self._host_call(x, residual, out, return_routing, workspace)
        device = _lib.require_cuda(x, residual)
        h = self.experts.hidden
        if x.shape[-1] != h or residual.shape != x.shape:
            raise ValueError("activation width does not match in_features")
        tokens = x.numel() // h
        xr = x.contiguous()
        res = residual.to(x.dtype).contiguous()
        if out is None:
            out = torch.empty_like(res)
        elif out.shape != residual.shape or out.dtype != x.dtype or not out.is_contiguous() or out.device != device:
            raise ValueError("out must be a contiguous tensor like the residual in x's dtype")
        if graph:
            if xr is not x or res is not residual or workspace is not None:
                raise ValueError("graph=True takes contiguous x and residual of one dtype and no workspace")
            return self._graph_call(xr, res, out, tokens, device, return_routing, x.shape[:-1])
        ids = torch.empty(tokens, 9, dtype=torch.int32, device=device)
        scores = torch.empty(tokens, 8, dtype=torch.float32, device=device)
        need = self.workspace_bytes(tokens)
        if workspace is None:
            if self._workspace is None or self._workspace.numel() < need or self._workspace.device != device:
                self._workspace = _lib.workspace(need, device)
            workspace = self._workspace
        self._launch(xr, res, out, ids, scores, workspace, tokens, device)
        if return_routing:
            return out, ids.reshape(tuple(x.shape[:-1]) + (9,)), scores.reshape(tuple(x.shape[:-1]) + (8,))
        return out

    def _graph_call(self, xr, res, out, tokens, device, return_routing, lead_shape):
        key = (xr.data_ptr(), res.data_ptr(), out.data_ptr(), tokens, xr.dtype, device)
        entry = self._graphs.get(key)
        if entry is None:
            # Its own workspace and routing buffers: the graph holds their
            # addresses.  The first call runs eagerly (the result of this call,
            # and the library's one-time launch setup), then is captured.
            ids = torch.empty(tokens, 9, dtype=torch.int32, device=device)
            scores = torch.empty(tokens, 8, dtype=torch.float32, device=device)
            ws = _lib.workspace(self.workspace_bytes(tokens), device)
            self._launch(xr, res, out, ids, scores, ws, tokens, device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._launch(xr, res, out, ids, scores, ws, tokens, device)
            entry = (g, ids, scores, ws)
            self._graphs[key] = entry
        else:
            entry[0].replay()
        if return_routing:
            return out, entry[1].reshape(tuple(lead_shape) + (9,)), entry[2].reshape(tuple(lead_shape) + (8,))
        return out

    def _host_call(self, x, residual, out, return_routing, workspace):
        out, tokens = self._host_operands(x, residual, out)
        device = self.gate_weight.device
        xd = torch.empty(x.shape, dtype=x.dtype, device=device)
        rd = torch.empty_like(xd)
        ids = torch.empty(tokens, 9, dtype=torch.int32, device=device)
        scores = torch.empty(tokens, 8, dtype=torch.float32, device=device)
        need = self.workspace_bytes(tokens)
        if workspace is None:
            if self._workspace is None or self._workspace.numel() < need or self._workspace.device != device:
                self._workspace = _lib.workspace(need, device)
            workspace = self._workspace
        self._stage_in(x, residual, xd, rd, device)
        self._launch(xd, rd, out, ids, scores, workspace, tokens, device, out_ptr=_lib.host_device_pointer(out))
        if return_routing:
            lead = tuple(x.shape[:-1])
            return out, ids.reshape(lead + (9,)), scores.reshape(lead + (8,))
        return out

    def _graph_call_host(self, x, residual, out, return_routing):
        if out is None:
            raise ValueError("host graph mode takes an out tensor (the graph holds its address)")
        out, tokens = self._host_operands(x, residual, out)
        device = self.gate_weight.device
        key = ("host", x.data_ptr(), residual.data_ptr(), out.data_ptr(), tokens, x.dtype, device)
        entry = self._graphs.get(key)
        if entry is None:
            xd = torch.empty(x.shape, dtype=x.dtype, device=device)
            rd = torch.empty_like(xd)
            ids = torch.empty(tokens, 9, dtype=torch.int32, device=device)
            scores = torch.empty(tokens, 8, dtype=torch.float32, device=device)
            ws = _lib.workspace(self.workspace_bytes(tokens), device)
            out_ptr = _lib.host_device_pointer(out)

            def body():
                self._stage_in(x, residual, xd, rd, device)
                self._launch(xd, rd, out, ids, scores, ws, tokens, device, out_ptr=out_ptr)

            body()  # this call's result, and the library's one-time launch setup
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                body()
            entry = (g, ids, scores, (ws, xd, rd))
            self._graphs[key] = entry
        else:
            entry[0].replay()
        if return_routing:
            lead = tuple(x.shape[:-1])
            return out, entry[1].reshape(lead + (9,)), entry[2].reshape(lead + (8,))
        return out

    def clear_graphs(self):
        """Release the captured graphs (and their buffers)."""
        self._graphs.clear()
