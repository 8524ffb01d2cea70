"""Resident four-bit experts with joined gate/up: ``exlr8.joined_mxfp4`` on B200.

The reference builds ``JoinedMXFP4(expert)`` by re-encoding trellis experts
to MXFP4 at load time (joined_mxfp4.py:12-47) and then runs MLX
``gather_qmm(mode="mxfp4")`` products (joined_mxfp4.py:90-134).  Here
``encode(expert)`` re-encodes on the GPU (one fused decode + in-scale fold +
quantise launch per projection, ``exlr8_mxfp4_encode_trellis``) into the
``weights`` dictionary of the reference:
``{"gate_up": (codes, scales, None), "down": (codes, scales, None)}`` with
uint32 codes (held as int32 bits), eight E2M1 values per word, low nibble
first, and E8M0 scales per 32 inputs.  ``JoinedMXFP4(expert)`` encodes;
``JoinedMXFP4(unit, weights, scales, hidden, intermediate)`` takes weights
already encoded.  Every product runs as a grouped block-scaled tcgen05 GEMM
in ``libexlr8_b200.so``:

* ``slots(x, ids)`` -> ``[*ids.shape, hidden]`` per-slot expert outputs in
  ``x.dtype`` (joined_mxfp4.py:147-150);
* ``finish(x, ids, scores, residual)`` -> the routing-weighted combine with
  the shared slot 8 and the residual (joined_mxfp4.py:152-163).

``JoinedMoELayer`` adds the router in front (the MoE branch of
``DecoderLayer``, model.py:385-418) for prefill-size batches.
"""

from __future__ import annotations

import torch

from . import _lib


def _prepare(scales: torch.Tensor, rows: int, in_features: int, device) -> torch.Tensor:
    """E8M0 [rows, in/32] -> the 512-byte block layout of the GEMM."""
    src = scales.reshape(rows, in_features // 32).contiguous()
    out = torch.empty(int(_lib.lib().exlr8_mxfp4_prepared_scales_bytes(rows, in_features)), dtype=torch.uint8,
                      device=device)
    _lib.check(_lib.lib().exlr8_mxfp4_prepare_scales(src.data_ptr(), rows, in_features, out.data_ptr(),
                                                     _lib.stream_handle(device)))
    return out


def encode(expert):
    """``encode(expert)`` (joined_mxfp4.py:12-47) on the GPU -> (unit, weights).

    ``expert`` is a resident trellis layer (``ExpertLayer``: ``packed``,
    ``scales``, ``k``, ``hidden``, ``intermediate``).  ``unit`` is the sign of
    matrix 0's gate in-scale, shape [1, hidden] in the scale dtype
    (joined_mxfp4.py:13).  Every matrix of each projection is decoded
    (decode.metal), gate/up rows multiplied by ``in_scale[e] * unit``
    (joined_mxfp4.py:22,30-31) and quantised transposed with MLX's mxfp4 rule;
    gate rows land at 0..m-1 and up rows at m..2m-1 of the joined
    [E, 2m, h/8] buffer (joined_mxfp4.py:41-45)."""
    packed = expert.packed
    device = _lib.require_cuda(packed["gate"], packed["up"], packed["down"])
    h, m, k = expert.hidden, expert.intermediate, expert.k
    matrices = packed["gate"].numel() // (h * m * k // 8)
    gate_in = expert.scales["gate"][0]
    unit = torch.sign(gate_in[:1]).contiguous()
    weights = {
        "gate_up": (torch.empty(matrices, 2 * m, h // 8, dtype=torch.int32, device=device),
                    torch.empty(matrices, 2 * m, h // 32, dtype=torch.uint8, device=device), None),
        "down": (torch.empty(matrices, h, m // 8, dtype=torch.int32, device=device),
                 torch.empty(matrices, h, m // 32, dtype=torch.uint8, device=device), None),
    }
    stream = _lib.stream_handle(device)
    for projection, offset in (("gate", 0), ("up", m), ("down", 0)):
        incoming, outgoing, side = (m, h, 2) if projection == "down" else (h, m, 1)
        codes, sc, _ = weights["down" if projection == "down" else "gate_up"]
        src = packed[projection].contiguous()
        in_scale = unit_arg = None
        code = 0
        if side == 1:
            in_scale = expert.scales[projection][0].contiguous()
            if tuple(in_scale.shape) != (matrices, incoming):
                raise ValueError("expert side vectors must contain full signed channel scales")
            unit_arg = unit.to(in_scale.dtype).contiguous()
            code = _lib.scale_code(in_scale)
        _lib.check(_lib.lib().exlr8_mxfp4_encode_trellis(
            src.data_ptr(), src.numel(), k, incoming, outgoing, side,
            in_scale.data_ptr() if in_scale is not None else None,
            unit_arg.data_ptr() if unit_arg is not None else None, code, codes.data_ptr(), sc.data_ptr(),
            codes.shape[1], offset, stream))
    return unit, weights


def quantize(w):
    """MLX ``quantize(w, mode="mxfp4")`` of float32 rows w [..., k] ->
    (codes [..., k/8] int32 bits of uint32, scales [..., k/32] uint8)."""
    device = _lib.require_cuda(w)
    k = w.shape[-1]
    src = w.to(torch.float32).contiguous()
    rows = src.numel() // k if k else 0
    codes = torch.empty(tuple(w.shape[:-1]) + (k // 8,), dtype=torch.int32, device=device)
    scales = torch.empty(tuple(w.shape[:-1]) + (k // 32,), dtype=torch.uint8, device=device)
    _lib.check(_lib.lib().exlr8_mxfp4_quantize(src.data_ptr(), rows, k, codes.data_ptr(), scales.data_ptr(),
                                               _lib.stream_handle(device)))
    return codes, scales


class JoinedMXFP4:
    """``JoinedMXFP4(expert)`` re-encodes a resident trellis layer
    (joined_mxfp4.py:137-141); ``JoinedMXFP4(unit, weights, scales, hidden,
    intermediate)`` takes ``unit`` [hidden] and ``weights`` as above and the
    expert scale dictionary (only ``scales["gate"][1]``, ``scales["up"][1]``,
    ``scales["down"][0]`` and ``scales["down"][1]`` are read, as in the
    reference's joined path)."""

    def __init__(self, unit, weights=None, scales=None, hidden: int | None = None, intermediate: int | None = None):
        if weights is None:
            expert = unit
            unit, weights = encode(expert)
            scales, hidden, intermediate = expert.scales, expert.hidden, expert.intermediate
        codes_gu, scales_gu = weights["gate_up"][0], weights["gate_up"][1]
        codes_d, scales_d = weights["down"][0], weights["down"][1]
        device = _lib.require_cuda(unit, codes_gu, scales_gu, codes_d, scales_d)
        experts = codes_gu.shape[0]
        h, m = hidden, intermediate
        if tuple(codes_gu.shape) != (experts, 2 * m, h // 8) or tuple(codes_d.shape) != (experts, h, m // 8):
            raise ValueError("joined MXFP4 codes must be [E, 2m, h/8] and [E, h, m/8] uint32")
        if tuple(scales_gu.shape) != (experts, 2 * m, h // 32) or tuple(scales_d.shape) != (experts, h, m // 32):
            raise ValueError("joined MXFP4 scales must be [E, 2m, h/32] and [E, h, m/32] uint8")
        self.unit = unit.reshape(-1).contiguous()
        self.weights = weights
        self.hidden, self.intermediate, self.experts = h, m, experts
        side = scales["gate"][1]
        self._keep = [
            codes_gu.contiguous(), _prepare(scales_gu, experts * 2 * m, h, device),
            codes_d.contiguous(), _prepare(scales_d, experts * h, m, device), self.unit,
            scales["gate"][1].to(side.dtype).contiguous(), scales["up"][1].to(side.dtype).contiguous(),
            scales["down"][0].to(side.dtype).contiguous(), scales["down"][1].to(side.dtype).contiguous(),
        ]
        if self.unit.dtype != side.dtype:
            self._keep[4] = self.unit.to(side.dtype).contiguous()
        st = _lib.JoinedMXFP4Weights()
        (st.gate_up, st.gate_up_scales, st.down, st.down_scales, st.unit, st.gate_out, st.up_out, st.down_in,
         st.down_out) = [t.data_ptr() for t in self._keep]
        st.scale_dtype = _lib.scale_code(side)
        st.experts, st.hidden, st.intermediate = experts, h, m
        self._struct = st
        self._workspace = None

    def _ws(self, tokens, slots, device, extra=0):
        need = int(_lib.lib().exlr8_joined_workspace(tokens, slots, self.hidden, self.intermediate,
                                                     self.experts)) + extra
        if self._workspace is None or self._workspace.numel() < need or self._workspace.device != device:
            self._workspace = _lib.workspace(need, device)
        return self._workspace

    def slots(self, x, ids):
        device = _lib.require_cuda(x, ids)
        h = self.hidden
        slots = ids.shape[-1]
        ids_flat = ids.reshape(-1, slots).to(torch.int32).contiguous()
        tokens = ids_flat.shape[0]
        if x.shape[-1] != h or x.numel() // h != tokens:
            raise ValueError("activation rows do not match the expert indices")
        xr = x.reshape(tokens, h).contiguous()
        out = torch.empty(tokens, slots, h, dtype=x.dtype, device=device)
        ws = self._ws(tokens, slots, device)
        _lib.check(_lib.lib().exlr8_joined_slots(xr.data_ptr(), _lib.act_code(xr), ids_flat.data_ptr(), tokens, slots,
                                                 self._struct, out.data_ptr(), ws.data_ptr(), ws.numel(),
                                                 _lib.stream_handle(device)))
        return out.reshape(tuple(ids.shape) + (h,))

    def finish(self, x, ids, scores, residual):
        device = _lib.require_cuda(x, ids, scores, residual)
        h = self.hidden
        if ids.shape[-1] != 9 or scores.shape[-1] != 8:
            raise ValueError("finish takes nine slot ids and eight routing scores per token")
        tokens = ids.numel() // 9
        if x.numel() // h != tokens or residual.numel() // h != tokens:
            raise ValueError("activation rows do not match the expert indices")
        xr = x.reshape(tokens, h).contiguous()
        res = residual.reshape(tokens, h).to(residual.dtype).contiguous()
        ids_flat = ids.reshape(tokens, 9).to(torch.int32).contiguous()
        sc = scores.reshape(tokens, 8).to(torch.float32).contiguous()
        out = torch.empty(tokens, h, dtype=residual.dtype, device=device)
        if res.dtype != xr.dtype:
            raise ValueError("residual and activations must share a dtype")
        ws = self._ws(tokens, 9, device)
        _lib.check(_lib.lib().exlr8_joined_finish(xr.data_ptr(), _lib.act_code(xr), ids_flat.data_ptr(),
                                                  sc.data_ptr(), res.data_ptr(), tokens, self._struct,
                                                  out.data_ptr(), ws.data_ptr(), ws.numel(),
                                                  _lib.stream_handle(device)))
        return out.reshape(residual.shape)

    def dispatch_header(self, tokens: int, slots: int = 9):
        """[chunks, padded rows, unit counter, unit counter, GEMM error] of the last call."""
        return dispatch_header(self._workspace, tokens, slots, self.experts)


def dispatch_header(workspace: torch.Tensor, tokens: int, slots: int, experts: int):
    """Device dispatch header of the last joined call that used ``workspace``:
    [chunks, padded rows, gate/up unit counter, down unit counter, GEMM error
    code (0 = none)]."""
    header = torch.zeros(8, dtype=torch.int32)
    _lib.check(_lib.lib().exlr8_joined_status(workspace.data_ptr(), tokens, slots, experts, header.data_ptr(),
                                              _lib.stream_handle(workspace.device)))
    return header.tolist()[:5]


class JoinedMoELayer:
    """Router + ``JoinedMXFP4.finish`` in one C-ABI call (``exlr8_joined_moe_layer``)."""

    def __init__(self, gate_weight, bias, joined: JoinedMXFP4):
        self.gate_weight = gate_weight.to(torch.float32).contiguous()
        self.bias = bias.to(torch.float32).contiguous()
        self.joined = joined
        if tuple(self.gate_weight.shape) != (256, joined.hidden) or self.bias.numel() != 256:
            raise ValueError("gate weight must be [256, hidden] and bias [256]")
        self._workspace = None

    def dispatch_header(self, tokens: int):
        return dispatch_header(self._workspace, tokens, 9, self.joined.experts)

    def workspace_bytes(self, tokens):
        j = self.joined
        return int(_lib.lib().exlr8_joined_moe_layer_workspace(tokens, j.hidden, j.intermediate, j.experts))

    def __call__(self, x, residual, return_routing=False, workspace=None):
        device = _lib.require_cuda(x, residual)
        h = self.joined.hidden
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
        _lib.check(_lib.lib().exlr8_joined_moe_layer(xr.data_ptr(), _lib.act_code(xr), res.data_ptr(), tokens,
                                                     self.gate_weight.data_ptr(), self.bias.data_ptr(),
                                                     self.joined._struct, out.data_ptr(), ids.data_ptr(),
                                                     scores.data_ptr(), workspace.data_ptr(), workspace.numel(),
                                                     _lib.stream_handle(device)))
        if return_routing:
            return out, ids.reshape(tuple(x.shape[:-1]) + (9,)), scores.reshape(tuple(x.shape[:-1]) + (8,))
        return out
