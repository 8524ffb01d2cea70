"""Expert-parallel routed MoE layer over one node's GPUs.

The reference runs all 257 experts of a layer on one device
(model.py:385-418).  Across several B200s the routed experts shard
naturally: rank r holds experts [r * E / N, (r + 1) * E / N) and its own
slice of the tokens, and one layer is

    router (local tokens)                      exlr8_router
    dispatch: routed rows -> owner rank        exlr8_ep_dispatch
    all-to-all of rows and local expert ids    NCCL (torch.distributed)
    grouped expert MLP on the received rows    exlr8_expert_mlp (slots = 1)
    all-to-all of the typed slot values back   NCCL
    shared expert on the local tokens          exlr8_shared_expert / trellis
    weighted combine + shared + residual       exlr8_ep_combine

Each slot value comes from the same expert operator (exlr8_expert_mlp on the
owner's rows) and the combine follows the single-device finish order, so the
layer matches the single-device layer within the expert operator's
tolerance (bit-exact when both take the same path).  The exchange uses
a fixed capacity of tokens * 8 rows per destination (no host round trip for
counts); empty rows carry expert id -1 and produce zeros.  Every rank must
pass the same number of tokens.
"""

from __future__ import annotations

import torch

from . import _lib
from .experts import ExpertLayer
from .fast_decode import dense_expert, fast_expert_mlp


def shard_experts(layer: ExpertLayer, rank: int, world: int, routed: int = 256) -> ExpertLayer:
    """The routed experts of `rank` (contiguous blocks of routed / world)."""
    if routed % world:
        raise ValueError("routed experts must divide evenly over the ranks")
    per = routed // world
    lo, hi = rank * per, (rank + 1) * per
    nbytes = layer.expert_bytes
    packed = {p: layer.packed[p][lo * nbytes:hi * nbytes] for p in ("gate", "up", "down")}
    scales = {p: tuple(s[lo:hi] for s in layer.scales[p]) for p in ("gate", "up", "down")}
    return ExpertLayer(packed, scales, layer.k, layer.hidden, layer.intermediate)


def shared_trellis(layer: ExpertLayer, index: int = 256) -> ExpertLayer | None:
    """Trellis matrix `index` (the shared expert) as a one-expert layer, or None."""
    if layer.experts <= index:
        return None
    nbytes = layer.expert_bytes
    packed = {p: layer.packed[p][index * nbytes:(index + 1) * nbytes] for p in ("gate", "up", "down")}
    scales = {p: tuple(s[index:index + 1] for s in layer.scales[p]) for p in ("gate", "up", "down")}
    return ExpertLayer(packed, scales, layer.k, layer.hidden, layer.intermediate)


class Exchange:
    """Equal-split all-to-all over dim 0 of [world, ...] tensors.  Several
    tensors go in one grouped set of NCCL sends and receives."""

    def __init__(self, world: int, group=None, rank: int = 0):
        self.world, self.group, self.rank = world, group, rank

    def __call__(self, *tensors: torch.Tensor):
        if self.world == 1:
            return tensors[0] if len(tensors) == 1 else tensors
        import torch.distributed as dist

        outs = [torch.empty_like(t) for t in tensors]
        if len(tensors) == 1:
            dist.all_to_all_single(outs[0], tensors[0].contiguous(), group=self.group)
            return outs[0]
        ops = []
        for t, o in zip(tensors, outs):
            t = t.contiguous()
            for peer in range(self.world):
                if peer == self.rank:
                    o[peer].copy_(t[peer])
                    continue
                gpeer = peer if self.group is None else dist.get_global_rank(self.group, peer)
                ops.append(dist.P2POp(dist.isend, t[peer], gpeer, self.group))
                ops.append(dist.P2POp(dist.irecv, o[peer], gpeer, self.group))
        for work in dist.batch_isend_irecv(ops):
            work.wait()
        return tuple(outs)


class ExpertParallelMoE:
    """One MoE layer with this rank's routed shard (`local`, from
    shard_experts) and a replicated shared expert: the dense bf16 triple
    `shared`, or the one-expert trellis layer `shared_layer`."""

    def __init__(self, gate_weight, bias, local: ExpertLayer, rank: int, world: int, group=None, shared=None,
                 shared_layer: ExpertLayer | None = None, routed: int = 256):
        if (shared is None) == (shared_layer is None):
            raise ValueError("give exactly one shared expert (dense bf16 or trellis)")
        if routed % world or local.experts != routed // world:
            raise ValueError("the local shard must hold routed / world experts")
        self.gate_weight = gate_weight.to(torch.float32).contiguous()
        self.bias = bias.to(torch.float32).contiguous()
        self.local, self.rank, self.world = local, rank, world
        self.per_rank = routed // world
        self.shared = None if shared is None else tuple(t.contiguous() for t in shared)
        self.shared_layer = shared_layer
        self.exchange = Exchange(world, group, rank)
        self._side = None
        self._shared_struct = None
        if self.shared is not None:
            self._shared_struct, self._keep = dense_expert(self.shared)

    def shared_values(self, x):
        """Typed shared-expert output [tokens][hidden] of the local tokens."""
        h = x.shape[-1]
        tokens = x.shape[0]
        if self.shared_layer is not None:
            ids = torch.zeros(tokens, 1, dtype=torch.int32, device=x.device)
            return self.shared_layer(x, ids).reshape(tokens, h)
        lib = _lib.lib()
        m = self.shared[0].shape[0]
        out = torch.empty(tokens, h, dtype=x.dtype, device=x.device)
        ws = _lib.workspace(lib.exlr8_shared_expert_workspace(tokens, h, m), x.device)
        _lib.check(lib.exlr8_shared_expert(x.data_ptr(), _lib.act_code(x), tokens, h, m, self._shared_struct,
                                           out.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_handle(x.device)))
        return out

    def route(self, xr):
        """(ids [tokens][9], scores [tokens][8]) of the local tokens."""
        from .fast_router import route, router, router_logits

        if xr.shape[0] >= 64:  # the prefill gate product on the tensor cores
            return route(router_logits(xr, self.gate_weight), self.bias)
        _, ids, scores = router(xr, self.gate_weight, self.bias)
        return ids, scores

    def __call__(self, x, residual, return_routing=False):
        device = _lib.require_cuda(x, residual)
        h = self.local.hidden
        tokens = x.numel() // h
        xr = x.reshape(tokens, h).contiguous()
        res = residual.reshape(tokens, h).to(x.dtype).contiguous()
        ids, scores = self.route(xr)
        lib = _lib.lib()
        stream = _lib.stream_handle(device)
        cap = tokens * 8
        send_x = torch.empty(self.world, cap, h, dtype=x.dtype, device=device)
        send_meta = torch.empty(self.world, cap, dtype=torch.int32, device=device)
        slot_pos = torch.empty(max(tokens * 8, 1), dtype=torch.int32, device=device)
        counts = torch.empty(self.world, dtype=torch.int32, device=device)
        status = torch.zeros(1, dtype=torch.int32, device=device)
        _lib.check(lib.exlr8_ep_dispatch(ids.data_ptr(), tokens, xr.data_ptr(), _lib.act_code(xr), h, self.world,
                                         self.per_rank, cap, send_x.data_ptr(), send_meta.data_ptr(),
                                         slot_pos.data_ptr(), counts.data_ptr(), status.data_ptr(), stream))
        # The replicated shared expert runs on a side stream, overlapping the
        # exchange and the owner's expert products.
        main = torch.cuda.current_stream(device)
        if self._side is None or self._side.device != device:
            self._side = torch.cuda.Stream(device)
        self._side.wait_stream(main)
        with torch.cuda.stream(self._side):
            shared = self.shared_values(xr)
        recv_x, recv_meta = self.exchange(send_x, send_meta)
        rows = self.world * cap
        local = self.local
        values = fast_expert_mlp(recv_x.reshape(rows, h), recv_meta.reshape(rows, 1), local.packed, local.scales,
                                 local.k, h, local.intermediate)
        back = self.exchange(values.reshape(self.world, cap, h))
        main.wait_stream(self._side)
        shared.record_stream(main)
        out = torch.empty_like(res)
        _lib.check(lib.exlr8_ep_combine(back.data_ptr(), _lib.act_code(xr), slot_pos.data_ptr(), scores.data_ptr(),
                                        shared.data_ptr(), res.data_ptr(), tokens, h, out.data_ptr(), stream))
        out = out.reshape(residual.shape)
        if return_routing:
            return out, ids, scores
        return out
