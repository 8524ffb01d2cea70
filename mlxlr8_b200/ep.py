"""Expert-parallel routed MoE layer over one node's GPUs.

The reference runs all 257 experts of a layer on one device
(model.py:385-418).  Across several B200s the routed experts shard
naturally: rank r holds experts [r * E / N, (r + 1) * E / N) and its own
slice of the tokens, and one layer is

    router (local tokens)                      exlr8_router
    dispatch: routed rows -> owner rank        exlr8_ep_dispatch
    all-to-all of rows and local expert ids    NCCL (torch.distributed)
    grouped expert MLP on the received rows,   exlr8_expert_mlp_shared (the bf16
      and the shared expert on the local        shared expert's rows stream inside
      tokens                                    the trellis kernels)
    all-to-all of the typed slot values back   NCCL
    weighted combine + shared + residual       exlr8_ep_combine

With a trellis shared expert the received rows go through exlr8_expert_mlp
and the shared expert runs on a side stream.

Each slot value comes from the same expert operator (exlr8_expert_mlp on the
owner's rows) and the combine follows the single-device finish order, so the
layer matches the single-device layer within the expert operator's
tolerance (bit-exact when both take the same path).  The exchange uses
a fixed capacity of tokens * 8 rows per destination (no host round trip for
counts); empty rows carry expert id -1 and produce zeros.  Every rank must
pass the same number of tokens.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .experts import ExpertLayer
from .fast_decode import dense_expert, fast_expert_mlp, trellis_experts


def seeded_placement(seed: int, routed: int = 256, device="cuda") -> torch.Tensor:
    """A seeded permutation of the routed experts over the ranks:
    ``placement[e]`` is expert e's position in the rank-major order, so rank
    r owns the experts placed at [r * per, (r + 1) * per).  Under skewed
    (Zipf) routing it spreads the popular experts over the ranks instead of
    leaving the lowest ids on rank 0."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return torch.randperm(routed, generator=g).to(device=device, dtype=torch.int32)


def _owned(rank: int, world: int, routed: int, placement: torch.Tensor | None) -> list[int]:
    per = routed // world
    if placement is None:
        return list(range(rank * per, (rank + 1) * per))
    order = torch.argsort(placement.to("cpu", torch.int64)).tolist()  # position -> expert
    return order[rank * per:(rank + 1) * per]


def shard_experts(layer: ExpertLayer, rank: int, world: int, routed: int = 256,
                  placement: torch.Tensor | None = None) -> ExpertLayer:
    """The routed experts of `rank`: contiguous blocks of routed / world, or
    with `placement` (``seeded_placement``) the experts placed at this rank's
    positions, in position order."""
    if routed % world:
        raise ValueError("routed experts must divide evenly over the ranks")
    if placement is not None and sorted(placement.tolist()) != list(range(routed)):
        raise ValueError("placement must be a permutation of the routed experts")
    owned = _owned(rank, world, routed, placement)
    nbytes = layer.expert_bytes
    if placement is None:
        lo, hi = owned[0], owned[-1] + 1
        packed = {p: layer.packed[p][lo * nbytes:hi * nbytes] for p in ("gate", "up", "down")}
        scales = {p: tuple(s[lo:hi] for s in layer.scales[p]) for p in ("gate", "up", "down")}
    else:
        idx = torch.tensor(owned, dtype=torch.int64, device=layer.packed["gate"].device)
        packed = {p: torch.cat([layer.packed[p][e * nbytes:(e + 1) * nbytes] for e in owned])
                  for p in ("gate", "up", "down")}
        scales = {p: tuple(s.index_select(0, idx.to(s.device)) for s in layer.scales[p]) for p in ("gate", "up", "down")}
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


class PeerExchange:
    """The peer-memory exchange of one expert-parallel layer
    (exlr8_ep_send / exlr8_ep_return): this rank's region, mapped by every
    other rank through CUDA IPC, and theirs mapped here.  Construction is a
    collective over `group` (the IPC handles are all-gathered); every rank
    must then make the same calls with the same token count, at most
    `max_tokens` per call."""

    def __init__(self, world: int, rank: int, hidden: int, max_tokens: int, dtype: torch.dtype,
                 device: torch.device, group=None):
        import torch.distributed as dist

        lib = _lib.lib()
        self.world, self.rank, self.hidden = world, rank, hidden
        self.code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[dtype]
        self.max_capacity = max_tokens * 8
        nbytes = lib.exlr8_ep_peer_bytes(world, self.max_capacity, hidden, self.code)
        if nbytes == 0:
            raise ValueError("unsupported peer-exchange shape")
        region = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        _lib.check(lib.exlr8_ep_peer_create(nbytes, ctypes.byref(region), handle))
        self.region = region.value
        self._opened = []
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
        handles = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(handles, mine, group=group)
        addrs = []
        for r in range(world):
            if r == rank:
                addrs.append(self.region)
                continue
            theirs = (ctypes.c_ubyte * 64).from_buffer_copy(bytes(handles[r].cpu().tolist()))
            ptr = ctypes.c_void_p()
            _lib.check(lib.exlr8_ep_peer_open(theirs, ctypes.byref(ptr)))
            self._opened.append(ptr.value)
            addrs.append(ptr.value)
        self.peers = torch.tensor(addrs, dtype=torch.int64, device=device)
        meta, rows, back = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
        _lib.check(lib.exlr8_ep_peer_offsets(world, self.max_capacity, hidden, self.code, ctypes.byref(meta),
                                             ctypes.byref(rows), ctypes.byref(back)))
        self.meta, self.rows, self.back = self.region + meta.value, self.region + rows.value, self.region + back.value
        self.status = torch.zeros(2, dtype=torch.int32, device=device)
        self._status_host = torch.zeros(2, dtype=torch.int32).pin_memory()
        self._status_event = None
        self._group = group
        self.broken = False

    def check(self):
        """Raise if the last exchange lost slots or a wait for a peer timed out
        (synchronises the status word to the host).

        After a timeout the ranks' epoch flags no longer agree, so the
        exchange is marked unusable: later calls raise until it is closed and
        a new one is created."""
        self._raise_for(self.status.cpu())

    def check_deferred(self):
        """The check of an earlier call, without synchronising: the status
        word (cumulative over the exchange's life) is copied to pinned host
        memory behind an event; once a copy has landed its value is checked
        and a new copy is queued.  An error surfaces a call or two after it
        happened."""
        ev = self._status_event
        if ev is not None and ev.query():
            self._status_event = None
            self._raise_for(self._status_host)
        if self._status_event is None:
            self._status_host.copy_(self.status, non_blocking=True)
            self._status_event = torch.cuda.Event()
            self._status_event.record()

    def _raise_for(self, values):
        lost, timeouts = (int(v) for v in values)
        if timeouts & 3:
            self.broken = True
            raise RuntimeError(f"expert-parallel exchange: a wait for a peer timed out (flags {timeouts}); "
                               "the exchange must be re-created")
        if timeouts & 4:
            raise RuntimeError("expert-parallel exchange: ranks passed different token counts")
        if lost:
            raise RuntimeError(f"expert-parallel exchange: {lost} routed slots exceeded the capacity")

    def close(self):
        """Unmap the peers' regions and free this rank's (a collective)."""
        import torch.distributed as dist

        if self.region is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self._group)
        lib = _lib.lib()
        for ptr in self._opened:
            _lib.check(lib.exlr8_ep_peer_close(ptr))
        dist.barrier(group=self._group)
        _lib.check(lib.exlr8_ep_peer_destroy(self.region))
        self._opened, self.region = [], None


class ExpertParallelMoE:
    """One MoE layer with this rank's routed shard (`local`, from
    shard_experts) and a replicated shared expert: the dense bf16 triple
    `shared`, or the one-expert trellis layer `shared_layer`.

    With the peer-memory exchange a bounded wait that times out (a peer that
    stopped) or a capacity overflow leaves partial rows in the output.  Eager
    calls therefore check the exchange status and raise: by default without
    a host synchronisation (``PeerExchange.check_deferred``: an error
    surfaces a call or two later), with ``deferred_check=False`` after every
    call (``check``, a synchronisation).  Calls made while a CUDA graph is
    being captured cannot check, so whoever replays such a graph must call
    ``self.peer.check()`` after the replays (bench.py does)."""

    def __init__(self, gate_weight, bias, local: ExpertLayer, rank: int, world: int, group=None, shared=None,
                 shared_layer: ExpertLayer | None = None, routed: int = 256, exchange: str = "nccl",
                 max_tokens: int = 16, peer: "PeerExchange | None" = None, placement: torch.Tensor | None = None,
                 deferred_check: bool = True):
        if (shared is None) == (shared_layer is None):
            raise ValueError("give exactly one shared expert (dense bf16 or trellis)")
        if routed % world or local.experts != routed // world:
            raise ValueError("the local shard must hold routed / world experts")
        self.gate_weight = gate_weight.to(torch.float32).contiguous()
        self.bias = bias.to(torch.float32).contiguous()
        self.local, self.rank, self.world = local, rank, world
        # Expert placement (seeded_placement): the exchange addresses expert e
        # by its position placement[e]; None = contiguous blocks.  The local
        # shard must come from shard_experts with the same placement.
        self._place = None
        if placement is not None:
            if placement.numel() != routed:
                raise ValueError("placement must hold one position per routed expert")
            lut = torch.arange(routed + 1, dtype=torch.int32, device=gate_weight.device)
            lut[:routed] = placement.to(device=gate_weight.device, dtype=torch.int32)
            self._place = lut  # id 256 (the shared slot) maps to itself
        self.per_rank = routed // world
        self.shared = None if shared is None else tuple(t.contiguous() for t in shared)
        self.shared_layer = shared_layer
        self.exchange = Exchange(world, group, rank)
        if exchange not in ("nccl", "peer"):
            raise ValueError("exchange must be 'nccl' or 'peer'")
        if exchange == "peer" and shared_layer is not None:
            raise ValueError("the peer-memory exchange runs with the bf16 shared expert")
        self.exchange_kind = exchange
        self.deferred_check = deferred_check
        self.max_tokens = max_tokens
        self.group = group
        # PeerExchange: given (shared by the layers of a stack, which run one
        # after another on one stream, so one region serves them all: a
        # source writes the next layer's rows only after the previous
        # layer's values came back), or created on the first call (a
        # collective).
        self.peer = peer
        if peer is not None and (peer.world != world or peer.rank != rank or peer.hidden != local.hidden
                                 or peer.max_capacity < max_tokens * 8):
            raise ValueError("the shared peer exchange does not fit this layer")
        self._side = None
        self._host_graphs = {}
        self._shared_struct = None
        self._owner_ws = None
        if self.shared is not None:
            self._shared_struct, self._keep = dense_expert(self.shared)
            self._local_struct, self._local_count = trellis_experts(local.packed, local.scales, local.k, local.hidden,
                                                                    local.intermediate)

    def owner_mlp(self, recv_x, recv_meta, xr):
        """(values [rows][hidden], shared [tokens][hidden]): the trellis MLP of
        the received rows and the bf16 shared expert of the local tokens in one
        call (exlr8_expert_mlp_shared)."""
        return self._owner_mlp(recv_x.data_ptr(), recv_meta.reshape(-1).contiguous(), recv_x.shape[0], xr)

    def _owner_mlp(self, recv_x_ptr, recv_meta, rows, xr):
        local = self.local
        h, m = local.hidden, local.intermediate
        tokens = xr.shape[0]
        device = xr.device
        values = torch.empty(rows, h, dtype=xr.dtype, device=device)
        shared = torch.empty(tokens, h, dtype=xr.dtype, device=device)
        lib = _lib.lib()
        need = lib.exlr8_expert_mlp_shared_workspace(rows, h, m, self._local_count, tokens)
        if self._owner_ws is None or self._owner_ws.numel() < need or self._owner_ws.device != device:
            self._owner_ws = _lib.workspace(need, device)
        ids_ptr = recv_meta if isinstance(recv_meta, int) else recv_meta.data_ptr()
        _lib.check(lib.exlr8_expert_mlp_shared(recv_x_ptr, _lib.act_code(xr), ids_ptr, rows,
                                               self._local_struct, xr.data_ptr(), tokens, self._shared_struct,
                                               values.data_ptr(), shared.data_ptr(), self._owner_ws.data_ptr(),
                                               self._owner_ws.numel(), _lib.stream_handle(device)))
        return values, shared

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

    def exchange_ids(self, ids: torch.Tensor) -> torch.Tensor:
        """The ids the exchange sends by: expert positions under a placement,
        else the ids themselves (out-of-range ids stay out of range)."""
        if self._place is None:
            return ids
        routed = self._place.numel() - 1
        safe = ids.clamp(0, routed).long()
        return torch.where((ids >= 0) & (ids < routed), self._place[safe], ids).to(ids.dtype).contiguous()

    def route(self, xr):
        """(ids [tokens][9], scores [tokens][8]) of the local tokens."""
        from .fast_router import route, router, router_logits

        if xr.shape[0] >= 64:  # the prefill gate product on the tensor cores
            return route(router_logits(xr, self.gate_weight), self.bias)
        _, ids, scores = router(xr, self.gate_weight, self.bias)
        return ids, scores

    def _peer_call(self, xr, res, ids, scores, residual, return_routing, out_ptr=None):
        """The layer with the peer-memory exchange (PeerExchange).  With
        out_ptr (a page-locked host buffer's device address) the combine
        writes the result there and no device output is made."""
        device = xr.device
        tokens, h = xr.shape
        if tokens > self.max_tokens:
            raise ValueError("more tokens than the peer exchange was sized for")
        if self.peer is None:
            self.peer = PeerExchange(self.world, self.rank, h, self.max_tokens, xr.dtype, device, self.group)
        peer = self.peer
        if peer.broken:
            raise RuntimeError("expert-parallel exchange is unusable after a timed-out wait; re-create the layer")
        lib = _lib.lib()
        stream = _lib.stream_handle(device)
        act = _lib.act_code(xr)
        slot_pos = torch.empty(max(tokens * 8, 1), dtype=torch.int32, device=device)
        xids = self.exchange_ids(ids)
        _lib.check(lib.exlr8_ep_send(xids.data_ptr(), tokens, xr.data_ptr(), act, h, self.world, self.rank,
                                     self.per_rank, peer.max_capacity, peer.peers.data_ptr(), peer.region,
                                     slot_pos.data_ptr(), peer.status.data_ptr(), stream))
        rows = self.world * tokens * 8
        values, shared = self._owner_mlp(peer.rows, peer.meta, rows, xr)
        _lib.check(lib.exlr8_ep_return(values.data_ptr(), act, h, self.world, self.rank, tokens, peer.max_capacity,
                                       peer.peers.data_ptr(), peer.region, peer.status.data_ptr(), stream))
        out = torch.empty_like(res) if out_ptr is None else None
        _lib.check(lib.exlr8_ep_combine(peer.back, act, slot_pos.data_ptr(), scores.data_ptr(), shared.data_ptr(),
                                        res.data_ptr(), tokens, h, out.data_ptr() if out_ptr is None else out_ptr,
                                        stream))
        out = None if out is None else out.reshape(residual.shape)
        if not torch.cuda.is_current_stream_capturing():
            peer.check_deferred() if self.deferred_check else peer.check()
        if return_routing:
            return out, ids, scores
        return out

    def __call__(self, x, residual, return_routing=False, out=None, graph=False):
        """``residual + moe(x)`` for this rank's tokens.  Every rank makes the
        same calls in the same order (the exchange is collective).

        Pinned host x and residual: the library's staging kernel reads them
        over PCIe at the head of the launch chain and the combine writes the
        result straight into ``out`` (a pinned host tensor, made here when not
        given), asynchronously on the current stream.  ``graph=True`` (host
        tensors and ``out``): the call is captured into a CUDA graph once per
        (x, residual, out) address triple and replayed on later calls --
        every rank must then capture and replay in the same order."""
        if x.device.type == "cpu":
            return self._host_call(x, residual, out, graph, return_routing)
        if out is not None or graph:
            raise ValueError("out= and graph=True take pinned host tensors")
        return self._device_call(x, residual, return_routing)

    def _host_call(self, x, residual, out, graph, return_routing):
        h = self.local.hidden
        if x.shape[-1] != h or residual.shape != x.shape or (out is not None and out.shape != x.shape):
            raise ValueError("host buffers take x, residual and out of one shape [..., hidden]")
        if out is None:
            if graph:
                raise ValueError("host graph mode takes an out tensor (the graph holds its address)")
            out = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        if not all(t.device.type == "cpu" and t.is_pinned() and t.is_contiguous() and t.dtype == x.dtype
                   for t in (x, residual, out)):
            raise ValueError("host buffers must be contiguous page-locked (pinned) tensors of one dtype")
        _lib.act_code(x)
        device = self.gate_weight.device
        tokens = x.numel() // h
        key = (x.data_ptr(), residual.data_ptr(), out.data_ptr(), tokens, x.dtype)
        entry = self._host_graphs.get(key) if graph else None
        if entry is None:
            xd = torch.empty(tokens, h, dtype=x.dtype, device=device)
            rd = torch.empty_like(xd)
            out_ptr = _lib.host_device_pointer(out)
            nbytes = x.numel() * x.element_size()

            def body():
                _lib.check(_lib.lib().exlr8_stage_in(x.data_ptr(), xd.data_ptr(), residual.data_ptr(),
                                                     rd.data_ptr(), nbytes, _lib.stream_handle(device)))
                return self._device_call(xd, rd, True, out_ptr=out_ptr)

            _, ids, scores = body()  # eager (and, for a graph, the call before its capture)
            if graph:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    _, ids, scores = body()
                self._host_graphs[key] = (g, ids, scores, xd, rd)
        else:
            entry[0].replay()
            ids, scores = entry[1], entry[2]
        if return_routing:
            return out, ids, scores
        return out

    def clear_graphs(self):
        """Release the host-mode graphs (before the process group goes away)."""
        self._host_graphs.clear()

    def _device_call(self, x, residual, return_routing=False, out_ptr=None):
        device = _lib.require_cuda(x, residual)
        h = self.local.hidden
        tokens = x.numel() // h
        xr = x.reshape(tokens, h).contiguous()
        res = residual.reshape(tokens, h).to(x.dtype).contiguous()
        ids, scores = self.route(xr)
        lib = _lib.lib()
        stream = _lib.stream_handle(device)
        cap = tokens * 8
        if self.exchange_kind == "peer" and self.world > 1:
            return self._peer_call(xr, res, ids, scores, residual, return_routing, out_ptr)
        send_x = torch.empty(self.world, cap, h, dtype=x.dtype, device=device)
        send_meta = torch.empty(self.world, cap, dtype=torch.int32, device=device)
        slot_pos = torch.empty(max(tokens * 8, 1), dtype=torch.int32, device=device)
        counts = torch.empty(self.world, dtype=torch.int32, device=device)
        status = torch.zeros(1, dtype=torch.int32, device=device)
        xids = self.exchange_ids(ids)
        _lib.check(lib.exlr8_ep_dispatch(xids.data_ptr(), tokens, xr.data_ptr(), _lib.act_code(xr), h, self.world,
                                         self.per_rank, cap, send_x.data_ptr(), send_meta.data_ptr(),
                                         slot_pos.data_ptr(), counts.data_ptr(), status.data_ptr(), stream))
        rows = self.world * cap
        local = self.local
        if self.shared is not None:
            recv_x, recv_meta = self.exchange(send_x, send_meta)
            values, shared = self.owner_mlp(recv_x.reshape(rows, h), recv_meta, xr)
            back = self.exchange(values.reshape(self.world, cap, h))
        else:
            # The trellis shared expert runs on a side stream, overlapping the
            # exchange and the owner's expert products.
            main = torch.cuda.current_stream(device)
            if self._side is None or self._side.device != device:
                self._side = torch.cuda.Stream(device)
            self._side.wait_stream(main)
            with torch.cuda.stream(self._side):
                shared = self.shared_values(xr)
            recv_x, recv_meta = self.exchange(send_x, send_meta)
            values = fast_expert_mlp(recv_x.reshape(rows, h), recv_meta.reshape(rows, 1), local.packed, local.scales,
                                     local.k, h, local.intermediate)
            back = self.exchange(values.reshape(self.world, cap, h))
            main.wait_stream(self._side)
            shared.record_stream(main)
        out = torch.empty_like(res) if out_ptr is None else None
        _lib.check(lib.exlr8_ep_combine(back.data_ptr(), _lib.act_code(xr), slot_pos.data_ptr(), scores.data_ptr(),
                                        shared.data_ptr(), res.data_ptr(), tokens, h,
                                        out.data_ptr() if out_ptr is None else out_ptr, stream))
        out = None if out is None else out.reshape(residual.shape)
        if return_routing:
            return out, ids, scores
        return out
