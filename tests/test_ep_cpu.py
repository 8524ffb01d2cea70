"""Host side of the expert-parallel layer on CPU: the equal-split all-to-all
over gloo ranks (world size 2) and the expert sharding."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange_worker(rank, world, port, queue):
    import torch.distributed as dist

    from mlxlr8_b200.ep import Exchange

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cap, h = 3, 4
        # send[d][row] = 100 * source + 10 * destination + row
        send = torch.stack([torch.full((cap, h), 100.0 * rank + 10.0 * d) + torch.arange(cap)[:, None]
                            for d in range(world)])
        ex = Exchange(world, rank=rank)
        recv = ex(send)
        meta = ex(torch.full((world, cap), rank, dtype=torch.int32))
        back = ex(recv)
        # Two tensors in one grouped exchange (rows and their expert ids).
        recv2, meta2 = ex(send, torch.full((world, cap), rank, dtype=torch.int32))
        grouped = torch.equal(recv2, recv) and torch.equal(meta2, meta)
        queue.put((rank, recv.tolist(), meta.tolist(), torch.equal(back, send) and grouped))
    finally:
        dist.destroy_process_group()


def test_exchange_round_trip_over_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, recv, meta, round_trip = queue.get(timeout=120)
        results[rank] = (recv, meta, round_trip)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in range(world):
        recv, meta, round_trip = results[rank]
        assert round_trip
        for src in range(world):
            # row `row` of the block from `src` was addressed to this rank
            assert [r[0] for r in recv[src]] == [100.0 * src + 10.0 * rank + row for row in range(3)]
            assert meta[src] == [src] * 3


def test_shard_experts_slices_contiguous_blocks():
    from mlxlr8_b200.ep import shard_experts, shared_trellis
    from mlxlr8_b200.experts import ExpertLayer

    h, m, k, experts = 128, 128, 4, 9
    nbytes = h * m * k // 8
    packed = {p: torch.arange(experts * nbytes, dtype=torch.int64).to(torch.uint8) for p in ("gate", "up", "down")}
    scales = {p: (torch.arange(experts, dtype=torch.float16)[:, None].repeat(1, h),
                  torch.arange(experts, dtype=torch.float16)[:, None].repeat(1, m)) for p in ("gate", "up", "down")}
    layer = ExpertLayer(packed, scales, k, h, m)
    shard = shard_experts(layer, 1, 2, routed=8)
    assert shard.experts == 4
    assert torch.equal(shard.packed["gate"], packed["gate"][4 * nbytes:8 * nbytes])
    assert shard.scales["down"][0][0, 0] == 4 and shard.scales["down"][1][3, 0] == 7
    shared = shared_trellis(layer, index=8)
    assert shared.experts == 1 and shared.scales["up"][0][0, 0] == 8
    assert shared_trellis(layer, index=9) is None
    with pytest.raises(ValueError):
        shard_experts(layer, 0, 3, routed=8)


def test_peer_region_layout_and_checks():
    """Peer-exchange region (exlr8_ep_peer_*): flags, then meta, rows and back
    areas on 256-byte boundaries sized for ranks x max capacity rows; shapes
    outside the supported range are refused (host-only calls)."""
    import ctypes

    from mlxlr8_b200 import _lib

    lib = _lib.lib()
    meta, rows, back = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
    ranks, cap, hidden = 8, 128, 6144
    assert lib.exlr8_ep_peer_offsets(ranks, cap, hidden, 2, ctypes.byref(meta), ctypes.byref(rows),
                                     ctypes.byref(back)) == 0
    total = lib.exlr8_ep_peer_bytes(ranks, cap, hidden, 2)
    assert meta.value == 1536                                       # epoch, flags, capacities, counters
    assert rows.value >= meta.value + ranks * cap * 4 and rows.value % 256 == 0
    assert back.value == rows.value + ranks * cap * hidden * 2
    assert total == back.value + ranks * cap * hidden * 2
    assert lib.exlr8_ep_peer_bytes(65, cap, hidden, 2) == 0          # at most 64 ranks
    assert lib.exlr8_ep_peer_bytes(ranks, 8192, hidden, 2) == 0      # at most 4096 rows per pair
    assert lib.exlr8_ep_peer_bytes(ranks, cap, 100, 2) == 0          # rows of whole 16-byte vectors
    status = lib.exlr8_ep_send(None, 3, None, 2, hidden, ranks, 0, 32, 16, None, None, None, None, None)
    assert status != 0                                              # 3 tokens x 8 > 16 rows


def test_seeded_placement_partitions_the_experts():
    """ep.seeded_placement is a seeded permutation; rank r owns the experts
    placed at [r * per, (r + 1) * per), every expert exactly once."""
    from mlxlr8_b200.ep import _owned, seeded_placement

    a = seeded_placement(7, device="cpu")
    assert torch.equal(a, seeded_placement(7, device="cpu"))
    assert sorted(a.tolist()) == list(range(256))
    assert not torch.equal(a, seeded_placement(8, device="cpu"))
    for world in (1, 2, 4, 8):
        owned = [_owned(r, world, 256, a) for r in range(world)]
        assert sorted(e for part in owned for e in part) == list(range(256))
        for r, part in enumerate(owned):
            assert all(a[e].item() // (256 // world) == r for e in part)
        if world > 1:
            assert _owned(1, world, 256, None) == list(range(256 // world, 2 * 256 // world))
