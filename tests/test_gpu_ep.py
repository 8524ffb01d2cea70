"""Expert-parallel layer on one GPU: dispatch positions against a plain
restatement, and the whole exchange (dispatch, all-to-all, grouped expert
MLP on the owner, all-to-all back, combine) with N emulated ranks against the
oracle of the single-device MoE layer (model.py:385-418).

The all-to-all of N ranks is emulated by stacking the ranks' send buffers;
the NCCL exchange itself runs in test_gpu_ep_multi.py on two GPUs.
"""

import numpy as np
import pytest

from helpers import host, rel_l2
from oracle import trellis_oracle as ref

pytestmark = pytest.mark.gpu


def _positions_reference(ids, ranks, per_rank, capacity):
    """Destination rank * capacity + row of every routed slot, rows in slot order."""
    ids = np.asarray(ids)
    tokens = ids.shape[0]
    pos = np.full(tokens * 8, -1, np.int64)
    meta = np.full((ranks, capacity), -1, np.int64)
    fill = [0] * ranks
    for i in range(tokens * 8):
        e = int(ids[i // 8, i % 8])
        if e >= ranks * per_rank:
            continue
        d = e // per_rank
        if fill[d] < capacity:
            pos[i] = d * capacity + fill[d]
            meta[d, fill[d]] = e % per_rank
        fill[d] += 1
    return pos, meta, fill


def _dispatch(ids, x, ranks, per_rank, capacity):
    import torch

    from mlxlr8_b200 import _lib

    tokens, h = x.shape
    send_x = torch.empty(ranks, capacity, h, dtype=x.dtype, device="cuda")
    send_meta = torch.empty(ranks, capacity, dtype=torch.int32, device="cuda")
    slot_pos = torch.empty(max(tokens * 8, 1), dtype=torch.int32, device="cuda")
    counts = torch.empty(ranks, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.check(_lib.lib().exlr8_ep_dispatch(ids.data_ptr(), tokens, x.data_ptr(), _lib.act_code(x), h, ranks,
                                            per_rank, capacity, send_x.data_ptr(), send_meta.data_ptr(),
                                            slot_pos.data_ptr(), counts.data_ptr(), status.data_ptr(),
                                            _lib.stream_handle(x.device)))
    return send_x, send_meta, slot_pos[:tokens * 8], counts, status


@pytest.mark.parametrize("tokens, ranks, capacity", [(5, 2, 40), (300, 8, 2400), (37, 4, 20)])
def test_dispatch_positions_match_restatement(tokens, ranks, capacity):
    import torch

    rng = np.random.default_rng(tokens)
    per_rank = 256 // ranks
    ids = np.concatenate([rng.integers(0, 260, (tokens, 8)), np.full((tokens, 1), 256)], axis=1).astype(np.int32)
    x = torch.randn(tokens, 256, device="cuda").to(torch.bfloat16)
    send_x, send_meta, slot_pos, counts, status = _dispatch(torch.from_numpy(ids).cuda(), x, ranks, per_rank,
                                                           capacity)
    torch.cuda.synchronize()
    pos, meta, fill = _positions_reference(ids, ranks, per_rank, capacity)
    np.testing.assert_array_equal(slot_pos.cpu().numpy(), pos)
    np.testing.assert_array_equal(send_meta.cpu().numpy(), meta)
    np.testing.assert_array_equal(counts.cpu().numpy(), np.minimum(fill, capacity))
    assert status.item() == sum(max(f - capacity, 0) for f in fill)
    xs = x.cpu()
    flat = send_x.reshape(-1, 256).cpu()
    for i in np.nonzero(pos >= 0)[0][:200]:
        assert torch.equal(flat[pos[i]], xs[i // 8])


def _emulated_layer(layer, x, residual, world, placement=None):
    """The expert-parallel layer over `world` emulated ranks on one GPU
    (contiguous expert blocks, or the given placement)."""
    import torch

    from mlxlr8_b200 import _lib
    from mlxlr8_b200.ep import ExpertParallelMoE, shard_experts, shared_trellis
    from mlxlr8_b200.fast_decode import fast_expert_mlp

    e = layer.experts
    tokens, h = x.shape
    tl = tokens // world
    shared_layer = shared_trellis(e) if e.shared is None else None
    ranks = [ExpertParallelMoE(layer.gate_weight, layer.bias, shard_experts(e, r, world, placement=placement), r,
                               world, shared=e.shared, shared_layer=shared_layer, placement=placement)
             for r in range(world)]
    cap = tl * 8
    sends, routing = [], []
    for r, m in enumerate(ranks):
        xr = x[r * tl:(r + 1) * tl].contiguous()
        ids, scores = m.route(xr)
        send_x, send_meta, slot_pos, counts, status = _dispatch(m.exchange_ids(ids), xr, world, 256 // world, cap)
        sends.append((send_x, send_meta))
        routing.append((ids, scores, slot_pos, status))
    back_parts = [[None] * world for _ in range(world)]
    for r, m in enumerate(ranks):
        recv_x = torch.stack([sends[s][0][r] for s in range(world)])
        recv_meta = torch.stack([sends[s][1][r] for s in range(world)])
        values = fast_expert_mlp(recv_x.reshape(-1, h), recv_meta.reshape(-1, 1), m.local.packed, m.local.scales,
                                 m.local.k, h, m.local.intermediate).reshape(world, cap, h)
        for s in range(world):
            back_parts[s][r] = values[s]
    outs, all_ids, all_scores = [], [], []
    for r, m in enumerate(ranks):
        xr = x[r * tl:(r + 1) * tl].contiguous()
        res = residual[r * tl:(r + 1) * tl].contiguous()
        ids, scores, slot_pos, status = routing[r]
        assert status.item() == 0
        back = torch.stack(back_parts[r])
        shared = m.shared_values(xr)
        out = torch.empty_like(res)
        _lib.check(_lib.lib().exlr8_ep_combine(back.data_ptr(), _lib.act_code(xr), slot_pos.data_ptr(),
                                               scores.data_ptr(), shared.data_ptr(), res.data_ptr(), tl, h,
                                               out.data_ptr(), _lib.stream_handle(x.device)))
        outs.append(out)
        all_ids.append(ids)
        all_scores.append(scores)
    return torch.cat(outs), torch.cat(all_ids), torch.cat(all_scores)


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("shared", ["bf16", "trellis"])
@pytest.mark.parametrize("tokens_per_rank", [2, 24])
def test_emulated_expert_parallel_layer_matches_oracle(world, shared, tokens_per_rank):
    import torch

    from mlxlr8_b200.fast_router import router, router_logits
    from mlxlr8_b200.synthetic import host_copy, make_layer

    layer = make_layer(seed=31, hidden=256, intermediate=128, shared=shared)
    tokens = world * tokens_per_rank
    x, residual = layer.tokens(tokens)
    out, ids, scores = _emulated_layer(layer, x, residual, world)
    torch.cuda.synchronize()
    # Routing is per rank; each rank's logits come from the same gate product.
    if tokens_per_rank >= 64:
        logits = router_logits(x, layer.gate_weight)
    else:
        logits, _, _ = router(x, layer.gate_weight, layer.bias)
    ids_np = ids.cpu().numpy()
    hc = host_copy(layer, np.unique(ids_np[:, :8] if shared == "bf16" else ids_np))
    e_out, e_ids, e_scores = ref.moe_layer(host(x), host(residual), hc["gate_weight"], hc["bias"], hc["packed"],
                                           hc["scales"], 4, 256, 128, shared=hc["shared"], dtype="bfloat16",
                                           logits=host(logits))
    np.testing.assert_array_equal(ids_np, e_ids)
    got, want = host(out) - host(residual), e_out - host(residual)
    scale = float(np.max(np.abs(want)))
    assert float(np.max(np.abs(got - want))) <= 1e-2 * scale
    assert rel_l2(got, want) < 5e-3


@pytest.mark.parametrize("world", [2, 4])
def test_seeded_placement_gives_the_same_layer(world):
    """Experts placed by a seeded permutation (ep.seeded_placement) instead of
    contiguous blocks: every slot's value comes from the same expert operator
    on the same rows, so the layer's output is identical bit for bit, and
    each rank holds the experts placed at its positions."""
    import torch

    from mlxlr8_b200.ep import seeded_placement
    from mlxlr8_b200.synthetic import make_layer

    layer = make_layer(seed=33, hidden=256, intermediate=128, shared="bf16")
    x, residual = layer.tokens(world * 24)
    plain, ids, _ = _emulated_layer(layer, x, residual, world)
    placement = seeded_placement(7)
    placed, ids2, _ = _emulated_layer(layer, x, residual, world, placement=placement)
    torch.cuda.synchronize()
    assert torch.equal(ids, ids2)
    assert torch.equal(plain, placed)
    per = 256 // world
    owners = placement.cpu().numpy() // per
    assert sorted(np.bincount(owners, minlength=world).tolist()) == [per] * world


@pytest.mark.parametrize("rows, tokens", [(16, 2), (40, 5), (24, 0)])
def test_owner_mlp_with_shared_matches_separate_calls(rows, tokens):
    """exlr8_expert_mlp_shared (the owner's trellis MLP over received rows with
    the local tokens' bf16 shared expert streamed in the same kernels) against
    exlr8_expert_mlp (slots = 1) and exlr8_shared_expert called separately.
    Empty rows (id -1) give zeros."""
    import torch

    from mlxlr8_b200.ep import ExpertParallelMoE, shard_experts
    from mlxlr8_b200.fast_decode import fast_expert_mlp
    from mlxlr8_b200.synthetic import make_layer

    layer = make_layer(seed=41, hidden=256, intermediate=128, shared="bf16")
    e = layer.experts
    world = 4
    moe = ExpertParallelMoE(layer.gate_weight, layer.bias, shard_experts(e, 1, world), 1, world, shared=e.shared)
    g = torch.Generator(device="cuda")
    g.manual_seed(rows)
    recv_x = torch.randn(rows, 256, generator=g, device="cuda").to(torch.bfloat16)
    meta = torch.randint(-1, 64, (rows,), generator=g, device="cuda", dtype=torch.int32)
    xr = torch.randn(max(tokens, 1), 256, generator=g, device="cuda").to(torch.bfloat16)[:tokens]
    values, shared = moe.owner_mlp(recv_x, meta, xr)
    local = moe.local
    want_values = fast_expert_mlp(recv_x, meta.reshape(rows, 1), local.packed, local.scales, local.k, 256, 128)
    want_values = want_values.reshape(rows, 256)
    torch.cuda.synchronize()
    got, want = host(values), host(want_values)
    assert np.all(got[host(meta) < 0] == 0)
    scale = float(np.max(np.abs(want)))
    assert float(np.max(np.abs(got - want))) <= 1e-2 * scale
    if tokens:
        want_shared = host(moe.shared_values(xr))
        got_shared = host(shared)
        s2 = float(np.max(np.abs(want_shared)))
        # Same bf16 products; only the K-split summation order differs.
        assert float(np.max(np.abs(got_shared - want_shared))) <= 1e-2 * s2
        assert rel_l2(got_shared, want_shared) < 5e-3


def test_peer_exchange_wait_times_out_and_reports():
    """The peer exchange's waits are bounded: with a peer that never sends
    (rank 1's region is this rank's own, and nothing sets rank 1's flags) the
    send and return kernels give up after about a second each and set their
    status bits; the stream stays usable."""
    import ctypes

    import torch

    from mlxlr8_b200 import _lib

    lib = _lib.lib()
    ranks, max_cap, hidden = 2, 8, 256
    nbytes = lib.exlr8_ep_peer_bytes(ranks, max_cap, hidden, 2)
    region, handle = ctypes.c_void_p(), (ctypes.c_ubyte * 64)()
    _lib.check(lib.exlr8_ep_peer_create(nbytes, ctypes.byref(region), handle))
    try:
        peers = torch.tensor([region.value, region.value], dtype=torch.int64, device="cuda")
        ids = torch.tensor([[0, 1, 2, 3, 200, 201, 202, 203, 256]], dtype=torch.int32, device="cuda")
        x = torch.randn(1, hidden, device="cuda").to(torch.bfloat16)
        slot_pos = torch.empty(8, dtype=torch.int32, device="cuda")
        status = torch.zeros(2, dtype=torch.int32, device="cuda")
        stream = _lib.stream_handle(x.device)
        _lib.check(lib.exlr8_ep_send(ids.data_ptr(), 1, x.data_ptr(), 2, hidden, ranks, 0, 128, max_cap,
                                     peers.data_ptr(), region.value, slot_pos.data_ptr(), status.data_ptr(), stream))
        torch.cuda.synchronize()
        assert status[1].item() & 1
        values = torch.zeros(ranks * 8, hidden, dtype=torch.bfloat16, device="cuda")
        _lib.check(lib.exlr8_ep_return(values.data_ptr(), 2, hidden, ranks, 0, 1, max_cap, peers.data_ptr(),
                                       region.value, status.data_ptr(), stream))
        torch.cuda.synchronize()
        assert status[1].item() & 2
        assert torch.equal(slot_pos.cpu()[:4], torch.tensor([0, 1, 2, 3], dtype=torch.int32))
        assert torch.equal(slot_pos.cpu()[4:], torch.tensor([8, 9, 10, 11], dtype=torch.int32))
        torch.zeros(4, device="cuda").sum().item()  # the context still works
    finally:
        _lib.check(lib.exlr8_ep_peer_destroy(region.value))


def test_deferred_status_check_raises_without_synchronising():
    """PeerExchange.check_deferred: the first call only queues a copy of the
    (cumulative) status word; once that copy has landed the next call raises
    for a timed-out wait and marks the exchange unusable."""
    import torch

    from mlxlr8_b200.ep import PeerExchange

    ex = PeerExchange.__new__(PeerExchange)
    ex.status = torch.zeros(2, dtype=torch.int32, device="cuda")
    ex._status_host = torch.zeros(2, dtype=torch.int32).pin_memory()
    ex._status_event = None
    ex.broken = False
    ex.check_deferred()  # nothing wrong, a copy is queued
    torch.cuda.synchronize()
    ex.check_deferred()  # the clean copy is checked, the next queued
    ex.status[1] = 2     # a return wait timed out
    torch.cuda.synchronize()
    ex.check_deferred()  # checks the copy made before the error; queues a new one
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="timed out"):
        ex.check_deferred()
    assert ex.broken


@pytest.mark.parametrize("tokens", [1, 4])
def test_host_buffer_modes_match_the_device_call(tokens):
    """ExpertParallelMoE with pinned host x / residual / out (world 1, where
    the exchange is the identity): eager and graph modes stage the inputs by
    the library's kernel and the combine writes the pinned out; both equal
    the device call bit for bit, and the graph replays on new contents."""
    import torch

    from mlxlr8_b200.ep import ExpertParallelMoE, shard_experts
    from mlxlr8_b200.synthetic import make_layer

    layer = make_layer(seed=43, hidden=256, intermediate=128, shared="bf16")
    e = layer.experts
    moe = ExpertParallelMoE(layer.gate_weight, layer.bias, shard_experts(e, 0, 1), 0, 1, shared=e.shared)
    x, r = layer.tokens(tokens, seed_offset=5)
    xh, rh = x.cpu().pin_memory(), r.cpu().pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    want = moe(x, r)
    got = moe(xh, rh, out=oh)
    torch.cuda.synchronize()
    assert got.data_ptr() == oh.data_ptr() and torch.equal(oh, want.cpu())
    for step in range(3):
        x2, r2 = layer.tokens(tokens, seed_offset=20 + step)
        xh.copy_(x2.cpu())
        rh.copy_(r2.cpu())
        moe(xh, rh, out=oh, graph=True)
        want = moe(x2, r2)
        torch.cuda.synchronize()
        assert torch.equal(oh, want.cpu())
    moe.clear_graphs()
