"""One rank of the two-GPU expert-parallel check (launched by
test_gpu_ep_multi.py under torch.distributed.run).  Every rank builds the
same seeded layer, runs ExpertParallelMoE on its token slice (argv[4]:
'nccl' exchange, or 'peer': the peer-memory exchange, run for three calls and
compared with the NCCL exchange), and rank 0 writes the gathered output,
routing and the single-device layer's output to the path in argv[1]."""

import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    from datetime import timedelta

    from mlxlr8_b200.ep import ExpertParallelMoE, shard_experts, shared_trellis
    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.synthetic import make_layer

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    try:
        out_path, shared, tokens_per_rank = sys.argv[1], sys.argv[2], int(sys.argv[3])
        exchange = sys.argv[4] if len(sys.argv) > 4 else "nccl"
        layer = make_layer(seed=31, hidden=256, intermediate=128, shared=shared)
        e = layer.experts
        moe = ExpertParallelMoE(layer.gate_weight, layer.bias, shard_experts(e, rank, world), rank, world,
                                shared=e.shared, shared_layer=shared_trellis(e) if e.shared is None else None,
                                exchange=exchange)
        x, residual = layer.tokens(world * tokens_per_rank)
        lo, hi = rank * tokens_per_rank, (rank + 1) * tokens_per_rank
        xs, rs = x[lo:hi].contiguous(), residual[lo:hi].contiguous()
        extra = {}
        if exchange == "peer":
            # Three calls (the epoch advances each time; the middle one has other
            # inputs), then the NCCL exchange on the same inputs for comparison.
            first = moe(xs, rs)
            x2, r2 = layer.tokens(world * tokens_per_rank, seed_offset=5)
            moe(x2[lo:hi].contiguous(), r2[lo:hi].contiguous())
            out, ids, scores = moe(xs, rs, return_routing=True)
            moe.peer.check()
            ref_moe = ExpertParallelMoE(layer.gate_weight, layer.bias, shard_experts(e, rank, world), rank, world,
                                        shared=e.shared)
            nccl_out = ref_moe(xs, rs)
            for name, t in (("first", first), ("nccl", nccl_out)):
                parts = [torch.empty_like(t) for _ in range(world)]
                dist.all_gather(parts, t)
                extra[name] = torch.cat(parts).cpu()
            moe.peer.close()
        else:
            out, ids, scores = moe(xs, rs, return_routing=True)
        parts = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(parts, out)
        id_parts = [torch.empty_like(ids) for _ in range(world)]
        dist.all_gather(id_parts, ids)
        torch.cuda.synchronize()
        if rank == 0:
            single = MoELayer(layer.gate_weight, layer.bias, e)(x, residual)
            torch.save({"ep": torch.cat(parts).cpu(), "ids": torch.cat(id_parts).cpu(), "single": single.cpu(),
                        "x": x.cpu(), "residual": residual.cpu(), **extra}, out_path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
