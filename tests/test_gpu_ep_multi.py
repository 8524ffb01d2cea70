"""Expert-parallel layer over NCCL on two GPUs (one process per GPU): the
gathered output equals the oracle of the single-device layer within the
layer tolerance.  Skipped on machines with fewer than two GPUs."""

import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _gpus():
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("shared, tokens_per_rank, exchange", [("bf16", 3, "nccl"), ("trellis", 20, "nccl"),
                                                               ("bf16", 2, "peer")])
def test_two_gpu_expert_parallel_layer(tmp_path, shared, tokens_per_rank, exchange):
    import torch

    from helpers import host, rel_l2
    from mlxlr8_b200.fast_router import router
    from mlxlr8_b200.synthetic import host_copy, make_layer
    from oracle import trellis_oracle as ref

    out_path = str(tmp_path / "ep.pt")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29517", os.path.join(ROOT, "tests", "ep_worker.py"), out_path,
           shared, str(tokens_per_rank), exchange]
    subprocess.run(cmd, check=True, env=env, timeout=600)
    got = torch.load(out_path)
    layer = make_layer(seed=31, hidden=256, intermediate=128, shared=shared)
    x = got["x"].cuda()
    logits, _, _ = router(x, layer.gate_weight, layer.bias)
    ids_np = got["ids"].numpy()
    hc = host_copy(layer, np.unique(ids_np[:, :8] if shared == "bf16" else ids_np))
    res = host(got["residual"])
    e_out, e_ids, _ = ref.moe_layer(host(got["x"]), res, hc["gate_weight"], hc["bias"], hc["packed"], hc["scales"], 4,
                                    256, 128, shared=hc["shared"], dtype="bfloat16", logits=host(logits))
    np.testing.assert_array_equal(ids_np, e_ids)
    want = e_out - res
    if exchange == "peer":
        # Same kernels on the same rows: the peer exchange is bit-exact against
        # the NCCL one, and repeated calls give the same result.
        assert torch.equal(got["ep"], got["nccl"])
        assert torch.equal(got["ep"], got["first"])
    for key in ("ep", "single"):
        diff = host(got[key]) - res
        assert float(np.max(np.abs(diff - want))) <= 1e-2 * float(np.max(np.abs(want)))
        assert rel_l2(diff, want) < 5e-3
