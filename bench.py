"""Benchmark: the GLM-5-shape routed-MoE layer (exlr8 MoE branch) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T] [--impl {b200,reference}]

Headline (single-layer decode, uniform routing): T tokens per GPU (default 1)
through one MoE layer -- router (fp32 gate 6144->256, sigmoid + bias top-8,
renormalised x2.5), 256 routed K4-trellis SwiGLU experts (6144 -> 2048 ->
6144), the bf16 shared expert and the combine with the residual.  Weights
are seeded synthetic tensors of that shape (no checkpoints here), one
independent layer per step, cycling through --layers layers so each step
streams weights that are not in L2 (every step touches > 233 MB; 8 layers
hold ~39 GB).  A "step" is one layer pass over one batch; the metric is
tokens per second.

value: device-resident inputs, the layer call replayed from a CUDA graph.
e2e:   the public API with pinned host buffers: per step x and residual
       cross PCIe to the GPU and the output back, inside the timed region.
       The call is MoELayer.__call__ (ExpertParallelMoE.__call__ on several
       GPUs) with pinned host x, residual and out (graph=True): the layer's
       first kernel reads the inputs from host memory and its combine writes
       the output there; with copy-engine copies around the device call
       instead, e2e was 5% lower on one GPU.
roofline: the dominant kernel (trellis gate/up streaming GEMV), its launch
       durations measured with CUDA events on the launching stream during a
       profiled pass of the same K steps; algorithmic bytes = packed trellis
       codes it must stream (U experts x 2 matrices x K*h*m/8) plus, on one
       GPU, the bf16 shared expert's gate/up rows the same launch streams.
cpu_baseline: the C restatement of the layer (oracle/c, OpenMP) on the host's
       cores, a bounded number of full layer steps.
--impl reference: the reference's expert operators are Metal kernels
       (unavailable here), so the reference arm is that same CPU restatement
       of the reference's arithmetic, on all host threads, on the same
       workload (all GPUs' tokens per step).

Under torchrun (N > 1) the headline layers are expert-parallel: each GPU
holds 256 / N routed experts of every layer and the replicated shared expert,
takes T tokens of its own (global batch T * N, weak scaling), and dispatch
and combine go over peer memory (NVLink stores + epoch flags; `--ep-exchange
nccl` for the NCCL all-to-all) inside each layer's CUDA graph; time is the
max over ranks.

ep_stack (every N): the 75-layer expert stack (layers 3-77; attention and the
three dense layers stubbed) at a fixed global batch of 64 decode tokens
(strong scaling: 64 / N tokens per GPU), each block a post-attention RMS norm
and the MoE layer; one CUDA graph per stack step.  One GPU runs the fused
single-device layer; N > 1 the expert-parallel layer over one shared
peer-memory exchange.  Where 75 layers of weights do not fit in HBM (N = 1,
2) the stack cycles the resident layers.  Reported: tokens/s, per-phase
device times, and the fraction of the per-layer max(HBM, NVLink) time.

Single-GPU extras:
- decode at T = 4 (the parity configuration), 8 and 32;
- the prefill configurations: joined MXFP4 at 4096 tokens; 128 tokens at K4
  and K3;
- the MoE block stack: the layers plus the K3 layer-78 block, each behind its
  post-attention RMS norm, attention stubbed; at T = 1, and at T = 128 with
  Zipf(1.1)-skewed routing;
- the joined MXFP4 decode;
- the load-time trellis -> MXFP4 re-encode;
- the static hot-expert cache against the codes;
- the checkpoint load.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HIDDEN, INTER, EXPERTS, K_BITS = 6144, 2048, 256, 4
METRIC = "MoE-layer tokens/s (decode GB/s vs HBM; prefill TFLOPS) at 1/2/4/8 B200"

# dram__bytes_read.sum + dram__bytes_write.sum of one gate/up streaming-GEMV
# launch from the ncu capture in profiles/trellis_stream_gate_up_decode.md:
# 8 distinct experts (16 matrices) plus the bf16 shared expert's gate/up rows,
# which the same launch streams.  The bench splits it into a per-matrix part
# (the codes scale with the matrices its own launches stream) and the shared
# expert's part, taken as its algorithmic bytes.
DENSE_GATE_UP_BYTES = 2 * 6144 * 2048 * 2
GATE_UP_TRAFFIC_8 = 151_499_520 + 6_107_136
TRAFFIC_PER_MATRIX = (GATE_UP_TRAFFIC_8 - DENSE_GATE_UP_BYTES) / 16


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=4000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--tokens", type=int, default=1)
    p.add_argument("--layers", type=int, default=8)
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--ncu-driver", choices=("layer", "mlp", "joined", "trellis", "encode"), default=None,
                   help="untimed run for an ncu capture: 'layer' calls one resident layer --calls times; 'mlp' "
                        "runs the nine-expert fast_expert_mlp at full size (about 170 MB of weights); 'joined' "
                        "runs JoinedMXFP4.finish at full width over --experts experts (the last one shared) with "
                        "--tokens tokens, top-8 uniform routing (about 4 GB on the device at 129 experts and 2048 "
                        "tokens); 'trellis' runs the grouped trellis prefill (expert_mlp_finish with the dense bf16 "
                        "shared expert) over --experts K4 experts with --tokens tokens, plus the tensor-core router "
                        "gate product; 'encode' re-encodes --experts full-size K4 experts to joined MXFP4")
    p.add_argument("--experts", type=int, default=129)
    p.add_argument("--no-extras", action="store_true",
                   help="skip the single-GPU extras (decode at T=8/32, the prefill configurations)")
    p.add_argument("--calls", type=int, default=5)
    p.add_argument("--peaks", action="store_true",
                   help="print the tensor-core and trellis-codec peak probes of GPU 0 as one JSON line and exit")
    p.add_argument("--no-stack", action="store_true", help="skip the 75-layer expert-parallel stack")
    p.add_argument("--stack-layers", type=int, default=75)
    p.add_argument("--stack-batch", type=int, default=64, help="global decode batch of the stack (strong scaling)")
    p.add_argument("--stack-steps", type=int, default=5)
    p.add_argument("--stack-budget-gb", type=float, default=110.0,
                   help="device memory for resident stack layers; beyond it the stack cycles resident layers")
    p.add_argument("--ep-exchange", choices=("peer", "nccl"), default="peer",
                   help="N > 1: the expert-parallel exchange, over peer memory (NVLink stores + epoch flags) or "
                        "NCCL all-to-all")
    return p.parse_args()


def ncu_driver(args):
    """Small, untimed workload for ncu (no graphs, no clocks, one GPU)."""
    import torch

    from mlxlr8_b200.fast_decode import fast_expert_mlp
    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.synthetic import make_layer

    torch.cuda.set_device(0)
    if args.ncu_driver == "joined":
        from mlxlr8_b200.joined_mxfp4 import JoinedMXFP4
        from mlxlr8_b200.synthetic import make_joined

        j = make_joined(seed=1, experts=args.experts)
        joined = JoinedMXFP4(j.unit, j.weights, j.scales, j.hidden, j.intermediate)
        t = args.tokens
        g = torch.Generator(device="cuda")
        g.manual_seed(1)
        routed = torch.rand(t, args.experts - 1, generator=g, device="cuda").argsort(dim=1)[:, :8].int()
        ids = torch.cat([routed, torch.full((t, 1), args.experts - 1, dtype=torch.int32, device="cuda")], dim=1)
        scores = torch.rand(t, 8, generator=g, device="cuda")
        x, r = j.tokens(t)
        for _ in range(args.calls):
            joined.finish(x, ids, scores, r)
    elif args.ncu_driver == "trellis":
        from mlxlr8_b200.fast_decode import expert_mlp_finish
        from mlxlr8_b200.fast_router import router_logits

        layer = make_layer(seed=1, routed=args.experts, shared="bf16")
        e = layer.experts
        t = args.tokens
        g = torch.Generator(device="cuda")
        g.manual_seed(2)
        routed = torch.rand(t, args.experts, generator=g, device="cuda").argsort(dim=1)[:, :8].int()
        ids = torch.cat([routed, torch.full((t, 1), 256, dtype=torch.int32, device="cuda")], dim=1)
        scores = torch.rand(t, 8, generator=g, device="cuda")
        x, r = layer.tokens(t)
        for _ in range(args.calls):
            router_logits(x, layer.gate_weight)
            expert_mlp_finish(x, ids, scores, r, e.packed, e.scales, K_BITS, HIDDEN, INTER, shared=e.shared)
    elif args.ncu_driver == "encode":
        from mlxlr8_b200.joined_mxfp4 import encode

        layer = make_layer(seed=1, routed=args.experts, shared="none")
        for _ in range(args.calls):
            encode(layer.experts)
    elif args.ncu_driver == "layer":
        layer = make_layer(seed=1)
        moe = MoELayer(layer.gate_weight, layer.bias, layer.experts)
        x, r = layer.tokens(args.tokens)
        for _ in range(args.calls):
            moe(x, r)
    else:
        layer = make_layer(seed=1, routed=9, shared="none")
        e = layer.experts
        x, _ = layer.tokens(args.tokens)
        ids = torch.arange(9, dtype=torch.int32, device="cuda").repeat(args.tokens, 1)
        for _ in range(args.calls):
            fast_expert_mlp(x, ids, e.packed, e.scales, K_BITS, HIDDEN, INTER)
    torch.cuda.synchronize()
    print("ncu driver done", flush=True)


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 50 ms from just
    before the warm-up until after the last timed pass (a short timed region
    alone would often fall between two samples)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.device_index = device_index
        self.proc = None
        self.lines = []

    def start(self):
        import threading

        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        first = threading.Event()

        def reader():
            for line in self.proc.stdout:
                if line.strip():
                    self.lines.append(line)
                    first.set()

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()
        first.wait(timeout=5.0)  # the first sample lands before the measured work starts
        return self

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
            self.thread.join(timeout=5)
            self.proc = None

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in list(self.lines):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, flag in zip(names, f[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons), "samples": len(sm),
                "window": "from the warm-up before the timed steps to the end of the e2e pass, every 50 ms"}


def workload_config(args, world):
    """The config of the JSON line: identical in both arms."""
    T = args.tokens
    return {"workload": f"decode, T={T} tokens per GPU through one GLM-5-shape MoE layer (router, 256 K4 trellis "
                        f"experts, bf16 shared expert, combine)",
            "tokens_per_gpu": T, "global_batch": T * world, "hidden": HIDDEN, "intermediate": INTER,
            "experts": EXPERTS, "k_bits": K_BITS, "layers_cycled": args.layers,
            "l2": "inputs larger than L2: each step is a different layer (>233 MB touched per step)",
            "parallelism": (f"expert parallel x{world}: {EXPERTS // world} routed experts per GPU, "
                            + ("peer-memory (NVLink) dispatch/combine" if args.ep_exchange == "peer"
                               else "NCCL all-to-all dispatch/combine")
                            + ", shared expert replicated") if world > 1 else "single GPU"}


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def cpu_baseline(layer, tokens, seconds, warmup=1, steps=None):
    """Time the C restatement of the layer on host copies of one layer:
    ``warmup`` untimed calls (at least one, which sizes the sample), then
    ``steps`` timed calls, at most as many as fit in ``seconds`` (at least
    two).  Returns (timed steps, seconds, warm-up calls, threads)."""
    from mlxlr8_b200.synthetic import host_copy
    from oracle import c_oracle, trellis_oracle as ref

    x, residual = layer.tokens(tokens, seed_offset=77)
    hc = host_copy(layer)
    shared = tuple(ref.bf16_bits(s) for s in hc["shared"])
    xs, rs = x.float().cpu().numpy(), residual.float().cpu().numpy()
    args = (xs, rs, hc["gate_weight"], hc["bias"], hc["packed"], hc["scales"], K_BITS, HIDDEN, INTER, shared)
    warmup = max(1, warmup)
    for _ in range(warmup):
        t0 = time.perf_counter()
        c_oracle.moe_layer(*args)
        last = time.perf_counter() - t0
    fit = max(2, int(seconds / max(last, 1e-3)))
    steps = fit if steps is None else max(2, min(steps, fit))
    t0 = time.perf_counter()
    for _ in range(steps):
        c_oracle.moe_layer(*args)
    dt = time.perf_counter() - t0
    return steps, dt, warmup, c_oracle.threads()


def reference_arm(args, world, rank):
    """CPU restatement of the reference operators (the Metal kernels cannot
    run here), on the same workload: each step is all GPUs' tokens of one
    layer (T * N tokens)."""
    if rank != 0:
        return
    import torch

    from mlxlr8_b200.synthetic import make_layer

    # Build one layer on the GPU when present (fast seeded generation), else on CPU.
    device = "cuda" if torch.cuda.is_available() else "cpu"
    layer = make_layer(seed=1000, device=device)
    budget = 60.0
    tokens = args.tokens * world
    steps_done, dt, warm, cores = cpu_baseline(layer, tokens, budget, args.warmup, args.steps)
    value = steps_done * tokens / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": steps_done, "warmup": warm, "ms_per_step": 1000 * dt / steps_done, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{steps_done} full layer steps of {tokens} tokens after {warm} warm-up steps "
                                   f"(--steps {args.steps} requested, capped at about {budget:.0f} s)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "exlr8's expert operators are Metal compute kernels (no CPU backend); this arm is the C restatement "
                "of their arithmetic (oracle/c), timed on the host cores",
    }
    print(json.dumps(line), flush=True)


def unique_experts(ids_list):
    return [len(set(int(e) for e in ids[:, :8].reshape(-1).tolist() if e >= 0)) for ids in ids_list]


def time_calls(fn, steps, warmup, stream):
    """Milliseconds per call of fn() on `stream` (CUDA events, after warm-up)."""
    import torch

    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        e1.synchronize()
    return e0.elapsed_time(e1) / steps


def decode_batches(layers, moes, batches, steps, stream):
    """Single-GPU decode tokens/s at other batch sizes of configs[1], graph replay over the same layers."""
    import torch

    out = {}
    L = len(layers)
    for T in batches:
        xs = [layer.tokens(T, seed_offset=50 + i) for i, layer in enumerate(layers)]
        graphs = []

        def capture(i):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                moes[i](*xs[i])
            return graph

        with torch.cuda.stream(stream):
            for i in range(L):
                moes[i](*xs[i])
            torch.cuda.synchronize()
            for i in range(L):
                graphs.append(capture(i))
        state = {"s": 0}

        def replay():
            graphs[state["s"] % L].replay()
            state["s"] += 1

        ms = time_calls(replay, steps, 5, stream)
        out[f"T{T}"] = {"tokens_per_s": T / (ms / 1000.0), "ms_per_step": ms}
        graphs.clear()
    return out


def joined_decode_configs(steps, stream):
    """Decode batches on the joined MXFP4 experts (the reference's resident
    path for K4 layers, experts.py:134-148): the router + MXFP4 streaming GEMV
    chain, one CUDA graph per layer cycled over 4 layers.  GB/s counts the
    MXFP4 codes and E8M0 scales of the distinct experts touched (routed +
    the shared expert 256) per step."""
    import torch

    from mlxlr8_b200.joined_mxfp4 import JoinedMoELayer, JoinedMXFP4
    from mlxlr8_b200.synthetic import make_joined

    peak, peak_kind = measured_peaks()
    per_expert = 3 * HIDDEN * INTER // 2 + 3 * HIDDEN * INTER // 32
    layers = []
    for i in range(4):
        j = make_joined(seed=200 + i)
        layers.append((j, JoinedMoELayer(j.gate_weight, j.bias,
                                         JoinedMXFP4(j.unit, j.weights, j.scales, j.hidden, j.intermediate))))
    res = {}
    for T in (1, 8):
        xs = [j.tokens(T, seed_offset=60 + i) for i, (j, _) in enumerate(layers)]
        uniq = []
        with torch.cuda.stream(stream):
            for (j, moe), (x, r) in zip(layers, xs):
                _, ids, _ = moe(x, r, return_routing=True)
                uniq.append(len(set(int(e) for e in ids.reshape(-1).tolist())))
            torch.cuda.synchronize()
            graphs = []
            for (j, moe), (x, r) in zip(layers, xs):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    moe(x, r)
                graphs.append(g)
        state = {"s": 0}

        def replay():
            graphs[state["s"] % len(graphs)].replay()
            state["s"] += 1

        ms = time_calls(replay, steps, 5, stream)
        gbs = statistics.mean(uniq) * per_expert / (ms / 1000.0) / 1e9
        res[f"joined_T{T}"] = {"tokens_per_s": T / (ms / 1000.0), "ms_per_layer": ms,
                               "experts_touched_mean": statistics.mean(uniq), "weight_gb_per_s": gbs,
                               "frac_of_hbm": gbs / peak, "peak_kind": peak_kind,
                               "path": "gate logits -> route + plan -> prep -> MXFP4 stream (gate/up) -> gate finish -> "
                                       "MXFP4 stream (down) -> fused finish"}
        del graphs
    del layers
    torch.cuda.empty_cache()
    return res


def tensor_peaks(device):
    """tcgen05.mma throughput of the two kinds the GEMMs issue (exlr8_tensor_peak),
    M = 128, N = 128 and 256, all SMs, dense TFLOP/s."""
    import ctypes

    import torch

    from mlxlr8_b200 import _lib

    status = torch.zeros(1, dtype=torch.int32, device=device)
    out = {}
    for kind, name in ((0, "bf16"), (1, "mxf8f6f4_e4m3")):
        for n in (128, 256):
            v = ctypes.c_double(0.0)
            _lib.check(_lib.lib().exlr8_tensor_peak(kind, n, 20000, ctypes.byref(v), status.data_ptr(),
                                                     torch.cuda.current_stream(device).cuda_stream))
            if int(status.item()):
                raise RuntimeError("tensor peak probe: the bounded wait timed out")
            out[f"{name}_n{n}_tflops"] = v.value
    sink = torch.zeros(1, dtype=torch.float32, device=device)
    w = ctypes.c_double(0.0)
    _lib.check(_lib.lib().exlr8_codec_peak(4000, ctypes.byref(w), sink.data_ptr(),
                                           torch.cuda.current_stream(device).cuda_stream))
    out["trellis_codec_weights_per_s"] = w.value
    out["trellis_codec_k4_code_gbs"] = w.value * K_BITS / 8 / 1e9
    out["note"] = ("tcgen05.mma issued back to back from shared tiles on every SM (kind::f16 bf16 and "
                   "kind::mxf8f6f4.block_scale E4M3 x E4M3), CUDA events; the trellis codec figure runs the decode "
                   "GEMV's inner loop (exact K4 decode + mma.sync) on codes in shared memory at the stream kernel's "
                   "occupancy: the compute ceiling of the decode; no clock or power changes")
    return out


def prefill_configs(layer_k4, steps, stream, peak_tflops, mx_peak_tflops=None):
    """configs[2] (joined MXFP4, 4096 tokens) and configs[4] (128 tokens, K4 and the K3 layer-78 width)."""
    import torch

    from mlxlr8_b200 import _lib
    from mlxlr8_b200.joined_mxfp4 import JoinedMoELayer, JoinedMXFP4
    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.synthetic import make_joined, make_layer

    res = {}
    j = make_joined(seed=5)
    joined = JoinedMoELayer(j.gate_weight, j.bias, JoinedMXFP4(j.unit, j.weights, j.scales, j.hidden, j.intermediate))
    x, r = j.tokens(4096)
    ms = time_calls(lambda: joined(x, r), steps, 3, stream)
    with torch.cuda.stream(stream):
        _lib.profile_enable(True)
        joined(x, r)
        torch.cuda.synchronize()
        prof = _lib.profile_read()
        _lib.profile_enable(False)
    gemm_ms = prof["gate_up"][1] + prof["down"][1]
    flops = 2.0 * 4096 * 9 * 3 * HIDDEN * INTER  # routed + shared slot, gate/up/down
    res["joined_mxfp4_T4096"] = {
        "tokens_per_s": 4096 / (ms / 1000.0), "ms_per_layer": ms,
        "useful_tflops": flops / (ms / 1000.0) / 1e12,
        "gemm_ms": gemm_ms, "gemm_useful_tflops": flops / (gemm_ms / 1000.0) / 1e12,
        "gemm_frac_of_bf16_peak": flops / (gemm_ms / 1000.0) / 1e12 / peak_tflops,
        "mxf8f6f4_peak_tflops": mx_peak_tflops,
        "gemm_frac_of_mxf8f6f4_peak_useful": (flops / (gemm_ms / 1000.0) / 1e12 / mx_peak_tflops
                                              if mx_peak_tflops else None),
        "gemm_frac_of_mxf8f6f4_peak_issued": (2 * flops / (gemm_ms / 1000.0) / 1e12 / mx_peak_tflops
                                              if mx_peak_tflops else None),
        "kernel_ms": {k: v[1] for k, v in prof.items() if v[0]},
        "note": "block-scaled tcgen05 MMA (kind::mxf8f6f4, E2M1 weights x E4M3 hi/lo activations); useful FLOPs "
                "count each product once (the hi/lo planes issue twice as many MMA FLOPs)"}
    del joined, j, x, r
    torch.cuda.empty_cache()
    for k, layer in (("k4", layer_k4), ("k3", None)):
        if layer is None:
            layer = make_layer(seed=78, k=3)
        moe = MoELayer(layer.gate_weight, layer.bias, layer.experts)
        x, r = layer.tokens(128, seed_offset=9)
        ms = time_calls(lambda: moe(x, r), steps, 3, stream)
        res[f"trellis_{k}_T128"] = {"tokens_per_s": 128 / (ms / 1000.0), "ms_per_layer": ms,
                                     "path": "grouped tcgen05 GEMM with in-kernel trellis decode"}
        del moe
    torch.cuda.empty_cache()
    return res


def encode_config(layer, steps, stream):
    """Load-time trellis -> MXFP4 re-encode of one K4 layer's 256 routed
    experts (joined_mxfp4.py:12-47): three fused decode + fold +
    quantise launches (gate and up into the joined [E, 2m, h/8] buffer, then
    down).  Algorithmic bytes: the packed codes and gate/up in-scales read,
    the MXFP4 codes and E8M0 scales written."""
    from mlxlr8_b200.joined_mxfp4 import encode

    e = layer.experts
    matrices = e.packed["gate"].numel() // (HIDDEN * INTER * K_BITS // 8)
    read = sum(t.numel() for t in e.packed.values()) + 2 * matrices * HIDDEN * e.scales["gate"][0].element_size()
    written = matrices * (3 * HIDDEN * INTER // 2 + 3 * HIDDEN * INTER // 32)
    ms = time_calls(lambda: encode(e), steps, 2, stream)
    peak, peak_kind = measured_peaks()
    achieved = (read + written) / (ms / 1000.0) / 1e9
    return {"ms_per_layer": ms, "matrices": matrices, "bytes_read": read, "bytes_written": written,
            "achieved_gbs": achieved, "peak_gbs": peak, "peak_kind": peak_kind, "frac": achieved / peak,
            "kernel": "mxfp4_encode_trellis_kernel (3 launches per layer)"}


def static_cache_config(layer, steps, stream):
    """Static hot-expert cache (static_cache.py:91-134): the selected-
    expert MLP of one decode token over eight routed experts, all cached as
    exact E4M3 bytes, against the same call decoding their trellis codes.  Two
    disjoint expert sets alternate, so no call finds its weights in L2.
    Algorithmic bytes: the weight bytes streamed (3 * h * m per cached expert,
    K * h * m * 3 / 8 per coded one)."""
    import torch

    from mlxlr8_b200.fast_decode import fast_expert_mlp
    from mlxlr8_b200.static_cache import StaticExpertCache

    e = layer.experts
    sets = [list(range(0, 8)), list(range(8, 16))]
    cache = StaticExpertCache(e, sets[0] + sets[1])
    idx = [torch.tensor([s], dtype=torch.int32, device="cuda") for s in sets]
    x, _ = layer.tokens(1, seed_offset=91)
    turn = [0]

    def call(cached):
        i = turn[0] = turn[0] ^ 1
        if cached:
            return fast_expert_mlp(x, idx[i], e.packed, e.scales, e.k, e.hidden, e.intermediate, fp8=cache.fp8,
                                   expert_to_slot=cache.expert_to_slot)
        return fast_expert_mlp(x, idx[i], e.packed, e.scales, e.k, e.hidden, e.intermediate)

    coded_ms = time_calls(lambda: call(False), steps, 3, stream)
    cached_ms = time_calls(lambda: call(True), steps, 3, stream)
    peak, peak_kind = measured_peaks()
    cached_bytes = 8 * 3 * HIDDEN * INTER
    coded_bytes = 8 * 3 * HIDDEN * INTER * K_BITS // 8
    del cache
    torch.cuda.empty_cache()
    return {"experts": 8, "coded_ms": coded_ms, "cached_ms": cached_ms,
            "coded_weight_gbs": coded_bytes / (coded_ms / 1000.0) / 1e9,
            "cached_weight_gbs": cached_bytes / (cached_ms / 1000.0) / 1e9,
            "cached_frac_of_hbm": cached_bytes / (cached_ms / 1000.0) / 1e9 / peak, "peak_kind": peak_kind}


def loader_config():
    """EXLR8 checkpoint -> device (experts.py:77-148): one
    full-size K4 layer (256 routed experts + shared, 4.85 GB of codes) written
    to a scratch directory, then ``ExpertStore(resident=True).layer(3)`` timed
    on the host clock around the load (and a device synchronize): read only
    (``optimize=False``) and read + joined MXFP4 re-encode (``optimize=True``,
    the reference's load path).  The files are dropped from the page cache
    before each load (posix_fadvise DONTNEED), so the read comes from the
    disk, not from memory."""
    import shutil
    import tempfile

    import torch

    from mlxlr8_b200.experts import ExpertStore
    from mlxlr8_b200.synthetic import write_checkpoint

    scratch = Path(tempfile.mkdtemp(prefix="exlr8-ckpt-"))
    try:
        free = shutil.disk_usage(scratch).free
        routed = 256 if free > 12 * 2**30 else max(8, int(free / 2**30 / 12 * 256) // 8 * 8)
        write_checkpoint(scratch, layers=(3,), routed=routed, seed=9)
        files = sorted(p for p in scratch.rglob("*.safetensors"))
        total = sum(p.stat().st_size for p in files)
        res = {"routed_experts": routed, "file_bytes": total}
        for optimize in (False, True):
            for p in files:
                fd = os.open(p, os.O_RDONLY)
                os.fsync(fd)
                os.posix_fadvise(fd, 0, 0, os.POSIX_FADV_DONTNEED)
                os.close(fd)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            store = ExpertStore(scratch, resident=True, optimize=optimize)
            store.layer(3)
            torch.cuda.synchronize()
            dt = time.perf_counter() - t0
            key = "read_and_reencode" if optimize else "read"
            res[key] = {"seconds": dt, "file_gb_per_s": total / dt / 1e9,
                        "resident_bytes": store.stats()["resident_bytes"]}
            del store
            torch.cuda.empty_cache()
        return res
    finally:
        shutil.rmtree(scratch, ignore_errors=True)


def stack_configs(layers, steps, stream):
    """The MoE block stack with the attention stubbed (model.py:373-418): the bench's
    layers (K4) plus the K3 layer-78 block, each behind its post-attention RMS
    norm, as one CUDA graph per stack call.  T = 1 (decode) and T = 128 with
    Zipf(1.1)-skewed routing (configs[4], the speculative-verify step)."""
    import torch

    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.stack import MoEStack
    from mlxlr8_b200.synthetic import make_layer, zipf_bias

    k3 = make_layer(seed=78, k=3)
    blocks = list(layers) + [k3]
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    norms = [(1.0 + 0.1 * torch.randn(HIDDEN, generator=g, device="cuda")).to(torch.bfloat16) for _ in blocks]
    res = {}
    for tokens, skew in ((1, False), (128, True)):
        moes = [MoELayer(l.gate_weight, zipf_bias(300 + i) if skew else l.bias, l.experts)
                for i, l in enumerate(blocks)]
        stack = MoEStack(list(zip(norms, moes)))
        h = (torch.randn(tokens, HIDDEN, generator=g, device="cuda")).to(torch.bfloat16)
        stream.wait_stream(torch.cuda.current_stream())  # weights and h come from the default stream
        with torch.cuda.stream(stream):
            for _ in range(2):
                stack(h)  # eager warm-up: workspaces, kernel attributes
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            stack(h)
        ms = time_calls(graph.replay, steps, 3, stream)
        del graph
        res[f"stack_{len(blocks)}blocks_T{tokens}"] = {
            "tokens_per_s": tokens / (ms / 1000.0), "ms_per_stack": ms, "ms_per_block": ms / len(blocks),
            "blocks": f"{len(layers)} K4 blocks + the K3 layer-78 block, post-attention RMS norm each",
            "routing": "Zipf(1.1)-skewed router bias" if skew else "uniform"}
        del stack, moes
    del k3
    torch.cuda.empty_cache()
    return res


def measured_bandwidths():
    """(HBM GB/s, kind) and the peer-store figure used for NVLink."""
    hbm, kind = measured_peaks()
    return hbm, kind


def peer_store_bandwidth(world, rank, device, nbytes=256 << 20, reps=20):
    """Per-direction NVLink store bandwidth: every rank writes `nbytes` into
    the next rank's buffer (CUDA IPC mapping, 16-byte SM stores, the exchange
    kernels' store path) at the same time; GB/s per GPU, min over ranks."""
    import ctypes

    import torch
    import torch.distributed as dist

    from mlxlr8_b200 import _lib

    lib = _lib.lib()
    region = ctypes.c_void_p()
    handle = (ctypes.c_ubyte * 64)()
    _lib.check(lib.exlr8_ep_peer_create(nbytes, ctypes.byref(region), handle))
    mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
    handles = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(handles, mine)
    nxt = (rank + 1) % world
    theirs = (ctypes.c_ubyte * 64).from_buffer_copy(bytes(handles[nxt].cpu().tolist()))
    peer = ctypes.c_void_p()
    _lib.check(lib.exlr8_ep_peer_open(theirs, ctypes.byref(peer)))
    src = torch.empty(nbytes, dtype=torch.uint8, device=device).fill_(rank)
    stream = torch.cuda.current_stream(device).cuda_stream
    for _ in range(3):
        _lib.check(lib.exlr8_peer_write(peer.value, src.data_ptr(), nbytes, stream))
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        _lib.check(lib.exlr8_peer_write(peer.value, src.data_ptr(), nbytes, stream))
    e1.record()
    e1.synchronize()
    gbs = torch.tensor([nbytes * reps / (e0.elapsed_time(e1) / 1000.0) / 1e9], device=device)
    dist.all_reduce(gbs, op=dist.ReduceOp.MIN)
    torch.cuda.synchronize()
    dist.barrier()
    _lib.check(lib.exlr8_ep_peer_close(peer.value))
    dist.barrier()
    _lib.check(lib.exlr8_ep_peer_destroy(region.value))
    return float(gbs.item())


def ep_stack(args, world, rank, device, stream):
    """The 75-layer expert stack at a fixed global batch (strong scaling)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from mlxlr8_b200 import _lib
    from mlxlr8_b200.fast_router import router
    from mlxlr8_b200.stack import MoEStack, residual_rms_norm
    from mlxlr8_b200.synthetic import make_shard

    G = args.stack_batch
    if G % world:
        return {"error": f"global batch {G} does not divide over {world} GPUs"}
    T = G // world
    per = EXPERTS // world
    codes = HIDDEN * INTER * K_BITS // 8
    per_layer = per * 3 * codes + per * 49152 + 3 * HIDDEN * INTER * 2 + 256 * HIDDEN * 4
    resident = max(1, min(args.stack_layers, int(args.stack_budget_gb * 1e9 // per_layer)))
    shards = [make_shard(seed=5000 + 31 * i, rank=rank, world=world, device=device) for i in range(resident)]
    peer = None
    if world == 1:
        from mlxlr8_b200.moe import MoELayer

        moes = [MoELayer(sh.gate_weight, sh.bias, sh.experts) for sh in shards]
    else:
        from mlxlr8_b200.ep import ExpertParallelMoE, PeerExchange

        peer = PeerExchange(world, rank, HIDDEN, T, torch.bfloat16, device)
        moes = [ExpertParallelMoE(sh.gate_weight, sh.bias, sh.experts, rank, world, shared=sh.shared,
                                  exchange="peer", max_tokens=T, peer=peer) for sh in shards]
    g = torch.Generator(device=device)
    g.manual_seed(77)
    norms = [(1.0 + 0.1 * torch.randn(HIDDEN, generator=g, device=device)).to(torch.bfloat16)
             for _ in range(args.stack_layers)]
    stack = MoEStack([(norms[i], moes[i % resident]) for i in range(args.stack_layers)])
    g.manual_seed(1000 + rank)
    h0 = torch.randn(T, HIDDEN, generator=g, device=device).to(torch.bfloat16)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # Eager pass: workspaces, kernel attributes, the exchange's first epochs.
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        stack(h0)
    barrier()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        stack(h0)
    barrier()
    with torch.cuda.stream(stream):
        for _ in range(2):
            graph.replay()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.stack_steps):
            graph.replay()
        e1.record(stream)
    e1.synchronize()
    barrier()
    ms = e0.elapsed_time(e1) / args.stack_steps
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        peer.check()

    # Per-phase device time of one eager stack step (events around each library
    # launch), the max over ranks per phase; and the routing of every block.
    with torch.cuda.stream(stream):
        _lib.profile_enable(True, capacity=args.stack_layers * 24 + 64)
        _, trace = stack(h0, trace=True)
        torch.cuda.synchronize()
        prof = _lib.profile_read()
        _lib.profile_enable(False)
    kinds = list(prof)
    phase = torch.tensor([prof[k][1] for k in kinds], dtype=torch.float64, device=device)
    launches = sum(n for n, _ in prof.values())
    if world > 1:
        dist.all_reduce(phase, op=dist.ReduceOp.MAX)
    phase_ms = {k: round(float(v), 4) for k, v in zip(kinds, phase.tolist()) if v > 0}
    hbm_bw, hbm_kind = measured_bandwidths()
    nvl_bw = peer_store_bandwidth(world, rank, device) if world > 1 else None
    ideal_s, hbm_bytes_total, nvl_bytes_total = 0.0, 0.0, 0.0
    u_owned = []
    for i in range(min(resident, args.stack_layers)):
        _, xn, _ = trace[i]
        sh = shards[i]
        ids = router(xn, sh.gate_weight, sh.bias)[1][:, :8].contiguous()
        if world > 1:
            parts = [torch.empty_like(ids) for _ in range(world)]
            dist.all_gather(parts, ids)
            every = torch.stack(parts).cpu().numpy()  # [src rank][token][8]
        else:
            every = ids.cpu().numpy()[None]
        owner = every // per
        worst = 0.0
        for r in range(world):
            mine = np.unique(every[owner == r])
            u_owned.append(len(mine))
            hbm = len(mine) * (3 * codes + 49152) + 3 * HIDDEN * INTER * 2 + 256 * HIDDEN * 4 + 4 * T * HIDDEN
            # rows r sends to other owners plus rows others send to r, each way one bf16 row
            sent = int(((owner[r] != r)).sum())
            received = int(sum(((owner[q] == r)).sum() for q in range(world) if q != r))
            nvl = (sent + received) * HIDDEN * 2
            t_hbm = hbm / (hbm_bw * 1e9)
            t_nvl = nvl / (nvl_bw * 1e9) if nvl_bw else 0.0
            worst = max(worst, t_hbm, t_nvl)
            hbm_bytes_total += hbm
            nvl_bytes_total += nvl
        ideal_s += worst
    layers_sampled = min(resident, args.stack_layers)
    ideal_step_ms = ideal_s / layers_sampled * args.stack_layers * 1000.0
    del graph, stack, moes, shards, trace
    torch.cuda.synchronize()
    if peer is not None:
        peer.close()
    torch.cuda.empty_cache()
    return {
        "tokens_per_s": G / (ms / 1000.0), "ms_per_step": ms, "global_batch": G, "tokens_per_gpu": T,
        "layers": args.stack_layers, "resident_layers": resident,
        "layers_note": ("all layers resident" if resident >= args.stack_layers else
                        f"{resident} distinct layers resident (75 do not fit at {per} experts per GPU); the stack cycles "
                        "them, each layer > L2, so no step reuses cached weights"),
        "steps": args.stack_steps, "scaling": "strong",
        "parallelism": (f"expert parallel x{world}, {per} routed experts per GPU, peer-memory exchange"
                        if world > 1 else "single GPU, fused layer (grouped GEMM path at 64 tokens)"),
        "phase_ms_per_step": phase_ms, "library_launches_per_step": launches,
        "roofline": {"ideal_ms_per_step": ideal_step_ms, "frac": ideal_step_ms / ms,
                     "hbm_gbs": hbm_bw, "hbm_kind": hbm_kind, "nvlink_store_gbs": nvl_bw,
                     "owned_experts_touched_mean": float(np.mean(u_owned)),
                     "owned_experts_touched_max": int(np.max(u_owned)),
                     "definition": "per layer max over ranks of max(HBM bytes / HBM GB/s, NVLink bytes / peer-store "
                                   "GB/s); HBM bytes = owned experts touched x 3 K4 matrices + scales + shared expert + "
                                   "router + activations; NVLink bytes = bf16 rows this rank sends and receives"},
    }


def main():
    args = parse()
    if args.ncu_driver:
        ncu_driver(args)
        return
    if args.peaks:
        import torch

        torch.cuda.set_device(0)
        print(json.dumps(tensor_peaks(torch.device("cuda", 0))), flush=True)
        return
    world, rank, local = dist_setup()
    if args.impl == "reference":
        reference_arm(args, world, rank)
        return
    import numpy as np
    import torch
    import torch.distributed as dist

    from mlxlr8_b200 import _lib
    from mlxlr8_b200.moe import MoELayer
    from mlxlr8_b200.synthetic import make_layer

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", device_id=device)
    T, L = args.tokens, args.layers

    # Every rank builds the same seeded layers; with N > 1 it keeps its block
    # of 256 / N routed experts (expert parallelism) and the shared expert,
    # and draws its own tokens.
    layers, moes, xs, rs = [], [], [], []
    for i in range(L):
        layer = make_layer(seed=1000 + 97 * i, device=device)
        if world == 1:
            moes.append(MoELayer(layer.gate_weight, layer.bias, layer.experts))
        else:
            from mlxlr8_b200.ep import ExpertParallelMoE, shard_experts

            shard = shard_experts(layer.experts, rank, world)
            for p in ("gate", "up", "down"):
                shard.packed[p] = shard.packed[p].clone()
            moes.append(ExpertParallelMoE(layer.gate_weight, layer.bias, shard, rank, world,
                                          shared=layer.experts.shared, exchange=args.ep_exchange, max_tokens=T))
        x, r = layer.tokens(T, seed_offset=i * world + rank)
        xs.append(x)
        rs.append(r)
        if world > 1:
            del layer.experts.packed  # only the shard stays resident
        layers.append(layer)
    torch.cuda.synchronize()
    if world > 1:
        # One eager call per layer, in the same order on every rank: the
        # peer-memory exchange maps its regions (a collective) on first use.
        for i in range(L):
            moes[i](xs[i], rs[i])
        torch.cuda.synchronize()

    # CUDA graphs of one layer call each (inputs resident in HBM); with several
    # GPUs the graphs hold the NCCL exchange too.  Graph references live only
    # in `graphs`, which is cleared before the process group goes away.
    outs, graphs = [], []
    stream = torch.cuda.Stream(device)

    def capture(i):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            outs.append(moes[i](xs[i], rs[i]))
        return graph

    with torch.cuda.stream(stream):
        for i in range(L):
            moes[i](xs[i], rs[i])  # allocate the cached workspace before capture
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        for i in range(L):
            graphs.append(capture(i))
    torch.cuda.synchronize()

    def step(s):
        if graphs:
            graphs[s % L].replay()
        else:
            moes[s % L](xs[s % L], rs[s % L])

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- headline: graph replay, device-resident inputs ----
    clocks = ClockSampler(local).start()
    with torch.cuda.stream(stream):
        for s in range(args.warmup):
            step(s)
    barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for s in range(args.steps):
            step(s)
        stop.record(stream)
    stop.synchronize()
    barrier()
    elapsed = start.elapsed_time(stop)
    if world > 1:
        t = torch.tensor([elapsed], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = float(t.item())
    ms_per_step = elapsed / args.steps
    value = world * T * args.steps / (elapsed / 1000.0)
    for m in moes:  # a peer exchange that timed out or lost slots invalidates the run
        if getattr(m, "peer", None) is not None:
            m.peer.check()

    # ---- profiled pass: per-kernel CUDA events on the launching stream ----
    routing = []
    with torch.cuda.stream(stream):
        for s in range(min(args.warmup, L)):
            moes[s % L](xs[s % L], rs[s % L])
        torch.cuda.synchronize()
        prof_steps = min(args.steps, 400)
        _lib.profile_enable(True, capacity=prof_steps * 16 + 64)
        for s in range(prof_steps):
            moes[s % L](xs[s % L], rs[s % L])
        torch.cuda.synchronize()
        prof = _lib.profile_read()
        _lib.profile_enable(False)
        for i in range(L):
            _, ids, _ = moes[i](xs[i], rs[i], return_routing=True)
            ids_np = ids.cpu().numpy()
            if world > 1:  # this rank streams the experts it owns, of every rank's tokens
                per = EXPERTS // world
                parts = [torch.empty_like(ids) for _ in range(world)]
                dist.all_gather(parts, ids)
                ids_np = torch.cat(parts).cpu().numpy()
                ids_np = np.where((ids_np // per) == rank, ids_np, -1)
            routing.append(ids_np)
    launches_per_step = sum(n for n, _ in prof.values()) / max(prof_steps, 1)
    u = unique_experts(routing)
    u_mean = sum(u) / len(u)
    codes_per_matrix = HIDDEN * INTER * K_BITS // 8
    gate_up_n, gate_up_ms = prof["gate_up"]
    gate_up_avg_ms = gate_up_ms / max(gate_up_n, 1)
    # The single-GPU layer streams the bf16 shared expert's gate/up rows in the
    # same launch (its dense warp); expert-parallel ranks run it separately.
    dense_bytes = DENSE_GATE_UP_BYTES if world == 1 else 0
    gate_up_bytes = u_mean * 2 * codes_per_matrix + dense_bytes
    achieved = gate_up_bytes / (gate_up_avg_ms / 1000.0) / 1e9
    peak, peak_kind = measured_peaks()
    share = {k: round(ms / max(sum(v for _, v in prof.values()), 1e-9), 4) for k, (n, ms) in prof.items()}

    # The trellis decode's compute ceiling on this GPU (codes held in shared
    # memory): the codes part of the dominant launch against it.
    codec_ceiling = None
    try:
        import ctypes

        sink = torch.zeros(1, dtype=torch.float32, device=device)
        w = ctypes.c_double(0.0)
        _lib.check(_lib.lib().exlr8_codec_peak(4000, ctypes.byref(w), sink.data_ptr(),
                                               torch.cuda.current_stream(device).cuda_stream))
        codec_ceiling = w.value * K_BITS / 8 / 1e9
    except Exception:  # noqa: BLE001 - the line carries null then
        codec_ceiling = None
    codes_gbs = u_mean * 2 * codes_per_matrix / (gate_up_avg_ms / 1000.0) / 1e9

    # Whole-step algorithmic bytes (codes, scales, shared expert, router, activations) for context.
    step_bytes = u_mean * 3 * codes_per_matrix + u_mean * 49152 + 3 * HIDDEN * INTER * 2 + 256 * HIDDEN * 4 + 4 * T * HIDDEN

    # ---- e2e through the public API with host buffers ----
    # The layer call (MoELayer, or ExpertParallelMoE on several GPUs) with
    # pinned host x, residual and out, in its graph-replay mode: the graph's
    # first kernel reads the inputs over PCIe and the combine writes the
    # result to the pinned out (no copy-engine transfer in the chain).  Each
    # layer's graph is captured by the priming pass below, before the warm-up,
    # in the same order on every rank.
    xh = [x.cpu().pin_memory() for x in xs]
    rh = [r.cpu().pin_memory() for r in rs]
    oh = [torch.empty(T, HIDDEN, dtype=torch.bfloat16).pin_memory() for _ in range(L)]
    e2e_steps = min(args.steps, 1000)

    def e2e_step(i):
        moes[i](xh[i], rh[i], out=oh[i], graph=True)

    with torch.cuda.stream(stream):
        for i in range(L):
            e2e_step(i)  # priming: every layer's first call and its graph capture
        for s in range(args.warmup):
            e2e_step(s % L)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for s in range(e2e_steps):
            e2e_step(s % L)
        e1.record(stream)
        e1.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * T * e2e_steps / (e2e_ms / 1000.0)
    h2d = 2 * T * HIDDEN * 2
    d2h = T * HIDDEN * 2
    clocks.stop()

    extras = {}
    if world == 1 and not args.no_extras:
        extras["decode_batches"] = decode_batches(layers, moes, [4, 8, 32], min(args.steps, 200), stream)
        bf16_peak = 1645.3
        peaks_path = ROOT / "MEASURED_PEAKS.json"
        if peaks_path.exists():
            bf16_peak = float(json.loads(peaks_path.read_text()).get("bf16_tflops", bf16_peak))
        try:
            extras["tensor_peaks"] = tensor_peaks(device)
            mx_peak = extras["tensor_peaks"]["mxf8f6f4_e4m3_n256_tflops"]
        except Exception as exc:  # noqa: BLE001 - reported in the JSON line
            extras["tensor_peaks"] = {"error": f"{type(exc).__name__}: {exc}"}
            mx_peak = None
        extras["prefill"] = prefill_configs(layers[0], 10, stream, bf16_peak, mx_peak)
        extras["stack"] = stack_configs(layers, 20, stream)
        extras["joined_decode"] = joined_decode_configs(min(args.steps, 200), stream)
        extras["encode"] = encode_config(layers[0], 5, stream)
        try:  # a failure here must not cost the lines above
            extras["static_cache"] = static_cache_config(layers[0], min(args.steps, 200), stream)
        except Exception as exc:  # noqa: BLE001 - reported in the JSON line
            extras["static_cache"] = {"error": f"{type(exc).__name__}: {exc}"}
        extras["loader"] = loader_config()

    if not args.no_stack:
        # The headline's layers and graphs make room for the stack's resident layers.
        graphs.clear()
        outs.clear()
        for m in moes:
            m.clear_graphs()
            if getattr(m, "peer", None) is not None:
                m.peer.close()
        del moes[:]
        if world > 1:
            del layers[:]
        else:
            del layers[1:]
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        try:
            extras["ep_stack"] = ep_stack(args, world, rank, device, stream)
        except Exception as exc:  # noqa: BLE001 - reported in the JSON line
            extras["ep_stack"] = {"error": f"{type(exc).__name__}: {exc}"}
            if world > 1:
                raise

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        steps_done, dt, _, cores = cpu_baseline(layers[0], T, args.cpu_seconds)
        cpu = {"value": steps_done * T / dt, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"{steps_done} full layer steps of T={T} on host copies of one layer"}

    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": workload_config(args, world),
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps},
            "roofline": {"bound": "hbm", "kernel": ("trellis_stream_kernel<4> (gate/up" +
                                                    (" + bf16 shared gate/up rows)" if dense_bytes else ")")),
                         "achieved": achieved, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": TRAFFIC_PER_MATRIX * 2 * u_mean + dense_bytes,
                         "algorithmic_bytes_per_launch": gate_up_bytes, "avg_launch_ms": gate_up_avg_ms,
                         "unique_experts_mean": u_mean,
                         "codes_gbs": codes_gbs, "codec_ceiling_gbs": codec_ceiling,
                         "frac_of_codec_ceiling": codes_gbs / codec_ceiling if codec_ceiling else None,
                         "codec_ceiling_note": "exlr8_codec_peak: the exact K4 decode + mma.sync on codes in shared "
                                               "memory at the kernel's occupancy; the decode cannot stream codes "
                                               "faster than this on this GPU"},
            "step_roofline": {"algorithmic_bytes": step_bytes, "achieved_gbs": step_bytes / (ms_per_step / 1000) / 1e9,
                              "frac": step_bytes / (ms_per_step / 1000) / 1e9 / peak},
            "kernel_share": share,
            "gpu_launches": int(round(launches_per_step * args.steps)),
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        line.update(extras)
        print(json.dumps(line), flush=True)
    # Release graphs (they hold NCCL work) before tearing down the process group.
    graphs.clear()
    outs.clear()
    for m in moes:
        m.clear_graphs()
    torch.cuda.synchronize()
    if world > 1:
        for m in moes:
            if getattr(m, "peer", None) is not None and m.peer.region is not None:
                m.peer.close()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
