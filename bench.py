"""Benchmark: µs per fused MoE layer and achieved HBM GB/s (decode, bs=1).

python bench.py [--gpus N] [--steps K] [--warmup W] [--config mixtral|deepseek|dbrx|tiny]
                [--parallel tp|ep] [--impl ours|reference] [--extra-configs deepseek,dbrx]

One step = one MoE layer forward for one decode token (router -> top-K ->
SwiGLU over the selected experts -> weighted combine; plus the hidden-sized
all-reduce when N > 1).  The default workload is the Mixtral-shaped layer
(H 4096, I 14336, E 8, top_k 2, bf16 weights, fp32 accumulation/output),
tensor-parallel over N GPUs.  Inputs are synthetic and seeded; layers rotate
so every step streams weights from HBM (each step reads more than L2 holds).

Rank 0 prints one JSON line.  `value` is µs per layer (max over ranks, CUDA
events on the launching stream; the timed steps replay a CUDA graph of the
layer calls; at N > 1 every rank's region starts behind a device-side
rendezvous, so host skew between ranks is not charged to it); `e2e` is the
same through the public API with the token copied in from pinned host memory
and the output copied back every step (copies on their own streams,
overlapping the kernels; the steps replayed from CUDA graphs of 64 steps, or
eagerly with --no-graph); `roofline` relates the fused kernel's algorithmic
bytes to the measured HBM copy bandwidth; `parity` checks a sampled layer,
run through the timed path, against warp-route's CPU composition (and, at
N > 1, against the whole layer on rank 0's GPU, plus bit-identity across the
ranks); `cpu_baseline` times that CPU composition (restated in
oracle/torch_composition.py) on a bounded sample.  `other_configs` carries the
same measurement for the DeepSeek- and DBRX-shaped layers (expert parallel at
N > 1).  `--impl reference` times the CPU composition alone, as the reference
arm.

The line also carries `batched_sweep`: the batched-decode sweep on
the Mixtral shape (tokens 1, 4, 16, 64, 256; router bias N(0,1) per expert to
skew the load; 32 stacked layers with independent weights, each applied to
the same seeded token batch), µs per layer from CUDA-graph replays of the 32
layer calls.  Batches of two or more bf16 tokens run on the grouped
tensor-core path (tcgen05 GEMMs over tokens bucketed per expert).  At N > 1
the sweep is expert parallel (E/N experts of every layer per GPU) with one
NCCL all-reduce of the layer output, both inside the replayed graph.
`batched_sweep_fp32` is the same sweep in fp32, warp-route's own dtype
(tokens 16 and 64, 8 stacked layers of 5.6 GB): batches of three or more fp32
tokens take the grouped path with the weights split into bf16 hi and lo
parts in shared memory.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
# NCCL's version banner would land on stdout ahead of the one JSON line
os.environ.setdefault("NCCL_DEBUG", "WARN")
sys.path.insert(0, os.path.join(REPO, "warp-route_b200"))

import torch  # noqa: E402

METRIC = "µs per MoE layer & achieved HBM GB/s, Mixtral shape bs=1, at 1/2/4/8 B200"
SHAPES = {"tiny": (8, 512, 1024, 2), "mixtral": (8, 4096, 14336, 2),
          "deepseek": (64, 2048, 1408, 6), "dbrx": (16, 6144, 10752, 4)}
L2_BYTES = 126 * 1024 * 1024
E2E_CHUNK = 64  # e2e steps per captured graph


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--config", default="mixtral", choices=sorted(SHAPES))
    ap.add_argument("--parallel", default="tp", choices=["tp", "ep"])
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "fp32"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="budget of the bounded CPU-baseline sample")
    ap.add_argument("--allreduce", default="fused", choices=["fused", "nccl"],
                    help="N > 1: sum the ranks' outputs inside the layer kernel over NVLink peer "
                         "memory (fused) or with a separate NCCL all-reduce after it")
    ap.add_argument("--no-graph", action="store_true",
                    help="time the layer calls eagerly instead of replaying a CUDA graph of them")
    ap.add_argument("--layers", type=int, default=0,
                    help="rotating layers (0: enough to exceed 4x L2 between reuses)")
    ap.add_argument("--sweep-tokens", default="1,4,16,64,256",
                    help="batched-decode sweep token counts; empty: no sweep")
    ap.add_argument("--sweep-layers", type=int, default=32)
    ap.add_argument("--fp32-sweep-tokens", default="16,64",
                    help="the same sweep in fp32 (warp-route's dtype); empty: none")
    ap.add_argument("--fp32-sweep-layers", type=int, default=8)
    ap.add_argument("--sweep-steps", type=int, default=3)
    ap.add_argument("--sweep-fused-allreduce", action="store_true",
                    help="N > 1: sum the sweep's batch outputs in the layer's combine step "
                         "over NVLink peer memory instead of NCCL (needs --allreduce fused)")
    ap.add_argument("--extra-configs", default="deepseek,dbrx",
                    help="other BASELINE configurations measured in the same run (expert "
                         "parallel at N > 1), reported under other_configs; empty: none")
    ap.add_argument("--decode-layers", type=int, default=32,
                    help="layers of the timed decode step (Mixtral shape, one token, tensor "
                         "parallel at N > 1); 0: no decode step")
    ap.add_argument("--decode-steps", type=int, default=5)
    ap.add_argument("--only-sweep", action="store_true",
                    help="run only the batched-decode sweep (N = 1) and print its JSON line")
    ap.add_argument("--profile-layer", default="",
                    help="CONFIG:T or ExHxIxK:T — run that layer (in --dtype, router bias when "
                         "top_k < E) three times eagerly on one GPU and exit: the case the "
                         "profiles/ ncu captures use")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ncu_traffic(workload: str):
    """DRAM bytes per launch of the fused kernel from a committed ncu summary."""
    try:
        with open(os.path.join(REPO, "profiles", "ncu_traffic.json")) as f:
            return json.load(f).get(workload)
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100", "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, busy_only=True):
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        try:
            rows = [r.split(",") for r in open(self.path).read().strip().splitlines() if r.strip()]
        except Exception:
            return out
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm, mx, reasons = [], [], set()
        for r in rows:
            r = [c.strip() for c in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if sm:
            out.update(sm_mhz=statistics.median(sm), sm_max_mhz=max(mx), samples=len(sm))
        out["reasons"] = sorted(reasons)
        try:
            os.unlink(self.path)
        except OSError:
            pass
        return out


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and args.impl == "ours":
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    return world, rank, local


# ---------------------------------------------------------------------------
# CPU composition (warp-route's own CPU path, restated in oracle/): the CPU
# baseline, the reference arm and the parity checker of the bench line
# ---------------------------------------------------------------------------
def _composition():
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import torch_composition as tc
    return tc


def _host_experts(weight_buf, E, H, I, sel, dtype):
    """Host copies (in `dtype`) of the selected experts' [gate, up, down]."""
    elt = weight_buf.element_size()
    stride = ((3 * H * I * elt + 127) // 128 * 128) // elt
    n = I * H
    gate, up, down = [None] * E, [None] * E, [None] * E
    for e in sel:
        blk = weight_buf[e * stride:e * stride + 3 * n].to(dtype).cpu()
        gate[e] = blk[:n].view(I, H)
        up[e] = blk[n:2 * n].view(I, H)
        down[e] = blk[2 * n:].view(H, I)
    return gate, up, down


def cpu_composition_timing(x, gate_w, weight_buf, E, H, I, K, budget_s, max_calls=None,
                           bias=None, threads=None, dtype=torch.float32, warmup=3):
    """Time the restated torch_moe_reference on host threads: median µs per
    single-token forward over a bounded sample (at most `budget_s` seconds or
    `max_calls` calls, after `warmup` untimed calls).  Weights are the same
    layer's selected experts in `dtype` (float32 is warp-route's own dtype;
    the layer's bf16 values widen exactly).  Returns (µs, calls, threads)."""
    tc = _composition()
    threads = threads or (os.cpu_count() or 1)
    torch.set_num_threads(threads)
    xh = x.detach().to(dtype).cpu()
    gwh = gate_w.detach().to(dtype).cpu()
    bh = None if bias is None else bias.detach().float().cpu()
    probs = torch.softmax(gwh.float() @ xh.float() + (bh if bh is not None else 0), dim=0)
    sel = torch.topk(probs, K).indices.tolist()
    gate, up, down = _host_experts(weight_buf, E, H, I, sel, dtype)
    for _ in range(max(0, warmup)):
        tc.moe_forward(xh, gwh, gate, up, down, K, bh)
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end and (max_calls is None or len(times) < max_calls):
        t0 = time.perf_counter()
        tc.moe_forward(xh, gwh, gate, up, down, K, bh)
        times.append(time.perf_counter() - t0)
    if not times:  # the budget ran out in the warm-up: one timed call
        t0 = time.perf_counter()
        tc.moe_forward(xh, gwh, gate, up, down, K, bh)
        times.append(time.perf_counter() - t0)
    return statistics.median(times) * 1e6, len(times), threads


def cpu_reference_output(x, gate_w, weight_buf, E, H, I, K, bias=None):
    """The restated torch composition's fp32 output and selected experts for
    one token (the parity checker of the bench line)."""
    tc = _composition()
    torch.set_num_threads(os.cpu_count() or 1)
    xh = x.detach().float().cpu()
    gwh = gate_w.detach().float().cpu()
    bh = None if bias is None else bias.detach().float().cpu()
    probs = torch.softmax(gwh @ xh + (bh if bh is not None else 0), dim=0)
    sel = torch.topk(probs, K).indices.tolist()
    gate, up, down = _host_experts(weight_buf, E, H, I, sel, torch.float32)
    return tc.moe_forward(xh, gwh, gate, up, down, K, bh), sel


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.detach().double().cpu().reshape(-1), b.detach().double().cpu().reshape(-1)
    den = torch.linalg.vector_norm(b).item()
    return torch.linalg.vector_norm(a - b).item() / (den if den > 0 else 1.0)


# ---------------------------------------------------------------------------
def workload_name(cfg: str, dtype: str, parallel: str, world: int) -> str:
    return f"{cfg}_bs1_{dtype}" + (f"_{parallel}{world}" if world > 1 else "")


def config_dict(cfg: str, dtype: str, parallel: str, world: int, allreduce: str) -> dict:
    """The workload, identical in both arms' lines."""
    E, H, I, K = SHAPES[cfg]
    return {"workload": workload_name(cfg, dtype, parallel, world), "E": E, "H": H, "I": I,
            "top_k": K, "tokens": 1, "dtype": dtype,
            "parallelism": f"{parallel}{world}" if world > 1 else "single",
            "allreduce": ((("fused in the layer kernel (NVLink peer memory)"
                            if allreduce == "fused" else "NCCL") if world > 1 else None)),
            "l2": "inputs larger than L2 (rotating layers, > 4x L2 streamed between reuses)"}


def run_reference_arm(args, world, rank):
    """warp-route's CPU composition (restated) on all host threads, on the
    same workload as our arm: `--warmup` untimed forwards, then up to
    `--steps` timed forwards within a bounded budget; rank 0 only."""
    if rank != 0:
        return
    from warp_route import synthetic

    E, H, I, K = SHAPES[args.config]
    dt = torch.bfloat16 if args.dtype == "bf16" else torch.float32
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    L = synthetic.make_layer(E, H, I, K, dtype=dt, device=dev, seed=100, layer=0)
    budget = min(120.0, max(5.0, args.cpu_seconds))
    us, n, cores = cpu_composition_timing(L.x, L.gate_w, L.weight_buf, E, H, I, K, budget,
                                          max_calls=args.steps, warmup=args.warmup)
    sample = (f"{n} single-token forwards of the {args.config} layer (the selected experts "
              f"widened to fp32, warp-route's only dtype), median after {args.warmup} warm-ups; "
              f"warp-route's torch composition restated in oracle/torch_composition.py")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(us, 2), "unit": "us/layer",
        "n_gpus": args.gpus, "steps": n, "warmup": args.warmup,
        "ms_per_step": round(us / 1000, 5), "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args.config, args.dtype, args.parallel, world, args.allreduce),
        "cpu_baseline": {"value": round(us, 2), "unit": "us/layer", "cores": cores,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(us, 2), "unit": "us/layer", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def batched_sweep(args, dev, world=1, rank=0, comm=None, dtype=torch.bfloat16):
    """The batched-decode sweep (Mixtral shape, router bias, stacked layers):
    per token count, µs per layer over CUDA-graph replays of one step (every
    layer once) and the HBM GB/s of the distinct experts each layer streams.
    N > 1: expert parallel (rank r holds experts [r E/N, (r+1) E/N) of every
    layer) and the [T, H] output summed over the ranks per layer — by the
    layer's own combine step over NVLink peer memory (comm, a PeerComm) or by
    an NCCL all-reduce — inside the graph; the time is the max over ranks."""
    import torch.distributed as dist

    from warp_route import functional as F
    from warp_route import synthetic

    f32 = dtype == torch.float32
    spec = args.fp32_sweep_tokens if f32 else args.sweep_tokens
    tokens = [int(t) for t in spec.split(",") if t.strip()]
    if not tokens:
        return None
    E, H, I, K = SHAPES["mixtral"]
    if E % world:
        return None
    nl = args.fp32_sweep_layers if f32 else args.sweep_layers
    elt = 4 if f32 else 2
    layers = [synthetic.make_layer(E, H, I, K, dtype=dtype, device=dev, seed=900 + li,
                                   layer=li, router_bias=True, ep_rank=rank, ep_size=world)
              for li in range(nl)]
    results = []
    stream = torch.cuda.Stream()
    rv_buf = torch.zeros(1, device=dev)
    for T in tokens:
        gx = torch.Generator(device=dev)
        gx.manual_seed(7000 + T)
        x = torch.randn(T, H, generator=gx, device=dev).to(dtype)
        xin = x[0].contiguous() if T == 1 else x
        distinct, local_max = [], []
        for Lr in layers:
            _, ids, _ = F.fused_moe_routed(xin, Lr.gate_w, Lr.weight_buf, E, H, I, K,
                                           router_bias=Lr.router_bias,
                                           ep_first_expert=Lr.ep_first, ep_num_local=Lr.ep_num)
            sel = set(ids.cpu().view(-1).tolist())
            distinct.append(len(sel))
            if world > 1:
                local_max.append(max(sum(1 for e in sel if r * (E // world) <= e < (r + 1) * (E // world))
                                     for r in range(world)))

        def step():
            for Lr in layers:
                if comm is not None:
                    F.fused_moe_allreduce(xin, Lr.gate_w, Lr.weight_buf, E, H, I, K, comm,
                                          router_bias=Lr.router_bias,
                                          ep_first_expert=Lr.ep_first,
                                          ep_num_local=Lr.ep_num)
                    continue
                out = F.fused_moe_routed(xin, Lr.gate_w, Lr.weight_buf, E, H, I, K,
                                         router_bias=Lr.router_bias,
                                         ep_first_expert=Lr.ep_first,
                                         ep_num_local=Lr.ep_num)[0]
                if world > 1:
                    dist.all_reduce(out)

        with torch.cuda.stream(stream):
            for _ in range(2):
                step()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step()
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev.index) as clk:
            start_together(world, stream, lambda: dist.all_reduce(rv_buf))
            t0.record(stream)
            with torch.cuda.stream(stream):
                for _ in range(args.sweep_steps):
                    g.replay()
            t1.record(stream)
            torch.cuda.synchronize()
        tt = torch.tensor([t0.elapsed_time(t1)], device=dev)
        if world > 1:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        us = tt.item() * 1000.0 / (args.sweep_steps * nl)
        with torch.cuda.stream(stream):
            st = F._load_extension().workspace_status(xin)
        if st != 0:
            raise SystemExit(f"batched sweep T={T}: device status {st}: timing discarded")
        del g
        torch.cuda.synchronize()
        mean_distinct = sum(distinct) / len(distinct)
        wbytes = mean_distinct * 3 * H * I * elt
        gbs = wbytes / (us * 1e-6) / 1e9
        peak, _ = peaks()
        r = {"tokens": T, "us_per_layer": round(us, 2),
             "hbm_gbs": round(gbs, 1),
             "frac_of_hbm_peak": round(gbs / (peak * world), 4),
             "experts_per_layer": round(mean_distinct, 2),
             "path": ("streaming kernel" if T == 1 or (f32 and T < 3) else
                      "grouped tcgen05 GEMMs, fp32 split into bf16 hi + lo" if f32 else
                      "grouped tcgen05 GEMMs"),
             "clocks": clk.summary()}
        if world > 1:
            r["busiest_rank_experts"] = round(sum(local_max) / len(local_max), 2)
            r["hbm_gbs_note"] = "aggregate over all ranks"
        results.append(r)
    del layers
    torch.cuda.empty_cache()
    how = ("summed in the layer's combine step over NVLink peer memory" if comm is not None
           else "NCCL all-reduce")
    par = (f"expert parallel over {world} GPUs ({E // world} experts each), [T,H] fp32 output "
           f"{how}, in the graph" if world > 1 else "single GPU")
    return {"config": f"mixtral, router bias N(0,1), {'fp32' if f32 else 'bf16'}", "layers": nl,
            "steps": args.sweep_steps, "parallelism": par,
            "note": "each layer has its own weights, gate and bias and takes the same seeded "
                    "token batch; value = µs per layer (graph replays of the layer stack, max "
                    "over ranks); hbm_gbs = distinct selected experts' weight bytes / time; "
                    "frac_of_hbm_peak = hbm_gbs / (N x measured HBM bandwidth)",
            "results": results}


def decode_step(args, dev, world=1, rank=0):
    """A 32-layer decode step (Mixtral shape, one token, tensor parallel over
    the N GPUs with the ranks' sum fused into each layer kernel): the layers
    chained with their residual connection, h <- (h + moe(h)).to(bf16), one
    CUDA-graph replay per step.  `us_per_step` uses moe_decode_layer (the
    residual and the next input written by the layer's own last step, one
    kernel per layer); `unfused_us_per_step` the same stack with the residual
    added by separate kernels after each layer (and, at N > 1, an NCCL
    all-reduce instead of the fused sum).  The graph output is checked equal,
    bit for bit, to the stack run eagerly."""
    import torch.distributed as dist

    from warp_route import functional as F
    from warp_route import synthetic
    from warp_route.decode import MoEStack, StackLayer

    nl = args.decode_layers
    if nl <= 0:
        return None
    E, H, I, K = SHAPES["mixtral"]
    tp = world
    layers = []
    for li in range(nl):
        L = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, device=dev, seed=300 + li,
                                 layer=li, tp_rank=rank, tp_size=tp)
        layers.append(StackLayer(L.gate_w, L.weight_buf))
    comm = F.PeerComm(H) if world > 1 else None
    fused = MoEStack(layers, E, H, I // tp, K, 1, comm=comm)
    unfused = MoEStack(layers, E, H, I // tp, K, 1,
                       all_reduce=(dist.all_reduce if world > 1 else (lambda t: None)))
    gx = torch.Generator(device=dev)
    gx.manual_seed(4242)
    # The synthetic stack has no normalisation between layers and each layer
    # adds roughly 0.5 |h|^2 to h, so a unit-scale token overflows to inf
    # within ~15 layers; at 0.05 the hidden state stays near that scale over
    # all 32 layers (the layer time does not depend on the values).
    x = (torch.randn(H, generator=gx, device=dev) * 0.05).to(torch.bfloat16)
    res = {"layers": nl, "tokens": 1, "input_scale": 0.05,
           "parallelism": (f"tp{world}, ranks' sum fused into each layer kernel" if world > 1
                           else "single GPU")}
    rv_buf = torch.zeros(1, device=dev)
    stream = torch.cuda.current_stream()
    for name, stack in (("us_per_step", fused), ("unfused_us_per_step", unfused)):
        ref = stack.eager(x)
        got = stack.step(x).clone()
        for _ in range(2):
            stack.step(x)
        torch.cuda.synchronize()
        if name == "us_per_step":
            res["graph_equals_eager"] = bool(torch.equal(got, ref))
            res["output_finite"] = bool(torch.isfinite(got.float()).all())
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev.index) as clk:
            start_together(world, stream, lambda: dist.all_reduce(rv_buf))
            t0.record(stream)
            for _ in range(args.decode_steps):
                stack.graph.replay()
            t1.record(stream)
            torch.cuda.synchronize()
        tt = torch.tensor([t0.elapsed_time(t1)], device=dev)
        if world > 1:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        res[name] = round(tt.item() * 1000.0 / args.decode_steps, 2)
        if name == "us_per_step":
            res["us_per_layer"] = round(res[name] / nl, 3)
            res["clocks"] = clk.summary()
        stack.close()
    st = torch.tensor([F._load_extension().workspace_status(x)], device=dev)
    with torch.cuda.stream(fused.stream):
        st = st + F._load_extension().workspace_status(x)
    if world > 1:
        dist.all_reduce(st, op=dist.ReduceOp.MAX)
    if st.item() != 0:
        raise SystemExit(f"decode step: device status {st.item()}: timing discarded")
    if comm is not None:
        torch.cuda.synchronize()
        dist.barrier()
        comm.close()
    del fused, unfused, layers
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    res["steps"] = args.decode_steps
    return res


# The GPU stays busy this long (≈ 2 ms at up to 2 GHz) while the host
# enqueues a timed region, so the region starts on the device, not when the
# host gets there.
SLEEP_CYCLES = 4_000_000


def start_together(world, stream, collective):
    """Device-side rendezvous in front of a timed region (N > 1).

    The ranks leave the host barrier at different times (process scheduling,
    the clock sampler's start-up), so an event recorded straight after it would
    charge that skew to the region through the first collective.  Instead each
    rank queues a sleep kernel (so the host has queued the whole region before
    the device reaches it) and one untimed collective step; that step ends on
    every rank when the slowest rank has joined, and the region's start event
    is recorded right behind it."""
    if world == 1:
        return
    import torch.distributed as dist

    dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        torch.cuda._sleep(SLEEP_CYCLES)
        collective()


def measure_config(args, cfg, parallel, world, rank, local, dev, *, cpu_leg):
    """Times one workload: one decode token through `cfg`'s layer per step
    (tensor- or expert-parallel over the ranks), device-resident (`value`) and
    end to end through the public API (`e2e`), and checks a sampled layer
    against the CPU composition (and, N > 1, against the whole layer run on
    rank 0's GPU).  Returns the dict that becomes the JSON line (rank 0)."""
    import torch.distributed as dist

    from warp_route import functional as F
    from warp_route import synthetic

    E, H, I, K = SHAPES[cfg]
    dt = torch.bfloat16 if args.dtype == "bf16" else torch.float32
    elt = 2 if dt == torch.bfloat16 else 4
    tp = world if parallel == "tp" and world > 1 else 1
    ep = world if parallel == "ep" and world > 1 else 1
    if I % tp or E % ep:
        raise SystemExit(f"{cfg}: cannot split I={I} over {tp} or E={E} over {ep} ranks")
    Il = I // tp
    # Rotate enough layers that the bytes streamed between two reads of the
    # same layer exceed 4x L2 (cold HBM every step).
    sel_bytes = K * 3 * H * Il * elt
    n_layers = max(2, math.ceil(4 * L2_BYTES / max(1, sel_bytes)) + 1)
    layer_bytes = E // ep * 3 * H * Il * elt
    n_layers = min(n_layers, max(2, int(100e9 // layer_bytes)))
    if args.layers > 0:
        n_layers = args.layers
    layers = [synthetic.make_layer(E, H, I, K, dtype=dt, device=dev, seed=100 + li, layer=li,
                                   tp_rank=rank if tp > 1 else 0, tp_size=tp,
                                   ep_rank=rank if ep > 1 else 0, ep_size=ep)
              for li in range(n_layers)]

    # Routing of each layer (identical on all ranks) -> algorithmic bytes of
    # the busiest rank (expert parallel: the rank holding the most selected
    # experts sets the layer's time) and of all ranks together.
    busiest, total = [], []
    for Lr in layers:
        _, ids, _ = F.fused_moe_routed(Lr.x, Lr.gate_w, Lr.weight_buf, E, H, Il, K,
                                       ep_first_expert=Lr.ep_first, ep_num_local=Lr.ep_num)
        sel = set(ids.cpu().view(-1).tolist())
        per_rank = [len([e for e in sel if r * (E // ep) <= e < (r + 1) * (E // ep)])
                    for r in range(ep)]
        busiest.append(synthetic.algorithmic_bytes(E, H, Il, max(per_rank), 1, elt))
        total.append(sum(synthetic.algorithmic_bytes(E, H, Il, u, 1, elt) for u in per_rank)
                     if ep > 1 else world * busiest[-1])
    avg_bytes = sum(busiest) / len(busiest)
    avg_total = sum(total) / len(total)

    # N > 1: every rank's partial output is summed inside the layer kernel
    # (PeerComm, NVLink peer memory), or by a separate NCCL all-reduce.
    fused_ar = world > 1 and args.allreduce == "fused"
    comm = F.PeerComm(H) if fused_ar else None

    def layer(Lr, x, routing=False):
        if fused_ar:
            r = F.fused_moe_allreduce(x, Lr.gate_w, Lr.weight_buf, E, H, Il, K, comm,
                                      ep_first_expert=Lr.ep_first, ep_num_local=Lr.ep_num,
                                      return_routing=True)
            return (r[0], r[1]) if routing else r[0]
        if ep > 1 or routing:
            out, ids, _ = F.fused_moe_routed(x, Lr.gate_w, Lr.weight_buf, E, H, Il, K,
                                             ep_first_expert=Lr.ep_first,
                                             ep_num_local=Lr.ep_num)
            return (out, ids) if routing else out
        return F.fused_moe(x, Lr.gate_w, Lr.weight_buf, E, H, Il, K)

    def reduce(out):
        if world > 1 and not fused_ar:
            dist.all_reduce(out)

    rv_buf = torch.zeros(1, device=dev)

    def rendezvous_step():
        if fused_ar:
            layer(layers[0], layers[0].x)
        else:
            dist.all_reduce(rv_buf)

    stream = torch.cuda.current_stream()
    W, Ksteps = args.warmup, args.steps
    for i in range(W):
        Lr = layers[i % n_layers]
        reduce(layer(Lr, Lr.x))
    torch.cuda.synchronize()

    # ---- device-resident timing ----
    # One fused-kernel launch per step (the all-reduce included when fused).
    # When nothing else is on the stream, the kernel's average launch
    # duration is the timed region over the launches (launch gaps included);
    # per-step events would sit between the kernels and stretch them.  With
    # a separate NCCL all-reduce, each layer call is bracketed by its own
    # events.  Serving replays decode steps from CUDA graphs: the timed steps
    # are replays of a graph of the rotating layers' calls (exactly K calls;
    # capture and warm-up happen before the timed region); the NCCL
    # comparison runs eagerly.
    per_step = world > 1 and not fused_ar
    use_graph = not args.no_graph and not per_step
    graphs, cap_stream = [], None
    if use_graph:
        cap_stream = torch.cuda.Stream()
        with torch.cuda.stream(cap_stream):  # warm up on the capture stream (its workspace)
            for _ in range(2):
                for Lr in layers:
                    layer(Lr, Lr.x)
        torch.cuda.synchronize()

        def capture(n):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap_stream):
                for i in range(n):
                    Lr = layers[i % n_layers]
                    layer(Lr, Lr.x)
            return g

        g_full = capture(n_layers)
        rem = Ksteps % n_layers
        graphs = [g_full] * (Ksteps // n_layers) + ([capture(rem)] if rem else [])
        for _ in range(2):
            g_full.replay()
        torch.cuda.synchronize()
    k_start = [torch.cuda.Event(enable_timing=True) for _ in range(Ksteps if per_step else 0)]
    k_end = [torch.cuda.Event(enable_timing=True) for _ in range(Ksteps if per_step else 0)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        start_together(world, stream, rendezvous_step)
        t0.record(stream)
        if use_graph:
            for g in graphs:
                g.replay()
        else:
            for i in range(Ksteps):
                if per_step:
                    k_start[i].record(stream)
                Lr = layers[i % n_layers]
                out = layer(Lr, Lr.x)
                if per_step:
                    k_end[i].record(stream)
                reduce(out)
        t1.record(stream)
        torch.cuda.synchronize()
    clocks = clk.summary()
    total_ms = t0.elapsed_time(t1)
    if per_step:
        kern_ms = [a.elapsed_time(b) for a, b in zip(k_start, k_end)]
        kern_avg_ms = sum(kern_ms) / len(kern_ms)
    else:
        kern_avg_ms = total_ms / Ksteps

    # ---- end-to-end through the public API, host buffers in and out ----
    # Every step copies its token in from pinned host memory and its output
    # back to pinned host memory.  The copies run on their own streams, as a
    # serving loop would run them: step i+1's input copy and step i's output
    # read overlap the layer kernels; events keep each step's copy-in before
    # its layer and its copy-out after it.  The timed region ends when the
    # last output has reached the host.
    Ke = Ksteps
    x_host = [torch.empty(H, dtype=dt).pin_memory() for _ in range(n_layers)]
    for li, Lr in enumerate(layers):
        x_host[li].copy_(Lr.x.cpu())
    y_host = torch.empty(Ke if Ke <= 4096 else 4096, H, dtype=torch.float32).pin_memory()
    NB = 2  # device input buffers in flight
    x_dev = [torch.empty(H, dtype=dt, device=dev) for _ in range(NB)]
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(NB)]
    ev_read = [torch.cuda.Event() for _ in range(NB)]  # the layer that read x_dev[b] is done

    def e2e_step(i):
        b, li = i % NB, i % n_layers
        with torch.cuda.stream(h2d):
            h2d.wait_event(ev_read[b])
            x_dev[b].copy_(x_host[li], non_blocking=True)
            ev_in[b].record(h2d)
        stream.wait_event(ev_in[b])
        o = layer(layers[li], x_dev[b])
        reduce(o)
        ev_read[b].record(stream)
        with torch.cuda.stream(d2h):
            d2h.wait_event(ev_read[b])
            o.record_stream(d2h)
            y_host[i % y_host.shape[0]].copy_(o, non_blocking=True)

    for i in range(min(W, 8)):
        e2e_step(i)
    torch.cuda.synchronize()
    # Unless --no-graph, the timed e2e steps are replays of a graph of
    # E2E_CHUNK steps, each step the same three operations (pinned-host ->
    # device copy of its token, the public layer call, device -> pinned-host
    # copy of its output) on the same three streams, ordered by the same
    # events (graph edges after capture).
    e2e_graphs = []
    if use_graph:
        cap2 = torch.cuda.Stream()
        with torch.cuda.stream(cap2):  # the capture stream's workspace exists before capture
            for Lr in layers:
                layer(Lr, Lr.x)
        torch.cuda.synchronize()

        def capture_e2e(n):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap2):
                h2d.wait_stream(cap2)
                d2h.wait_stream(cap2)
                for i in range(n):
                    b, li = i % NB, i % n_layers
                    with torch.cuda.stream(h2d):
                        if i >= NB:
                            h2d.wait_event(ev_read[b])
                        x_dev[b].copy_(x_host[li], non_blocking=True)
                        ev_in[b].record(h2d)
                    cap2.wait_event(ev_in[b])
                    o = layer(layers[li], x_dev[b])
                    reduce(o)
                    ev_read[b].record(cap2)
                    with torch.cuda.stream(d2h):
                        d2h.wait_event(ev_read[b])
                        y_host[i % y_host.shape[0]].copy_(o, non_blocking=True)
                cap2.wait_stream(h2d)
                cap2.wait_stream(d2h)
            return g

        chunk = min(Ke, E2E_CHUNK)
        g_e2e = capture_e2e(chunk)
        rem = Ke % chunk
        e2e_graphs = [g_e2e] * (Ke // chunk) + ([capture_e2e(rem)] if rem else [])
        g_e2e.replay()
        torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start_together(world, stream, rendezvous_step)
    e0.record(stream)
    if use_graph:
        for g in e2e_graphs:
            g.replay()
    else:
        h2d.wait_event(e0)
        for i in range(Ke):
            e2e_step(i)
        stream.wait_stream(d2h)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)

    # per-rank times -> max over ranks (the job's time) and the spread
    mine = torch.tensor([total_ms, kern_avg_ms, e2e_ms], device=dev, dtype=torch.float64)
    if world > 1:
        every = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
        every = torch.stack(every).cpu()
    else:
        every = mine.cpu().unsqueeze(0)
    total_ms, kern_avg_ms, e2e_ms = every.max(dim=0).values.tolist()
    spread_us = ((every[:, 0].max() - every[:, 0].min()).item() * 1000.0 / Ksteps)

    # A bounded device wait that gave up would make the timings meaningless.
    ext = F._load_extension()
    status = ext.workspace_status(layers[0].x)
    if use_graph:
        with torch.cuda.stream(cap_stream):  # the workspace the graph's launches used
            status = status or ext.workspace_status(layers[0].x)
    st = torch.tensor([status], device=dev)
    if world > 1:
        dist.all_reduce(st, op=dist.ReduceOp.MAX)
    if st.item() != 0:
        raise SystemExit(f"{cfg}: a fused kernel reported device status {st.item()}: "
                         "timing discarded")

    # ---- parity of a sampled layer (layer 0), through the timed path ----
    L0 = layers[0]
    out0, ids0 = layer(L0, L0.x, routing=True)
    reduce(out0)
    torch.cuda.synchronize()
    parity = {"sampled_layer": 0, "tolerance_rel_l2": 1e-3}
    ok = True
    if world > 1:
        every_out = [torch.empty_like(out0) for _ in range(world)]
        dist.all_gather(every_out, out0)
        parity["ranks_identical"] = all(torch.equal(every_out[0], o) for o in every_out[1:])
        ok = ok and parity["ranks_identical"]
    full = None
    if rank == 0:
        if world > 1:
            full = synthetic.make_layer(E, H, I, K, dtype=dt, device=dev, seed=100, layer=0)
            r_out, r_ids, _ = F.fused_moe_routed(full.x, full.gate_w, full.weight_buf, E, H, I, K)
            torch.cuda.synchronize()
            m = {"ids_match": r_ids.view(-1).tolist() == ids0.view(-1).tolist(),
                 "rel_l2": float(f"{rel_l2(out0, r_out):.3e}")}
            parity["vs_whole_layer_on_rank0_gpu"] = m
            ok = ok and m["ids_match"] and m["rel_l2"] <= 1e-3
        src = full if full is not None else L0
        c_out, c_sel = cpu_reference_output(src.x, src.gate_w, src.weight_buf, E, H, I, K)
        m = {"ids_match": c_sel == ids0.view(-1).tolist(),
             "rel_l2": float(f"{rel_l2(out0, c_out):.3e}")}
        parity["vs_cpu_composition"] = m
        ok = ok and m["ids_match"] and m["rel_l2"] <= 1e-3
        parity["ok"] = bool(ok)
    del full

    # ---- CPU baseline (rank 0, N = 1, the line's own workload) ----
    cpu = None
    if cpu_leg and rank == 0 and world == 1 and not args.no_cpu_baseline:
        us_cpu, ncalls, cores = cpu_composition_timing(L0.x, L0.gate_w, L0.weight_buf, E, H, Il,
                                                       K, args.cpu_seconds)
        variants = []
        for thr, cdt, name in ((1, torch.float32, "fp32"), (None, torch.bfloat16, "bf16")):
            v_us, v_n, v_thr = cpu_composition_timing(L0.x, L0.gate_w, L0.weight_buf, E, H, Il,
                                                      K, min(6.0, args.cpu_seconds),
                                                      threads=thr, dtype=cdt)
            variants.append({"value": round(v_us, 1), "unit": "us/layer", "cores": v_thr,
                             "dtype": name, "calls": v_n})
        cpu = {"value": round(us_cpu, 1), "unit": "us/layer", "cores": cores, "kind": "port",
               "dtype": "fp32",
               "sample": f"{ncalls} single-token forwards of layer 0 ({cfg}), the selected experts "
                         f"widened to fp32, median after 3 warm-ups; warp-route's torch "
                         f"composition restated in oracle/torch_composition.py",
               "variants": variants}

    if comm is not None:
        torch.cuda.synchronize()
        dist.barrier()
        comm.close()
    graphs.clear()
    e2e_graphs.clear()
    del layers
    torch.cuda.synchronize()
    torch.cuda.empty_cache()

    us_per_layer = total_ms * 1000.0 / Ksteps
    peak, peak_kind = peaks()
    achieved = avg_bytes / (kern_avg_ms * 1e-3) / 1e9
    workload = workload_name(cfg, args.dtype, parallel, world)
    res = {
        "value": round(us_per_layer, 3), "unit": "us/layer",
        "ms_per_step": round(total_ms / Ksteps, 6),
        "config": config_dict(cfg, args.dtype, parallel, world, args.allreduce),
        "method": {"layers_rotated": n_layers,
                   "mb_streamed_per_step_busiest_rank": round(avg_bytes / 1e6, 1),
                   "timing": ("CUDA-graph replay of the layer calls" if use_graph
                              else "eager layer calls") +
                             ("; device-side rendezvous (sleep + one untimed collective layer "
                              "call) before each timed region" if world > 1 else ""),
                   "rank_spread_us_per_layer": round(spread_us, 3) if world > 1 else 0.0},
        "hbm_gbs": round(avg_bytes / (us_per_layer * 1e-6) / 1e9, 1),
        "hbm_gbs_all_ranks": round(avg_total / (us_per_layer * 1e-6) / 1e9, 1),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": ncu_traffic(workload),
                     "kernel_us": round(kern_avg_ms * 1000, 3),
                     "algorithmic_bytes": int(avg_bytes),
                     "bytes_note": "selected local experts' weights + router + x + fp32 out, "
                                   "of the rank with the most selected experts"},
        "e2e": {"value": round(e2e_ms * 1000.0 / Ke, 3), "unit": "us/layer",
                "h2d_bytes_per_step": H * elt * world,
                "d2h_bytes_per_step": H * 4 * world,
                "timing": ("CUDA-graph replays of [H2D copy, layer call, D2H copy] steps"
                           if use_graph else "eager steps")},
        "parity": parity,
        "gpu_launches": Ksteps,
        "clocks": clocks,
    }
    if cpu is not None:
        res["cpu_baseline"] = cpu
    return res


def run_ours(args, world, rank, local):
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    main = measure_config(args, args.config, args.parallel, world, rank, local, dev, cpu_leg=True)
    extras = {}
    for cfg in [c for c in args.extra_configs.split(",") if c.strip()]:
        if cfg == args.config:
            continue
        # the other BASELINE configurations: expert parallel over N > 1 GPUs
        r = measure_config(args, cfg, "ep", world, rank, local, dev, cpu_leg=False)
        extras[r["config"]["workload"]] = r

    sweep = None
    if args.sweep_tokens.strip():
        # The sweep sums the ranks' batch outputs with NCCL: measured faster
        # than the all-reducing combine step for batches (2 GPUs, 8 layers:
        # 250 vs 260 µs at T = 16, 428 vs 456 µs at T = 256);
        # `--sweep-fused-allreduce` uses the combine step instead.
        from warp_route import functional as F
        comm = F.PeerComm(SHAPES["mixtral"][1]) if (args.sweep_fused_allreduce and world > 1) \
            else None
        sweep = batched_sweep(args, dev, world, rank, comm)
        if comm is not None:
            torch.cuda.synchronize()
            dist.barrier()
            comm.close()
    sweep32 = None
    if args.fp32_sweep_tokens.strip():
        sweep32 = batched_sweep(args, dev, world, rank, None, dtype=torch.float32)

    dec = decode_step(args, dev, world, rank)

    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {"metric": METRIC}
        line.update({k: main[k] for k in ("value", "unit")})
        line.update({"n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                     "ms_per_step": main["ms_per_step"], "higher_is_better": False,
                     "scaling": "strong", "vs_baseline": None, "dtype": args.dtype,
                     "data": "synthetic"})
        for k in ("config", "method", "hbm_gbs", "hbm_gbs_all_ranks", "roofline", "e2e",
                  "parity", "gpu_launches", "clocks"):
            line[k] = main[k]
        line["cpu_baseline"] = main.get("cpu_baseline")
        if extras:
            line["other_configs"] = extras
        if sweep is not None:
            line["batched_sweep"] = sweep
        if sweep32 is not None:
            line["batched_sweep_fp32"] = sweep32
        if dec is not None:
            line["decode_step"] = dec
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def profile_layer(args):
    """Three eager calls of one layer (one GPU), for an ncu capture of its kernels."""
    from warp_route import functional as F
    from warp_route import synthetic

    cfg, T = args.profile_layer.split(":")
    T = int(T)
    E, H, I, K = SHAPES[cfg] if cfg in SHAPES else (int(v) for v in cfg.split("x"))
    dt = torch.bfloat16 if args.dtype == "bf16" else torch.float32
    L = synthetic.make_layer(E, H, I, K, dtype=dt, seed=200, tokens=T, router_bias=K < E)
    for _ in range(3):
        out = F.fused_moe_routed(L.x, L.gate_w, L.weight_buf, E, H, I, K,
                                 router_bias=L.router_bias)[0]
    torch.cuda.synchronize()
    st = F._load_extension().workspace_status(L.x)
    if st != 0:
        raise SystemExit(f"profile layer: device status {st}")
    print(json.dumps({"profile_layer": args.profile_layer, "dtype": args.dtype,
                      "out_abs_mean": float(out.float().abs().mean())}), flush=True)


def main():
    args = parse()
    if args.profile_layer:
        torch.cuda.set_device(0)
        profile_layer(args)
        return
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        run_reference_arm(args, world, rank)
        return
    if args.only_sweep:
        if world != 1:
            raise SystemExit("--only-sweep runs on one GPU")
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        out = {"batched_sweep": batched_sweep(args, dev)}
        if args.fp32_sweep_tokens.strip():
            out["batched_sweep_fp32"] = batched_sweep(args, dev, dtype=torch.float32)
        print(json.dumps(out), flush=True)
        return
    run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
