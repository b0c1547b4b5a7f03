"""Benchmark: µs per fused MoE layer and achieved HBM GB/s (decode, bs=1).

python bench.py [--gpus N] [--steps K] [--warmup W] [--config mixtral|deepseek|dbrx|tiny]
                [--parallel tp|ep] [--impl ours|reference]

One step = one MoE layer forward for one decode token (router -> top-K ->
SwiGLU over the selected experts -> weighted combine; plus the hidden-sized
all-reduce when N > 1).  The default workload is the Mixtral-shaped layer
(H 4096, I 14336, E 8, top_k 2, bf16 weights, fp32 accumulation/output),
tensor-parallel over N GPUs.  Inputs are synthetic and seeded; layers rotate
so every step streams weights from HBM (each step reads more than L2 holds).

Rank 0 prints one JSON line.  `value` is µs per layer (max over ranks, CUDA
events on the launching stream; the timed steps replay a CUDA graph of the
layer calls); `e2e` is the same through the public API with the token copied
in from pinned host memory and the output copied back every step (copies on
their own streams, overlapping the kernels; the steps replayed from CUDA
graphs of 64 steps, or eagerly with --no-graph); `roofline` relates
the fused kernel's algorithmic bytes to the
measured HBM copy bandwidth; `cpu_baseline` times warp-route's own CPU
composition (restated in oracle/torch_composition.py) on a bounded sample.
`--impl reference` times that CPU composition alone, as the reference arm.

The line also carries `batched_sweep`: the batched-decode sweep on
the Mixtral shape (tokens 1, 4, 16, 64, 256; router bias N(0,1) per expert to
skew the load; 32 stacked layers with independent weights, each applied to
the same seeded token batch), µs per layer from CUDA-graph replays of the 32
layer calls.  Batches of two or more bf16 tokens run on the grouped
tensor-core path (tcgen05 GEMMs over tokens bucketed per expert).  At N > 1
the sweep is expert parallel (E/N experts of every layer per GPU) with one
NCCL all-reduce of the layer output, both inside the replayed graph.
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
    ap.add_argument("--sweep-steps", type=int, default=3)
    ap.add_argument("--sweep-fused-allreduce", action="store_true",
                    help="N > 1: sum the sweep's batch outputs in the layer's combine step "
                         "over NVLink peer memory instead of NCCL (needs --allreduce fused)")
    ap.add_argument("--only-sweep", action="store_true",
                    help="run only the batched-decode sweep (N = 1) and print its JSON line")
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
# CPU composition (warp-route's own CPU path, restated in oracle/)
# ---------------------------------------------------------------------------
def cpu_composition_timing(x, gate_w, weight_buf, E, H, I, K, budget_s, max_calls=None,
                           bias=None):
    """Time the restated torch_moe_reference on host threads.  Weights are the
    same layer's selected experts, widened to fp32 (warp-route's own dtype)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import torch_composition as tc

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    xh = x.detach().float().cpu()
    gwh = gate_w.detach().float().cpu()
    bh = None if bias is None else bias.detach().float().cpu()
    probs = torch.softmax(gwh @ xh + (bh if bh is not None else 0), dim=0)
    sel = torch.topk(probs, K).indices.tolist()
    elt = weight_buf.element_size()
    stride = ((3 * H * I * elt + 127) // 128 * 128) // elt
    n = I * H
    gate, up, down = [None] * E, [None] * E, [None] * E
    for e in sel:
        blk = weight_buf[e * stride:e * stride + 3 * n].float().cpu()
        gate[e] = blk[:n].view(I, H)
        up[e] = blk[n:2 * n].view(I, H)
        down[e] = blk[2 * n:].view(H, I)
    for _ in range(3):
        tc.moe_forward(xh, gwh, gate, up, down, K, bh)
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end and (max_calls is None or len(times) < max_calls):
        t0 = time.perf_counter()
        tc.moe_forward(xh, gwh, gate, up, down, K, bh)
        times.append(time.perf_counter() - t0)
    return statistics.median(times) * 1e6, len(times), threads


# ---------------------------------------------------------------------------
def workload_name(args, world: int) -> str:
    return f"{args.config}_bs1_{args.dtype}" + (f"_{args.parallel}{world}" if world > 1 else "")


def run_reference_arm(args, world, rank):
    if rank != 0:
        return
    from warp_route import synthetic

    E, H, I, K = SHAPES[args.config]
    dt = torch.bfloat16 if args.dtype == "bf16" else torch.float32
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    L = synthetic.make_layer(E, H, I, K, dtype=dt, device=dev, seed=0)
    budget = min(60.0, max(5.0, args.cpu_seconds))
    us, n, cores = cpu_composition_timing(L.x, L.gate_w, L.weight_buf, E, H, I, K, budget,
                                          max_calls=args.steps)
    sample = (f"{n} forwards of the {args.config} layer (bs=1, fp32 weights of the selected "
              f"experts), median; warp-route's torch composition restated")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(us, 2), "unit": "us/layer",
        "n_gpus": args.gpus, "steps": n, "warmup": 3, "ms_per_step": round(us / 1000, 4),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_name(args, world), "E": E, "H": H, "I": I, "top_k": K,
                   "tokens": 1,
                   "parallelism": f"{args.parallel}{world}" if world > 1 else "single",
                   "reference_compute": "fp32 (warp-route's only dtype): the layer's "
                                        f"{args.dtype} weights widened to fp32"},
        "cpu_baseline": {"value": round(us, 2), "unit": "us/layer", "cores": cores,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(us, 2), "unit": "us/layer", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def batched_sweep(args, dev, world=1, rank=0, comm=None):
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

    tokens = [int(t) for t in args.sweep_tokens.split(",") if t.strip()]
    if not tokens:
        return None
    E, H, I, K = SHAPES["mixtral"]
    if E % world:
        return None
    nl = args.sweep_layers
    layers = [synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, device=dev, seed=900 + li,
                                   layer=li, router_bias=True, ep_rank=rank, ep_size=world)
              for li in range(nl)]
    results = []
    stream = torch.cuda.Stream()
    for T in tokens:
        gx = torch.Generator(device=dev)
        gx.manual_seed(7000 + T)
        x = torch.randn(T, H, generator=gx, device=dev).to(torch.bfloat16)
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
        if world > 1:
            dist.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev.index) as clk:
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
        wbytes = mean_distinct * 3 * H * I * 2
        gbs = wbytes / (us * 1e-6) / 1e9
        peak, _ = peaks()
        r = {"tokens": T, "us_per_layer": round(us, 2),
             "hbm_gbs": round(gbs, 1),
             "frac_of_hbm_peak": round(gbs / (peak * world), 4),
             "experts_per_layer": round(mean_distinct, 2),
             "path": "streaming kernel" if T == 1 else "grouped tcgen05 GEMMs",
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
    return {"config": "mixtral, router bias N(0,1), bf16", "layers": nl,
            "steps": args.sweep_steps, "parallelism": par,
            "note": "each layer has its own weights, gate and bias and takes the same seeded "
                    "token batch; value = µs per layer (graph replays of the layer stack, max "
                    "over ranks); hbm_gbs = distinct selected experts' weight bytes / time; "
                    "frac_of_hbm_peak = hbm_gbs / (N x measured HBM bandwidth)",
            "results": results}


def run_ours(args, world, rank, local):
    import torch.distributed as dist

    from warp_route import functional as F
    from warp_route import synthetic

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    E, H, I, K = SHAPES[args.config]
    dt = torch.bfloat16 if args.dtype == "bf16" else torch.float32
    elt = 2 if dt == torch.bfloat16 else 4
    tp = world if args.parallel == "tp" and world > 1 else 1
    ep = world if args.parallel == "ep" and world > 1 else 1
    # Rotate enough layers that the bytes streamed between two reads of the
    # same layer exceed 4x L2 (cold HBM every step).
    sel_bytes = K * 3 * H * (I // tp) * elt
    n_layers = max(2, math.ceil(4 * L2_BYTES / max(1, sel_bytes)) + 1)
    layer_bytes = E // ep * 3 * H * (I // tp) * elt
    n_layers = min(n_layers, max(2, int(100e9 // layer_bytes)))
    if args.layers > 0:
        n_layers = args.layers
    layers = []
    for li in range(n_layers):
        layers.append(synthetic.make_layer(E, H, I, K, dtype=dt, device=dev, seed=100 + li,
                                           layer=li, tp_rank=rank if tp > 1 else 0, tp_size=tp,
                                           ep_rank=rank if ep > 1 else 0, ep_size=ep))
    Il = I // tp

    # routing of each layer (identical on all ranks) -> algorithmic bytes
    distinct = []
    for Lr in layers:
        _, ids, _ = F.fused_moe_routed(Lr.x, Lr.gate_w, Lr.weight_buf, E, H, Il, K,
                                       ep_first_expert=Lr.ep_first, ep_num_local=Lr.ep_num)
        sel = set(ids.cpu().view(-1).tolist())
        if ep > 1:
            sel = {e for e in sel if Lr.ep_first <= e < Lr.ep_first + Lr.ep_num}
        distinct.append(len(sel))
    bytes_per_layer = [synthetic.algorithmic_bytes(E, H, Il, u, 1, elt) for u in distinct]
    avg_bytes = sum(bytes_per_layer) / len(bytes_per_layer)

    # N > 1: every rank's partial output is summed inside the layer kernel
    # (PeerComm, NVLink peer memory), or by a separate NCCL all-reduce.
    fused_ar = world > 1 and args.allreduce == "fused"
    comm = F.PeerComm(H) if fused_ar else None

    def layer(Lr, x):
        if fused_ar:
            return F.fused_moe_allreduce(x, Lr.gate_w, Lr.weight_buf, E, H, Il, K, comm,
                                         ep_first_expert=Lr.ep_first, ep_num_local=Lr.ep_num)
        if ep > 1:
            return F.fused_moe_routed(x, Lr.gate_w, Lr.weight_buf, E, H, Il, K,
                                      ep_first_expert=Lr.ep_first, ep_num_local=Lr.ep_num)[0]
        return F.fused_moe(x, Lr.gate_w, Lr.weight_buf, E, H, Il, K)

    def reduce(out):
        if world > 1 and not fused_ar:
            dist.all_reduce(out)

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
    # events.
    per_step = world > 1 and not fused_ar
    # Serving replays decode steps from CUDA graphs: the timed steps are
    # replays of a graph of the rotating layers' calls (exactly K calls;
    # capture and warm-up happen before the timed region).  The NCCL
    # all-reduce comparison runs eagerly.
    use_graph = not args.no_graph and not per_step
    graphs = []
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
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
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
    if world > 1:
        dist.barrier()
    clocks = clk.summary()
    total_ms = t0.elapsed_time(t1)
    if per_step:
        kern_ms = [a.elapsed_time(b) for a, b in zip(k_start, k_end)]
        kern_avg_ms = sum(kern_ms) / len(kern_ms)
    else:
        kern_avg_ms = total_ms / Ksteps
    t = torch.tensor([total_ms, kern_avg_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, kern_avg_ms = t.tolist()
    us_per_layer = total_ms * 1000.0 / Ksteps

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
    # Serving replays its steps from CUDA graphs: unless --no-graph, the timed
    # e2e steps are replays of a graph of E2E_CHUNK steps, each step the same
    # three operations (pinned-host -> device copy of its token, the public
    # layer call, device -> pinned-host copy of its output) on the same three
    # streams, ordered by the same events (graph edges after capture).
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
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
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
    te = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_us = te.item() * 1000.0 / Ke
    # A bounded device wait that gave up would make the timings meaningless.
    status = F._load_extension().workspace_status(layers[0].x)
    if use_graph:
        with torch.cuda.stream(cap_stream):  # the workspace the graph's launches used
            status = status or F._load_extension().workspace_status(layers[0].x)
    if status != 0:
        raise SystemExit(f"fused kernel reported device status {status}: timing discarded")

    # ---- CPU baseline (rank 0, N = 1 only) ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        full = layers[0]
        us_cpu, ncalls, cores = cpu_composition_timing(full.x, full.gate_w, full.weight_buf, E, H,
                                                       Il, K, args.cpu_seconds)
        cpu = {"value": round(us_cpu, 1), "unit": "us/layer", "cores": cores, "kind": "port",
               "sample": f"{ncalls} single-token forwards of layer 0 ({args.config}), the "
                         f"selected experts widened to fp32, median of {ncalls} after 3 warm-ups; "
                         f"warp-route's torch composition restated in oracle/torch_composition.py"}

    # The sweep sums the ranks' batch outputs with NCCL: measured faster than the
    # all-reducing combine step for batches (2 GPUs, 8 layers: 250 vs 260 µs
    # at T = 16, 428 vs 456 µs at T = 256); `--sweep-fused-allreduce` uses the
    # combine step instead.
    sweep = batched_sweep(args, dev, world, rank,
                          comm if args.sweep_fused_allreduce else None)

    if world > 1:
        dist.barrier()
    if rank == 0:
        peak, peak_kind = peaks()
        # the fused kernel's bytes per launch on the busiest rank (identical per rank for TP)
        achieved = avg_bytes / (kern_avg_ms * 1e-3) / 1e9
        workload = workload_name(args, world)
        traffic = ncu_traffic(workload)
        line = {
            "metric": METRIC, "value": round(us_per_layer, 3), "unit": "us/layer",
            "n_gpus": world, "steps": Ksteps, "warmup": W,
            "ms_per_step": round(total_ms / Ksteps, 6), "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": args.dtype, "data": "synthetic",
            "config": {"workload": workload, "E": E, "H": H, "I": I, "top_k": K, "tokens": 1,
                       "parallelism": f"{args.parallel}{world}" if world > 1 else "single",
                       "allreduce": (("fused in the layer kernel (NVLink peer memory)"
                                      if fused_ar else "NCCL") if world > 1 else None),
                       "l2": f"inputs larger than L2: {n_layers} rotating layers, "
                             f"{avg_bytes / 1e6:.1f} MB streamed per step",
                       "layers_rotated": n_layers,
                       "timing": ("CUDA-graph replay of the layer calls" if use_graph
                                  else "eager layer calls")},
            "hbm_gbs": round(avg_bytes / (us_per_layer * 1e-6) / 1e9, 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_kind": peak_kind,
                         "traffic": traffic,
                         "kernel_us": round(kern_avg_ms * 1000, 3),
                         "algorithmic_bytes": int(avg_bytes)},
            "e2e": {"value": round(e2e_us, 3), "unit": "us/layer",
                    "h2d_bytes_per_step": H * elt * world,
                    "d2h_bytes_per_step": H * 4 * world,
                    "timing": ("CUDA-graph replays of [H2D copy, layer call, D2H copy] steps"
                               if use_graph else "eager steps")},
            "gpu_launches": Ksteps,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        if sweep is not None:
            line["batched_sweep"] = sweep
        print(json.dumps(line), flush=True)
    if comm is not None:
        torch.cuda.synchronize()
        dist.barrier()
        comm.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        run_reference_arm(args, world, rank)
        return
    if args.only_sweep:
        if world != 1:
            raise SystemExit("--only-sweep runs on one GPU")
        torch.cuda.set_device(local)
        sweep = batched_sweep(args, torch.device("cuda", local))
        print(json.dumps({"batched_sweep": sweep}), flush=True)
        return
    run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
