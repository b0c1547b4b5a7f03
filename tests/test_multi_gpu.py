"""Multi-GPU layers, run as one child process per GPU on 2 GPUs (skipped with
fewer): the all-reduce fused into the layer (wr_fused_moe_allreduce /
PeerComm), and the expert-parallel token batch on the grouped tcgen05 path
with an NCCL all-reduce (the batched sweep's 8-GPU layout).

Each rank holds a tensor-parallel slice (or an expert-parallel set) of one
layer; the fused call must return the full layer's output — compared with the
same layer run whole on one GPU, within the suite's relative-L2 tolerance —
bit-identical on every rank, over several consecutive calls (both buffer
parities) and a token batch of more than one launch.  The process group is
gloo (host only: the handle exchange and the result gathering); the kernels
use plain peer loads and stores, no multicast.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-3
WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double(), b.double()
    return (torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b)).item()


def _worker(rank: int, world: int, port: int, mode: str, dtype_name: str = "bf16") -> None:
    import sys
    from datetime import timedelta

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(repo, "warp-route_b200"))
    import torch.distributed as dist

    from warp_route import functional as F
    from warp_route import synthetic

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    torch.cuda.set_device(rank)
    dt = torch.float32 if dtype_name == "fp32" else torch.bfloat16
    try:
        E, H, I, K = 8, 1024, 2048, 2
        tp = world if mode == "tp" else 1
        ep = world if mode == "ep" else 1
        comm = F.PeerComm(H)
        full = synthetic.make_layer(E, H, I, K, dtype=dt, seed=5, tokens=1)
        shard = synthetic.make_layer(E, H, I, K, dtype=dt, seed=5, tokens=1,
                                     tp_rank=rank if tp > 1 else 0, tp_size=tp,
                                     ep_rank=rank if ep > 1 else 0, ep_size=ep)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(77)
        # several calls in a row (both parities of the peer buffers), then
        # batches on the grouped path, whose combine step sums the ranks'
        # outputs (100 tokens: two all-reducing launches of <= 64 tokens),
        # and single tokens again
        # (fp32: batches of >= 3 tokens on the fp32 grouped path)
        xs = [torch.randn(H, generator=gen, device="cuda").to(dt) for _ in range(5)]
        xs.append(torch.randn(6, H, generator=gen, device="cuda").to(dt))
        xs.append(torch.randn(100, H, generator=gen, device="cuda").to(dt))
        xs += [torch.randn(H, generator=gen, device="cuda").to(dt) for _ in range(2)]
        outs = []
        for x in xs:
            out = F.fused_moe_allreduce(x, shard.gate_w, shard.weight_buf, E, H, shard.I, K, comm,
                                        ep_first_expert=shard.ep_first, ep_num_local=shard.ep_num)
            outs.append(out)
        torch.cuda.synchronize()
        assert F._load_extension().workspace_status(xs[0]) == 0
        for x, out in zip(xs, outs):
            if x.dim() == 1:
                ref = F.fused_moe(x, full.gate_w, full.weight_buf, E, H, I, K)
            else:
                ref = F.batched_fused_moe(x, full.gate_w, full.weight_buf, E, H, I, K)
            err = _rel_l2(out, ref)
            assert err <= REL_L2_TOL, f"rank {rank} {mode} {dtype_name}: rel L2 {err:.3e}"
        # bit-identical on every rank
        flat = torch.cat([o.reshape(-1) for o in outs]).cpu()
        gathered = [torch.empty_like(flat) for _ in range(world)]
        dist.all_gather(gathered, flat)
        for g in gathered[1:]:
            assert torch.equal(g, gathered[0]), f"{mode}: ranks disagree"
        comm.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("dtype_name", ["bf16", "fp32"])
@pytest.mark.parametrize("mode", ["tp", "ep"])
def test_fused_allreduce_matches_whole_layer(mode, dtype_name):
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(WORLD, _free_port(), mode, dtype_name), nprocs=WORLD, join=True)


def _worker_batched_ep(rank: int, world: int, port: int) -> None:
    import sys
    from datetime import timedelta

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(repo, "warp-route_b200"))
    import torch.distributed as dist

    from warp_route import functional as F
    from warp_route import synthetic

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        E, H, I, K = 8, 1024, 2048, 2
        for T in (16, 100):
            full = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=41, tokens=T,
                                        router_bias=True)
            shard = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=41, tokens=T,
                                         router_bias=True, ep_rank=rank, ep_size=world)
            out, ids, _ = F.fused_moe_routed(shard.x, shard.gate_w, shard.weight_buf, E, H, I, K,
                                             router_bias=shard.router_bias,
                                             ep_first_expert=shard.ep_first,
                                             ep_num_local=shard.ep_num)
            dist.all_reduce(out)
            ref, ref_ids, _ = F.fused_moe_routed(full.x, full.gate_w, full.weight_buf, E, H, I, K,
                                                 router_bias=full.router_bias)
            torch.cuda.synchronize()
            assert torch.equal(ids, ref_ids), f"rank {rank}: routing differs from the whole layer"
            err = _rel_l2(out, ref)
            assert err <= REL_L2_TOL, f"rank {rank} T={T}: rel L2 {err:.3e}"
            # identical on both ranks
            other = out.clone()
            dist.broadcast(other, src=0)
            torch.cuda.synchronize()
            assert torch.equal(other, out), "ranks disagree after the all-reduce"
        assert F._load_extension().workspace_status(out) == 0
    finally:
        dist.destroy_process_group()


def test_batched_expert_parallel_matches_whole_layer():
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker_batched_ep, args=(WORLD, _free_port()), nprocs=WORLD, join=True)
