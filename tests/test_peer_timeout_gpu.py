"""Failure detection of the all-reduce fused into the layer: a rank that
stops making its calls.

warp-route has no multi-GPU path and its launchers `exit(1)` on any error
(src/fused_moe.cu:9-15,239-247); here every wait for a peer rank is bounded
(the communicator's peer timeout) and reported through the workspace status
word, and `wr_comm_reset` puts the ranks back in step afterwards.

The failure is made on the host: rank 1 skips one call (it leaves between
steps, with nothing of its own in flight) and waits at a host barrier.  Rank
0's call then waits for words that nobody writes; with a 20 ms peer timeout it
must end quickly with WR_ERR_TIMEOUT and the DEV_TIMEOUT_PEER bit (0x20).  No
GPU faults, traps or hangs: the kernel's wait simply gives up.

Two forms, as child processes with a gloo group for the host side:
  * two GPUs: one correctly paired call, the skipped call, a reset on both
    ranks, then paired calls whose output matches the whole layer again;
  * one GPU (both processes on GPU 0): rank 1 never launches anything, so
    only rank 0's kernel ever runs on the device; after its call times out
    a plain single-GPU call on the same context still matches the whole
    layer.  (Two ranks' waiting kernels never share one GPU here: the paired
    calls run only in the two-GPU form.)
"""
from __future__ import annotations

import ctypes
import os
import socket
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-3
PEER_TIMEOUT_S = 0.02
DEV_TIMEOUT_PEER = 0x20


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, same_gpu: bool) -> None:
    import sys
    from datetime import timedelta

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for sub in ("warp-route_b200", "tests"):
        sys.path.insert(0, os.path.join(repo, sub))
    import torch.distributed as dist

    from warp_route import _abi, synthetic
    from warp_route import functional as F

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    dev = 0 if same_gpu else rank
    torch.cuda.set_device(dev)
    lib = _abi.load()
    E, H, I, K = 8, 1024, 2048, 2
    comm = F.PeerComm(H)
    try:
        comm.set_peer_timeout(PEER_TIMEOUT_S)
        shard = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=5, tp_rank=rank,
                                     tp_size=world)
        full = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=5)
        d = _abi.desc(E, H, shard.I, K, _abi.WR_DTYPE_BF16)
        need = lib.wr_fused_moe_workspace_size(ctypes.byref(d), 1)
        ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
        wbytes = shard.weight_buf.numel() * shard.weight_buf.element_size()
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(91)
        xs = [torch.randn(H, generator=gen, device="cuda").to(torch.bfloat16) for _ in range(4)]

        def call(x):
            """One fused all-reduce layer call through the C ABI; returns
            (out, status, status text, seconds)."""
            out = torch.full((H,), float("nan"), dtype=torch.float32, device="cuda")
            t0 = time.perf_counter()
            _abi.check(lib.wr_fused_moe_allreduce(
                ctypes.byref(d), 1, ctypes.c_void_p(x.data_ptr()),
                ctypes.c_void_p(shard.gate_w.data_ptr()),
                ctypes.c_void_p(shard.weight_buf.data_ptr()), wbytes,
                ctypes.c_void_p(out.data_ptr()), None, None, ctypes.c_void_p(ws.data_ptr()),
                ws.numel(), ctypes.c_void_p(comm.handle), stream))
            st = lib.wr_workspace_status(ctypes.c_void_p(ws.data_ptr()), stream)
            dt = time.perf_counter() - t0
            return out, st, lib.wr_last_error_string().decode(), dt

        def whole(x):
            return F.fused_moe(x, full.gate_w, full.weight_buf, E, H, I, K)

        def rel(a, b):
            a, b = a.double(), b.double()
            return (torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b)).item()

        if not same_gpu:
            # a correctly paired call
            out, st, msg, _ = call(xs[0])
            assert st == _abi.WR_OK, msg
            assert rel(out, whole(xs[0])) <= REL_L2_TOL
        dist.barrier()
        # rank 1 skips this call: rank 0's wait for its words gives up
        if rank == 0:
            out, st, msg, secs = call(xs[1])
            assert st == _abi.WR_ERR_TIMEOUT, f"status {st}: {msg}"
            bits = int(msg.rsplit("0x", 1)[1].rstrip(")"), 16)
            assert bits & DEV_TIMEOUT_PEER, msg
            assert secs < 5.0, f"the bounded wait took {secs:.2f} s"
        dist.barrier()
        if same_gpu:
            # the context is still usable: a plain single-GPU layer is right
            if rank == 0:
                torch.cuda.synchronize()
                got = whole(xs[2])
                ref = F.fused_moe(xs[2], full.gate_w, full.weight_buf, E, H, I, K)
                torch.cuda.synchronize()
                assert torch.equal(got, ref)
                assert F._load_extension().workspace_status(xs[2]) == 0
            dist.barrier()
        else:
            # recovery: both ranks reset between two barriers, then calls are
            # paired and correct again (two in a row: both mailbox parities)
            comm.reset()
            outs = []
            for x in xs[2:]:
                out, st, msg, _ = call(x)
                assert st == _abi.WR_OK, msg
                assert rel(out, whole(x)) <= REL_L2_TOL, "wrong output after the reset"
                outs.append(out)
            flat = torch.cat(outs).cpu()
            every = [torch.empty_like(flat) for _ in range(world)]
            dist.all_gather(every, flat)
            assert torch.equal(every[0], every[1]), "ranks disagree after the reset"
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        comm.close()
        dist.destroy_process_group()


def _spawn(same_gpu: bool) -> None:
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _free_port(), same_gpu), nprocs=2, join=True)


def test_peer_that_skips_a_call_times_out_then_reset_recovers():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _spawn(same_gpu=False)


def test_peer_that_never_calls_times_out_on_one_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    _spawn(same_gpu=True)
