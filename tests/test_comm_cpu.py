"""Host-side parts of the fused all-reduce that need no GPU: the C ABI's
argument checks for the communicator, and the handle exchange among ranks
(world size 2 over gloo)."""
from __future__ import annotations

import ctypes
import os
import socket

import pytest
import torch

from warp_route import _abi
from warp_route import functional as F


def test_handle_bytes():
    assert _abi.load().wr_comm_handle_bytes() == 64  # one CUDA IPC memory handle


@pytest.mark.parametrize("rank,world,hidden", [(0, 0, 64), (0, 9, 64), (2, 2, 64), (-1, 2, 64),
                                               (0, 2, 0)])
def test_create_rejects_bad_arguments(rank, world, hidden):
    lib = _abi.load()
    out = ctypes.c_void_p(123)
    st = lib.wr_comm_create(rank, world, hidden, ctypes.byref(out))
    assert st in (_abi.WR_ERR_INVALID, _abi.WR_ERR_UNSUPPORTED)
    assert out.value is None  # nothing created
    assert lib.wr_last_error_string().decode()


def test_entry_points_reject_missing_comm():
    lib = _abi.load()
    assert lib.wr_comm_destroy(None) == _abi.WR_OK
    assert lib.wr_comm_get_handle(None, None) == _abi.WR_ERR_INVALID
    assert lib.wr_comm_open(None, None) == _abi.WR_ERR_INVALID
    d = _abi.desc(8, 512, 1024, 2, _abi.WR_DTYPE_F32)
    st = lib.wr_fused_moe_allreduce(ctypes.byref(d), 1, None, None, None, 0, None, None, None,
                                    None, 0, None, None)
    assert st == _abi.WR_ERR_INVALID
    assert "comm" in lib.wr_last_error_string().decode()


def _exchange_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = bytes([rank]) * 64
        q.put((rank, F.exchange_handles(mine)))
    finally:
        dist.destroy_process_group()


def test_handle_exchange_two_ranks():
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = bytes([0]) * 64 + bytes([1]) * 64
    assert got[0] == want and got[1] == want
