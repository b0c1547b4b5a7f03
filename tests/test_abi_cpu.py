"""CPU: the C-ABI library loads, exports every symbol include/*.h declares,
and rejects bad arguments with status codes before touching the GPU."""
from __future__ import annotations

import ctypes
import glob
import os
import re

import numpy as np
import pytest

import oracle
from warp_route import _abi

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        text = open(h).read()
        names |= set(re.findall(r"WR_API[^;(]*?\b(wr_\w+)\s*\(", text, flags=re.S))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    for n in ("wr_fused_moe", "wr_batched_fused_moe", "wr_naive_moe", "wr_router_topk",
              "wr_expert_offsets", "wr_total_weight_bytes"):
        assert n in names


@pytest.mark.parametrize("name", declared_symbols())
def test_library_exports_symbol(name):
    lib = _abi.load()
    assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    assert name in _abi.SIGNATURES, f"{name} has no ctypes prototype in warp_route/_abi.py"


def test_version_and_status_strings():
    lib = _abi.load()
    assert b"sm_100a" in lib.wr_version()
    assert lib.wr_status_string(_abi.WR_ERR_TOO_SMALL) == b"weight buffer too small"


@pytest.mark.parametrize("H,I,elt", [(512, 1024, 4), (4096, 14336, 2), (100, 52, 4), (200, 36, 2)])
def test_layout_matches_oracle(H, I, elt):
    lib = _abi.load()
    off = _abi.ExpertOffsets()
    _abi.check(lib.wr_expert_offsets(H, I, elt, ctypes.byref(off)))
    assert off.gate_proj_offset == 0
    assert off.up_proj_offset == I * H * elt
    assert off.down_proj_offset == 2 * I * H * elt
    assert off.expert_stride == oracle.expert_stride(H, I, elt)
    assert off.expert_stride % 128 == 0
    assert lib.wr_total_weight_bytes(8, H, I, elt) == 8 * off.expert_stride


def test_fp32_layout_is_warp_routes():
    # src/expert_layout.cuh:34-47: stride = (3*H*I*4 + 127) & ~127
    lib = _abi.load()
    assert lib.wr_total_weight_bytes(8, 4096, 14336, 4) == 8 * ((3 * 4096 * 14336 * 4 + 127) & ~127)


def _desc(**kw):
    base = dict(num_experts=8, hidden_dim=512, intermediate_dim=1024, top_k=2, dtype=0)
    base.update(kw)
    return _abi.desc(base["num_experts"], base["hidden_dim"], base["intermediate_dim"],
                     base["top_k"], base["dtype"], kw.get("ep_first", 0), kw.get("ep_num", 0))


FAKE = ctypes.c_void_p(0x10000)  # never dereferenced: every call below fails validation first


@pytest.mark.parametrize("kw,status", [
    (dict(top_k=0), _abi.WR_ERR_INVALID),
    (dict(top_k=9), _abi.WR_ERR_INVALID),
    (dict(num_experts=65, top_k=2), _abi.WR_ERR_UNSUPPORTED),
    (dict(hidden_dim=0), _abi.WR_ERR_INVALID),
    (dict(dtype=7), _abi.WR_ERR_INVALID),
    (dict(ep_first=6, ep_num=4), _abi.WR_ERR_INVALID),
])
def test_bad_descriptor_rejected(kw, status):
    lib = _abi.load()
    d = _desc(**kw)
    st = lib.wr_fused_moe(ctypes.byref(d), FAKE, FAKE, FAKE, 1 << 40, FAKE, None, None, FAKE,
                          1 << 30, None)
    assert st == status
    assert lib.wr_last_error_string()


def test_weight_buffer_too_small_message():
    lib = _abi.load()
    d = _desc()
    need = lib.wr_total_weight_bytes(8, 512, 1024, 4)
    st = lib.wr_fused_moe(ctypes.byref(d), FAKE, FAKE, FAKE, need - 4, FAKE, None, None, FAKE,
                          1 << 30, None)
    assert st == _abi.WR_ERR_TOO_SMALL
    msg = lib.wr_last_error_string().decode()
    assert msg == f"weight_buf too small: need {need} bytes, got {need - 4}"


def test_workspace_checks():
    lib = _abi.load()
    d = _desc()
    need = lib.wr_fused_moe_workspace_size(ctypes.byref(d), 1)
    assert need > 0
    wbytes = lib.wr_total_weight_bytes(8, 512, 1024, 4)
    st = lib.wr_fused_moe(ctypes.byref(d), FAKE, FAKE, FAKE, wbytes, FAKE, None, None, None, 0, None)
    assert st == _abi.WR_ERR_WORKSPACE
    st = lib.wr_fused_moe(ctypes.byref(d), FAKE, FAKE, FAKE, wbytes, FAKE, None, None,
                          ctypes.c_void_p(0x10010), need, None)
    assert st == _abi.WR_ERR_WORKSPACE  # not 256-byte aligned
    st = lib.wr_fused_moe(ctypes.byref(d), FAKE, FAKE, FAKE, wbytes, FAKE, None, None, FAKE,
                          need - 1, None)
    assert st == _abi.WR_ERR_WORKSPACE  # too small


def test_workspace_sizes_cover_activations():
    lib = _abi.load()
    d = _abi.desc(8, 4096, 14336, 2, 1)
    n1 = lib.wr_fused_moe_workspace_size(ctypes.byref(d), 1)
    assert n1 >= 2 * 14336 * 4
    n16 = lib.wr_fused_moe_workspace_size(ctypes.byref(d), 16)
    assert n16 >= n1
    assert lib.wr_naive_moe_workspace_size(ctypes.byref(d)) >= 3 * 14336 * 4


def test_grouped_workspace_covers_its_buffers():
    """Batches of >= 2 bf16 tokens take the grouped path, whose workspace holds
    the bucketed tokens, the hi/lo activations and the down partial sums."""
    lib = _abi.load()
    E, H, I, K, T = 8, 4096, 14336, 2, 256
    d = _abi.desc(E, H, I, K, _abi.WR_DTYPE_BF16)
    need = lib.wr_fused_moe_workspace_size(ctypes.byref(d), T)
    rows = T * K  # at least one bucketed row per (token, expert) pair
    assert need >= rows * H * 2 + 2 * rows * I * 2 + 4 * rows * H * 4
    # one token keeps the streaming kernel's much smaller workspace
    assert lib.wr_fused_moe_workspace_size(ctypes.byref(d), 1) < rows * I * 2
    # fp32 batches of 3 or more tokens take the fp32 grouped path: the tokens
    # bucketed as bf16 hi and lo rows; 2 tokens stay on the streaming kernel
    d32 = _abi.desc(E, H, I, K, _abi.WR_DTYPE_F32)
    assert lib.wr_fused_moe_workspace_size(ctypes.byref(d32), T) >= 2 * rows * H * 2
    assert lib.wr_fused_moe_workspace_size(ctypes.byref(d32), 2) < rows * I * 2
    # grows with the batch
    assert lib.wr_fused_moe_workspace_size(ctypes.byref(d), 2 * T) > need


def test_empty_batch_needs_no_gpu():
    lib = _abi.load()
    d = _desc()
    st = lib.wr_batched_fused_moe(ctypes.byref(d), 0, FAKE, FAKE, FAKE, 0, None, None, None, None,
                                  0, None)
    assert st == _abi.WR_OK


def test_pack_experts_argument_checks():
    """wr_pack_experts rejects bad shards before touching any memory."""
    lib = _abi.load()
    P = ctypes.c_void_p * 8
    ptrs = P(*([0x1000] * 8))
    ok_args = dict(E=8, H=512, I=1024, dtype=_abi.WR_DTYPE_BF16, first=0, num=8, tpr=0, tps=1)

    def call(**kw):
        a = dict(ok_args, **kw)
        return lib.wr_pack_experts(a["E"], a["H"], a["I"], a["dtype"], a["first"], a["num"],
                                   a["tpr"], a["tps"], ptrs, ptrs, ptrs, FAKE,
                                   kw.get("bytes", 1 << 40), None)

    assert call(first=6, num=4) == _abi.WR_ERR_INVALID          # shard outside [0, E)
    assert call(tps=3) == _abi.WR_ERR_INVALID                   # 3 does not divide I
    assert call(tpr=2, tps=2) == _abi.WR_ERR_INVALID            # rank out of range
    assert call(dtype=7) == _abi.WR_ERR_INVALID
    need = 8 * lib.wr_total_weight_bytes(1, 512, 1024, 2)
    assert call(bytes=need - 1) == _abi.WR_ERR_TOO_SMALL
    assert "weight_buf too small" in lib.wr_last_error_string().decode()
    empty = P(*([None] * 8))
    st = lib.wr_pack_experts(8, 512, 1024, _abi.WR_DTYPE_BF16, 0, 8, 0, 1, empty, ptrs, ptrs,
                             FAKE, need, None)
    assert st == _abi.WR_ERR_INVALID                            # NULL matrix in the shard
