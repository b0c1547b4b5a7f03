"""ctypes view of the C ABI in include/warp_route_b200.h.

This is the binding a non-torch caller would write; the tests use it to
drive the kernels through the exact C entry points.  Loading
fails loudly when libwarp_route_b200.so is missing — there is no fallback.
"""
from __future__ import annotations

import ctypes
import os

LIB_NAME = "libwarp_route_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

WR_OK = 0
WR_ERR_INVALID = 1
WR_ERR_UNSUPPORTED = 2
WR_ERR_CUDA = 3
WR_ERR_TIMEOUT = 4
WR_ERR_WORKSPACE = 5
WR_ERR_TOO_SMALL = 6
WR_ERR_COMM = 7

WR_DTYPE_F32 = 0
WR_DTYPE_BF16 = 1

# Every function the header declares, with (restype, argtypes).
_vp, _i32, _i64, _sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t


class MoeDesc(ctypes.Structure):
    _fields_ = [
        ("num_experts", ctypes.c_int32),
        ("hidden_dim", ctypes.c_int32),
        ("intermediate_dim", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("ep_first_expert", ctypes.c_int32),
        ("ep_num_local", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("router_bias", ctypes.c_void_p),
    ]


class ExpertOffsets(ctypes.Structure):
    _fields_ = [
        ("gate_proj_offset", ctypes.c_int64),
        ("up_proj_offset", ctypes.c_int64),
        ("down_proj_offset", ctypes.c_int64),
        ("expert_stride", ctypes.c_int64),
    ]


_D = ctypes.POINTER(MoeDesc)
SIGNATURES = {
    "wr_expert_offsets": (_i32, [_i32, _i32, _i32, ctypes.POINTER(ExpertOffsets)]),
    "wr_total_weight_bytes": (_i64, [_i32, _i32, _i32, _i32]),
    "wr_status_string": (ctypes.c_char_p, [_i32]),
    "wr_last_error_string": (ctypes.c_char_p, []),
    "wr_version": (ctypes.c_char_p, []),
    "wr_router_topk": (_i32, [_D, _i32, _vp, _vp, _vp, _vp, _vp, _vp]),
    "wr_fused_moe_workspace_size": (_sz, [_D, _i32]),
    "wr_fused_moe": (_i32, [_D, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "wr_fused_moe_noalloc": (_i32, [_D, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp]),
    "wr_fused_moe_noalloc_status": (_i32, [_vp]),
    "wr_batched_fused_moe": (_i32, [_D, _i32, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "wr_naive_moe_workspace_size": (_sz, [_D]),
    "wr_naive_moe": (_i32, [_D, _vp, _vp, _vp, _i64, _vp, _vp, _sz, _vp]),
    "wr_workspace_status": (_i32, [_vp, _vp]),
    "wr_pack_experts": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
                               ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                               _vp, _i64, _vp]),
    "wr_comm_handle_bytes": (_sz, []),
    "wr_comm_create": (_i32, [_i32, _i32, _i32, ctypes.POINTER(_vp)]),
    "wr_comm_get_handle": (_i32, [_vp, _vp]),
    "wr_comm_open": (_i32, [_vp, _vp]),
    "wr_comm_destroy": (_i32, [_vp]),
    "wr_comm_set_peer_timeout_ns": (_i32, [_vp, ctypes.c_uint64]),
    "wr_comm_reset": (_i32, [_vp, _vp]),
    "wr_fused_moe_allreduce": (_i32, [_D, _i32, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _sz, _vp,
                                      _vp]),
    "wr_moe_decode_layer": (_i32, [_D, _i32, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _sz,
                                   _vp, _vp]),
}

_lib = None


def load(path: str = LIB_PATH):
    """dlopen the library and set every prototype.  Raises OSError if absent."""
    global _lib
    if _lib is not None and path == LIB_PATH:
        return _lib
    if not os.path.exists(path):
        raise OSError(f"{path} not found: build it with python warp-route_b200/build.py")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path == LIB_PATH:
        _lib = lib
    return lib


class WrError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{msg} [status {status}]")
        self.status = status


def check(status: int) -> None:
    if status != WR_OK:
        raise WrError(status, load().wr_last_error_string().decode())


def desc(num_experts: int, hidden_dim: int, intermediate_dim: int, top_k: int, dtype: int,
         ep_first_expert: int = 0, ep_num_local: int = 0, router_bias_ptr: int = 0) -> MoeDesc:
    return MoeDesc(num_experts, hidden_dim, intermediate_dim, top_k, dtype, ep_first_expert,
                   ep_num_local, 0, router_bias_ptr or None)
