"""TEST INFRASTRUCTURE ONLY: ctypes front end of the CPU oracle (moe_oracle.c).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, always as the checker.  The product (warp-route_b200/) never imports
it.  See moe_oracle.c for what is restated from warp-route and where.

Arrays are numpy: float32 for fp32 data, uint16 (raw bf16 bits) for bf16.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libwr_oracle.so")
_lib = None

F32 = 0
BF16 = 1


def build() -> str:
    """Compile moe_oracle.c into oracle/libwr_oracle.so (make, incremental)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH) or (
        os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "moe_oracle.c"))
    ):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    vp, ip = ctypes.c_void_p, ctypes.c_int
    lib.wro_expert_stride.restype = ctypes.c_int64
    lib.wro_expert_stride.argtypes = [ip, ip, ip]
    lib.wro_router.restype = ip
    lib.wro_router.argtypes = [vp, vp, vp, ip, ip, ip, ip, ip, vp, vp, vp]
    lib.wro_moe.restype = ip
    lib.wro_moe.argtypes = [vp, vp, vp, vp, ip, ip, ip, ip, ip, ip, ip, ip, vp, vp, vp]
    lib.wro_pack.restype = ip
    lib.wro_pack.argtypes = [vp, vp, vp, ip, ip, ip, ip, vp]
    _lib = lib
    return lib


def _ptr(a: Optional[np.ndarray]):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def _dtype_code(a: np.ndarray) -> int:
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.uint16:
        return BF16
    raise TypeError(f"oracle arrays must be float32 or uint16 (bf16 bits), got {a.dtype}")


def expert_stride(hidden: int, inter: int, elt: int) -> int:
    return int(_load().wro_expert_stride(hidden, inter, elt))


def router(x: np.ndarray, gate_w: np.ndarray, top_k: int,
           bias: Optional[np.ndarray] = None) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """x [T,H] or [H]; gate_w [E,H].  Returns (logits [T,E], ids [T,K], weights [T,K])."""
    lib = _load()
    x2 = np.ascontiguousarray(x.reshape(-1, x.shape[-1]))
    T, H = x2.shape
    E = gate_w.shape[0]
    dt = _dtype_code(x2)
    assert _dtype_code(gate_w) == dt
    gw = np.ascontiguousarray(gate_w)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    logits = np.zeros((T, E), np.float32)
    ids = np.zeros((T, top_k), np.int32)
    w = np.zeros((T, top_k), np.float32)
    rc = lib.wro_router(_ptr(x2), _ptr(gw), _ptr(b), dt, T, E, H, top_k,
                        _ptr(logits), _ptr(ids), _ptr(w))
    if rc:
        raise ValueError(f"oracle router failed ({rc})")
    return logits, ids, w


def moe(x: np.ndarray, gate_w: np.ndarray, wbuf: np.ndarray, num_experts: int,
        hidden: int, inter: int, top_k: int, bias: Optional[np.ndarray] = None,
        ep_first: int = 0, ep_num: int = 0) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Full layer.  x [T,H] or [H]; wbuf is the packed buffer (any dtype view of
    the raw bytes, element type taken from x).  Returns (out fp32 [T,H] or [H],
    ids [T,K], weights [T,K])."""
    lib = _load()
    squeeze = x.ndim == 1
    x2 = np.ascontiguousarray(x.reshape(-1, hidden))
    T = x2.shape[0]
    dt = _dtype_code(x2)
    assert _dtype_code(gate_w) == dt
    gw = np.ascontiguousarray(gate_w)
    wb = np.ascontiguousarray(wbuf)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    out = np.zeros((T, hidden), np.float32)
    ids = np.zeros((T, top_k), np.int32)
    w = np.zeros((T, top_k), np.float32)
    rc = lib.wro_moe(_ptr(x2), _ptr(gw), _ptr(b), _ptr(wb), dt, T, num_experts, hidden,
                     inter, top_k, ep_first, ep_num, _ptr(out), _ptr(ids), _ptr(w))
    if rc:
        raise ValueError(f"oracle moe failed ({rc})")
    return (out[0] if squeeze else out), ids, w


def pack(gate: np.ndarray, up: np.ndarray, down: np.ndarray) -> np.ndarray:
    """gate/up [E,I,H], down [E,H,I] (float32 or uint16) -> packed uint8 buffer."""
    lib = _load()
    E, I, H = gate.shape
    dt = _dtype_code(gate)
    elt = 2 if dt == BF16 else 4
    stride = expert_stride(H, I, elt)
    dst = np.empty(E * stride, np.uint8)
    g, u, d = (np.ascontiguousarray(a) for a in (gate, up, down))
    lib.wro_pack(_ptr(g), _ptr(u), _ptr(d), dt, E, H, I, _ptr(dst))
    return dst


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    """||a - b|| / ||b|| in float64 (b is the reference)."""
    a64 = np.asarray(a, np.float64).ravel()
    b64 = np.asarray(b, np.float64).ravel()
    den = np.linalg.norm(b64)
    return float(np.linalg.norm(a64 - b64) / (den if den > 0 else 1.0))
