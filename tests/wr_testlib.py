"""Test helpers: call the C ABI on torch-owned device buffers, and move
device tensors into the oracle's numpy form."""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch

from warp_route import _abi


def dtype_code(t: torch.Tensor) -> int:
    return _abi.WR_DTYPE_BF16 if t.dtype == torch.bfloat16 else _abi.WR_DTYPE_F32


def host_array(t: torch.Tensor) -> np.ndarray:
    """float32 -> float32 ndarray; bfloat16 -> uint16 ndarray of the raw bits."""
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy().astype(np.float32, copy=False)


def ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_ptr():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def abi_layer(x, gate_w, wbuf, E, H, I, K, *, bias=None, ep_first=0, ep_num=0, ws=None,
              naive=False):
    """Run one layer through the C ABI.  x [H] -> wr_fused_moe, x [T,H] ->
    wr_batched_fused_moe, naive=True -> wr_naive_moe.  Returns
    (out fp32, ids int32 [T,K] or None, weights fp32 [T,K] or None)."""
    lib = _abi.load()
    d = _abi.desc(E, H, I, K, dtype_code(x), ep_first, ep_num,
                  bias.data_ptr() if bias is not None else 0)
    T = 1 if x.dim() == 1 else x.shape[0]
    out = torch.full(tuple(x.shape), float("nan"), dtype=torch.float32, device=x.device)
    ids = torch.full((T, K), -1, dtype=torch.int32, device=x.device)
    w = torch.full((T, K), float("nan"), dtype=torch.float32, device=x.device)
    wbytes = wbuf.numel() * wbuf.element_size()
    if naive:
        need = lib.wr_naive_moe_workspace_size(ctypes.byref(d))
        if ws is None:
            ws = torch.zeros(need, dtype=torch.uint8, device=x.device)
        _abi.check(lib.wr_naive_moe(ctypes.byref(d), ptr(x), ptr(gate_w), ptr(wbuf), wbytes,
                                    ptr(out), ptr(ws), ws.numel(), stream_ptr()))
        return out, None, None
    need = lib.wr_fused_moe_workspace_size(ctypes.byref(d), T)
    if ws is None:
        ws = torch.zeros(need, dtype=torch.uint8, device=x.device)
    if x.dim() == 1:
        st = lib.wr_fused_moe(ctypes.byref(d), ptr(x), ptr(gate_w), ptr(wbuf), wbytes, ptr(out),
                              ptr(ids), ptr(w), ptr(ws), ws.numel(), stream_ptr())
    else:
        st = lib.wr_batched_fused_moe(ctypes.byref(d), T, ptr(x), ptr(gate_w), ptr(wbuf), wbytes,
                                      ptr(out), ptr(ids), ptr(w), ptr(ws), ws.numel(),
                                      stream_ptr())
    _abi.check(st)
    _abi.check(lib.wr_workspace_status(ptr(ws), stream_ptr()))
    return out, ids, w


def oracle_inputs_from_device(x, gate_w, wbuf, E, H, I, K, bias=None, ep_first=0, ep_num=0):
    """Host copies for the oracle.  Only the experts the oracle's own router
    selects are copied out of the (possibly multi-GB) device buffer; the rest
    of the host buffer stays as untouched zero pages."""
    import oracle

    xa = host_array(x).reshape(-1, H)
    gwa = host_array(gate_w)
    ba = None if bias is None else bias.detach().cpu().numpy().astype(np.float32)
    _, ids, _ = oracle.router(np.ascontiguousarray(xa), gwa, K, ba)
    elt = wbuf.element_size()
    stride = oracle.expert_stride(H, I, elt)
    n_local = ep_num if ep_num else E
    host = np.zeros(n_local * stride, np.uint8)
    raw = wbuf.view(torch.uint8)
    first = ep_first if ep_num else 0
    for e in sorted(set(int(v) for v in ids.ravel())):
        if e < first or e >= first + n_local:
            continue
        j = e - first
        host[j * stride:(j + 1) * stride] = raw[j * stride:(j + 1) * stride].cpu().numpy()
    return xa, gwa, host, ba
