"""warp-route on B200: fused decode-time MoE layer (sm_100a kernels).

Same public surface as warp-route's warp_route package
(warp_route/__init__.py:1-105 of warp-route): `MoELayer` plus the functional
API re-exported here.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from .functional import (
    _expert_stride_elems,
    _pack_expert_weights,
    batched_fused_moe,
    fused_moe,
    fused_moe_batched,
    fused_moe_routed,
    moe_decode_layer,
    naive_moe,
    pack_expert_shard,
    router_topk,
)

__all__ = [
    "MoELayer",
    "fused_moe",
    "naive_moe",
    "batched_fused_moe",
    "fused_moe_batched",
    "fused_moe_routed",
    "moe_decode_layer",
    "router_topk",
    "pack_expert_shard",
    "_pack_expert_weights",
]


class MoELayer(nn.Module):
    """One MoE layer with per-expert SwiGLU FFN blocks.

    Same constructor, parameters and forward contract as warp-route's MoELayer
    (warp_route/__init__.py:10-105): router [E, H], ParameterLists gate_proj /
    up_proj / down_proj, N(0, 0.02) init, forward on [H] (one token) or
    [B, H] (a decode batch).  Differences: top_k may be any value in
    [1, num_experts]; `dtype` selects float32 (default) or bfloat16
    parameters; the output is float32; and the expert parameters are views
    into one packed [gate | up | down] buffer in the kernels' layout, so a
    forward hands that buffer to the kernel as it is (warp-route repacks
    every expert on every forward, warp_route/__init__.py:81).

    Because the parameters share the buffer's memory, every in-place write —
    `p.copy_(w)`, `p.data.copy_(w)`, an optimizer step, `load_state_dict` —
    is the packed buffer's content at once; nothing can go stale.  When a
    parameter stops being such a view (`module.to(...)`, `.cuda()`,
    `.bfloat16()`, assigning a new tensor to `p.data` or a new Parameter),
    the next forward repacks the parameters into a new buffer on their
    device and makes them views of it again.
    """

    def __init__(
        self,
        num_experts: int,
        hidden_dim: int,
        intermediate_dim: int,
        top_k: int = 2,
        dtype: torch.dtype = torch.float32,
    ) -> None:
        super().__init__()
        if not 1 <= top_k <= num_experts:
            raise ValueError(f"top_k must be in [1, num_experts={num_experts}], got {top_k}")
        if dtype not in (torch.float32, torch.bfloat16):
            raise ValueError(f"dtype must be float32 or bfloat16, got {dtype}")
        self.num_experts = num_experts
        self.hidden_dim = hidden_dim
        self.intermediate_dim = intermediate_dim
        self.top_k = top_k

        E, H, I = num_experts, hidden_dim, intermediate_dim
        self.router = nn.Parameter(torch.empty(E, H, dtype=dtype))
        buf = torch.zeros(E * _expert_stride_elems(H, I, torch.empty((), dtype=dtype).element_size()),
                          dtype=dtype)
        views = self._views(buf)
        self.gate_proj = nn.ParameterList([nn.Parameter(g) for g, _, _ in views])
        self.up_proj = nn.ParameterList([nn.Parameter(u) for _, u, _ in views])
        self.down_proj = nn.ParameterList([nn.Parameter(d) for _, _, d in views])
        self._packed: torch.Tensor = buf
        self._init_weights()

    def _init_weights(self) -> None:
        nn.init.normal_(self.router, std=0.02)
        for e in range(self.num_experts):
            nn.init.normal_(self.gate_proj[e], std=0.02)
            nn.init.normal_(self.up_proj[e], std=0.02)
            nn.init.normal_(self.down_proj[e], std=0.02)

    def _views(self, buf: torch.Tensor):
        """Per expert, the (gate [I,H], up [I,H], down [H,I]) views of a
        packed buffer (src/expert_layout.cuh:34-47 of warp-route)."""
        H, I = self.hidden_dim, self.intermediate_dim
        stride = _expert_stride_elems(H, I, buf.element_size())
        n = I * H
        out = []
        for e in range(self.num_experts):
            b = e * stride
            out.append((buf[b:b + n].view(I, H), buf[b + n:b + 2 * n].view(I, H),
                        buf[b + 2 * n:b + 3 * n].view(H, I)))
        return out

    def _params(self):
        return list(self.gate_proj) + list(self.up_proj) + list(self.down_proj)

    def _is_packed_view(self) -> bool:
        """Every expert parameter is still the view of the packed buffer at
        its own place (same memory, dtype and device)."""
        buf = self._packed
        for (g, u, d), pg, pu, pd in zip(self._views(buf), self.gate_proj, self.up_proj,
                                         self.down_proj):
            for v, p in ((g, pg), (u, pu), (d, pd)):
                if (p.data_ptr() != v.data_ptr() or p.dtype != buf.dtype
                        or p.device != buf.device or p.shape != v.shape):
                    return False
        return True

    def _pack_weights(self) -> torch.Tensor:
        """The packed [gate|up|down] buffer the kernels read.  It is the
        parameters' own memory; it is rebuilt (and the parameters re-pointed
        at it) only when a parameter no longer lives in it."""
        if not self._is_packed_view():
            buf = _pack_expert_weights(
                [p.data for p in self.gate_proj], [p.data for p in self.up_proj],
                [p.data for p in self.down_proj], self.num_experts, self.hidden_dim,
                self.intermediate_dim)
            for (g, u, d), pg, pu, pd in zip(self._views(buf), self.gate_proj, self.up_proj,
                                             self.down_proj):
                pg.data, pu.data, pd.data = g, u, d
            self._packed = buf
        return self._packed

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        weight_buf = self._pack_weights()
        router_w = self.router.data.contiguous()
        x = x.to(router_w.dtype)
        if x.dim() == 1:
            return fused_moe(x.contiguous(), router_w, weight_buf, self.num_experts,
                             self.hidden_dim, self.intermediate_dim, self.top_k)
        if x.dim() == 2:
            return batched_fused_moe(x.contiguous(), router_w, weight_buf, self.num_experts,
                                     self.hidden_dim, self.intermediate_dim, self.top_k)
        raise ValueError(f"Input must be 1D or 2D, got shape {x.shape}")
