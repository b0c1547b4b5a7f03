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
    _pack_expert_weights,
    batched_fused_moe,
    fused_moe,
    fused_moe_batched,
    fused_moe_routed,
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
    parameters; the packed weight buffer is cached and rebuilt only when a
    parameter changes (warp-route repacks every expert on every forward);
    the output is float32.
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

        self.router = nn.Parameter(torch.empty(num_experts, hidden_dim, dtype=dtype))
        self.gate_proj = nn.ParameterList(
            [nn.Parameter(torch.empty(intermediate_dim, hidden_dim, dtype=dtype))
             for _ in range(num_experts)])
        self.up_proj = nn.ParameterList(
            [nn.Parameter(torch.empty(intermediate_dim, hidden_dim, dtype=dtype))
             for _ in range(num_experts)])
        self.down_proj = nn.ParameterList(
            [nn.Parameter(torch.empty(hidden_dim, intermediate_dim, dtype=dtype))
             for _ in range(num_experts)])
        self._packed: Optional[torch.Tensor] = None
        self._packed_key = None
        self._init_weights()

    def _init_weights(self) -> None:
        nn.init.normal_(self.router, std=0.02)
        for e in range(self.num_experts):
            nn.init.normal_(self.gate_proj[e], std=0.02)
            nn.init.normal_(self.up_proj[e], std=0.02)
            nn.init.normal_(self.down_proj[e], std=0.02)
        self._packed = None

    def _params(self):
        return list(self.gate_proj) + list(self.up_proj) + list(self.down_proj)

    def _pack_weights(self) -> torch.Tensor:
        """Packed [gate|up|down] buffer, rebuilt only when a parameter's
        storage or version counter changed since the last pack."""
        key = tuple((p.data_ptr(), p._version, p.device, p.dtype) for p in self._params())
        if self._packed is None or key != self._packed_key:
            self._packed = _pack_expert_weights(
                [p.data for p in self.gate_proj], [p.data for p in self.up_proj],
                [p.data for p in self.down_proj], self.num_experts, self.hidden_dim,
                self.intermediate_dim)
            self._packed_key = key
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
