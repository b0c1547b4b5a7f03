"""Functional API of warp-route, backed by the B200-native kernels.

Drop-in for warp-route's warp_route/functional.py: the same names, positional
signatures and error behaviour (`_pack_expert_weights`, `fused_moe`,
`naive_moe`, `batched_fused_moe`), plus `fused_moe_batched` (alias of
`batched_fused_moe`) and a few keyword-only extras.

Differences a caller may notice (all additive):
  * float32 or bfloat16 inputs (x, gate_w and weight_buf share one dtype);
    the output is always float32 — bf16 rounding of the output alone would
    cost ~2e-3 relative error;
  * top_k may be anything in [1, num_experts] (num_experts <= 64);
  * calls are asynchronous on the current CUDA stream (warp-route calls
    cudaDeviceSynchronize after each launch);
  * optional `router_bias` (fp32 [E], added to the logits).
There is no CPU fallback: without the compiled extension every call raises.
"""
from __future__ import annotations

import functools
from typing import List, Optional, Tuple

import torch


@functools.lru_cache(maxsize=1)
def _load_extension():
    """Import warp_route._C (warp_route/functional.py:9-18 of warp-route)."""
    try:
        from . import _C  # noqa: F401  (built in-tree by warp-route_b200/build.py)
        return _C
    except ImportError as e:
        raise ImportError(
            "warp_route._C extension not found or failed to load "
            f"({e}). Build it with: python warp-route_b200/build.py "
            "(requires nvcc for sm_100a and PyTorch)"
        ) from e


def _expert_stride_elems(hidden_dim: int, intermediate_dim: int, elt: int) -> int:
    raw = (2 * intermediate_dim * hidden_dim + hidden_dim * intermediate_dim) * elt
    return ((raw + 127) & ~127) // elt


def _pack_expert_weights(
    gate_proj: List[torch.Tensor],
    up_proj: List[torch.Tensor],
    down_proj: List[torch.Tensor],
    num_experts: int,
    hidden_dim: int,
    intermediate_dim: int,
) -> torch.Tensor:
    """Pack per-expert weights into the flat layout the kernels read.

    Per expert, row-major: [gate I x H][up I x H][down H x I]; each expert
    block starts on a 128-byte boundary (warp_route/functional.py:21-57 and
    src/expert_layout.cuh:34-47 of warp-route).  The buffer keeps the dtype of
    the inputs (float32 or bfloat16) and lives on gate_proj[0]'s device.
    """
    dtype = gate_proj[0].dtype
    if dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"expert weights must be float32 or bfloat16, got {dtype}")
    elt = torch.empty((), dtype=dtype).element_size()
    n = intermediate_dim * hidden_dim
    stride = _expert_stride_elems(hidden_dim, intermediate_dim, elt)
    device = gate_proj[0].device
    buf = torch.zeros(num_experts * stride, dtype=dtype, device=device)
    for e in range(num_experts):
        base = e * stride
        buf[base:base + n] = gate_proj[e].contiguous().view(-1).to(dtype)
        buf[base + n:base + 2 * n] = up_proj[e].contiguous().view(-1).to(dtype)
        buf[base + 2 * n:base + 3 * n] = down_proj[e].contiguous().view(-1).to(dtype)
    return buf


def fused_moe(
    x: torch.Tensor,
    gate_w: torch.Tensor,
    weight_buf: torch.Tensor,
    num_experts: int,
    hidden_dim: int,
    intermediate_dim: int,
    top_k: int,
    *,
    router_bias: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """One decode token: x [hidden_dim] -> float32 [hidden_dim]."""
    _C = _load_extension()
    if router_bias is None:
        return _C.fused_moe_forward(x, gate_w, weight_buf, num_experts, hidden_dim,
                                    intermediate_dim, top_k)
    if x.dim() != 1:
        raise ValueError(f"fused_moe expects 1D input [hidden], got shape {tuple(x.shape)}")
    return _C.fused_moe_routed(x, gate_w, weight_buf, num_experts, hidden_dim,
                               intermediate_dim, top_k, router_bias)[0]


def naive_moe(
    x: torch.Tensor,
    gate_w: torch.Tensor,
    weight_buf: torch.Tensor,
    num_experts: int,
    hidden_dim: int,
    intermediate_dim: int,
    top_k: int,
) -> torch.Tensor:
    """One decode token through the unfused kernel-per-step path."""
    _C = _load_extension()
    return _C.naive_moe_forward(x, gate_w, weight_buf, num_experts, hidden_dim,
                                intermediate_dim, top_k)


def batched_fused_moe(
    x: torch.Tensor,
    gate_w: torch.Tensor,
    weight_buf: torch.Tensor,
    num_experts: int,
    hidden_dim: int,
    intermediate_dim: int,
    top_k: int,
    *,
    router_bias: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Decode batch: x [batch, hidden_dim] -> float32 [batch, hidden_dim]."""
    if x.dim() != 2:
        raise ValueError(f"batched_fused_moe expects 2D input [batch, hidden], got shape {x.shape}")
    batch_size, hd = x.shape
    if hd != hidden_dim:
        raise ValueError(f"Input hidden dim {hd} does not match hidden_dim={hidden_dim}")
    _C = _load_extension()
    if router_bias is None:
        return _C.batched_fused_moe_forward(x, gate_w, weight_buf, num_experts, hidden_dim,
                                            intermediate_dim, top_k)
    return _C.fused_moe_routed(x, gate_w, weight_buf, num_experts, hidden_dim,
                               intermediate_dim, top_k, router_bias)[0]


# The name used by the batched benchmark configuration.
fused_moe_batched = batched_fused_moe


def fused_moe_routed(
    x: torch.Tensor,
    gate_w: torch.Tensor,
    weight_buf: torch.Tensor,
    num_experts: int,
    hidden_dim: int,
    intermediate_dim: int,
    top_k: int,
    *,
    router_bias: Optional[torch.Tensor] = None,
    ep_first_expert: int = 0,
    ep_num_local: int = 0,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Layer output plus its routing: (out fp32, expert ids int32 [T,K],
    weights fp32 [T,K]).  x is [H] or [T,H].  With ep_num_local > 0 the
    weight_buf holds experts [ep_first_expert, ep_first_expert + ep_num_local)
    only, and the output is this shard's partial sum."""
    _C = _load_extension()
    return _C.fused_moe_routed(x, gate_w, weight_buf, num_experts, hidden_dim,
                               intermediate_dim, top_k, router_bias, ep_first_expert,
                               ep_num_local)


def router_topk(
    x: torch.Tensor,
    gate_w: torch.Tensor,
    num_experts: int,
    hidden_dim: int,
    top_k: int,
    *,
    router_bias: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Router only: (logits fp32 [T,E], ids int32 [T,K], weights fp32 [T,K])."""
    _C = _load_extension()
    return _C.router_topk(x, gate_w, num_experts, hidden_dim, top_k, router_bias)
