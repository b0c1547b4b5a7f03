"""TEST INFRASTRUCTURE ONLY: warp-route's PyTorch CPU composition, restated.

warp-route's own CPU path for this layer is the pure-torch composition
`torch_moe_reference` (tests/test_python.py:15-37 in the warp-route project):
router matmul -> softmax -> torch.topk -> per selected expert
silu(Wg x) * (Wu x) -> Wd -> weighted sum.  The reference tree does not exist
on the GPU box, so this module restates that composition (same torch ops, same
order) for bench.py's CPU baseline and its `--impl reference` arm, and as a
second cross-check in tests/.  Weights are read as views of the packed
[gate | up | down] buffer (warp_route/functional.py:21-57 layout).
"""
from __future__ import annotations

from typing import List, Tuple

import torch


def expert_views(weight_buf: torch.Tensor, num_experts: int, hidden: int,
                 inter: int) -> Tuple[List[torch.Tensor], List[torch.Tensor], List[torch.Tensor]]:
    """Per-expert (gate [I,H], up [I,H], down [H,I]) views into a packed 1-D buffer."""
    elt = weight_buf.element_size()
    raw = (2 * inter * hidden + hidden * inter) * elt
    stride = ((raw + 127) // 128) * 128 // elt
    n = inter * hidden
    gate, up, down = [], [], []
    for e in range(num_experts):
        base = e * stride
        gate.append(weight_buf[base:base + n].view(inter, hidden))
        up.append(weight_buf[base + n:base + 2 * n].view(inter, hidden))
        down.append(weight_buf[base + 2 * n:base + 3 * n].view(hidden, inter))
    return gate, up, down


def moe_forward(hidden: torch.Tensor, gate_w: torch.Tensor, gate: List[torch.Tensor],
                up: List[torch.Tensor], down: List[torch.Tensor], top_k: int,
                router_bias: torch.Tensor | None = None) -> torch.Tensor:
    """One token, in hidden's dtype, exactly as the reference composes it."""
    logits = gate_w @ hidden
    if router_bias is not None:
        logits = logits + router_bias.to(logits.dtype)
    probs = torch.softmax(logits, dim=0)
    weights, indices = torch.topk(probs, top_k)
    out = torch.zeros_like(hidden)
    for k in range(top_k):
        e = int(indices[k].item())
        w = weights[k].item()
        g = gate[e] @ hidden
        u = up[e] @ hidden
        act = g * torch.sigmoid(g) * u
        out += w * (down[e] @ act)
    return out
