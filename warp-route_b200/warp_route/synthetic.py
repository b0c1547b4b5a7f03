"""Seeded synthetic MoE layers, generated on the device, for benchmarks and
full-size tests.

Init of the benchmark configurations: x ~ N(0,1), router ~ N(0, 0.02),
gate/up ~ N(0, 1/sqrt(H)), down ~ N(0, 1/sqrt(I)), optional per-expert router
bias ~ N(0, 1).  Every expert is drawn from its own generator (seed, layer,
expert), so a tensor-parallel rank can draw the full expert and keep only its
slice, and every rank sees the same layer.  No public dataset is involved.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from .functional import _expert_stride_elems

# (name) -> (E, H, I, top_k)
SHAPES = {
    "tiny": (8, 512, 1024, 2),
    "mixtral": (8, 4096, 14336, 2),
    "deepseek": (64, 2048, 1408, 6),
    "dbrx": (16, 6144, 10752, 4),
}


@dataclass
class Layer:
    x: torch.Tensor            # [H] or [T, H]
    gate_w: torch.Tensor       # [E, H]
    weight_buf: torch.Tensor   # packed local experts (1-D, dtype)
    router_bias: Optional[torch.Tensor]
    E: int
    H: int
    I: int                     # intermediate size held by this buffer (I / tp under TP)
    K: int
    ep_first: int = 0
    ep_num: int = 0            # 0: all experts local


def _gen(device, *seeds: int) -> torch.Generator:
    g = torch.Generator(device=device)
    s = 0
    for v in seeds:
        s = (s * 1000003 + int(v) + 1) % (2 ** 62)
    g.manual_seed(s)
    return g


def make_layer(E: int, H: int, I: int, K: int, *, dtype=torch.bfloat16, device="cuda",
               seed: int = 0, layer: int = 0, tokens: int = 1, router_bias: bool = False,
               tp_rank: int = 0, tp_size: int = 1, ep_rank: int = 0, ep_size: int = 1,
               x: Optional[torch.Tensor] = None, gate_w: Optional[torch.Tensor] = None) -> Layer:
    """One layer on `device`.  With tp_size > 1 the buffer holds this rank's
    I/tp slice of every (local) expert; with ep_size > 1 it holds experts
    [ep_rank*E/ep, (ep_rank+1)*E/ep).  x / gate_w may be passed in to share
    them across layers."""
    if I % tp_size:
        raise ValueError(f"intermediate_dim {I} not divisible by tp_size {tp_size}")
    if E % ep_size:
        raise ValueError(f"num_experts {E} not divisible by ep_size {ep_size}")
    Il = I // tp_size
    e0, ne = ep_rank * (E // ep_size), E // ep_size
    if x is None:
        shape = (H,) if tokens == 1 else (tokens, H)
        x = torch.randn(*shape, generator=_gen(device, seed, 1), device=device,
                        dtype=torch.float32).to(dtype)
    if gate_w is None:
        gate_w = (torch.randn(E, H, generator=_gen(device, seed, 2), device=device,
                              dtype=torch.float32) * 0.02).to(dtype)
    bias = None
    if router_bias:
        bias = torch.randn(E, generator=_gen(device, seed, 3), device=device, dtype=torch.float32)
    elt = torch.empty((), dtype=dtype).element_size()
    stride = _expert_stride_elems(H, Il, elt)
    buf = torch.zeros(ne * stride, dtype=dtype, device=device)
    n = Il * H
    lo, hi = tp_rank * Il, (tp_rank + 1) * Il
    for j in range(ne):
        e = e0 + j
        g = _gen(device, seed, 100, layer, e)
        base = j * stride
        gate = torch.randn(I, H, generator=g, device=device, dtype=torch.float32) / H ** 0.5
        buf[base:base + n] = gate[lo:hi].reshape(-1).to(dtype)
        del gate
        up = torch.randn(I, H, generator=g, device=device, dtype=torch.float32) / H ** 0.5
        buf[base + n:base + 2 * n] = up[lo:hi].reshape(-1).to(dtype)
        del up
        down = torch.randn(H, I, generator=g, device=device, dtype=torch.float32) / I ** 0.5
        buf[base + 2 * n:base + 3 * n] = down[:, lo:hi].contiguous().reshape(-1).to(dtype)
        del down
    return Layer(x=x, gate_w=gate_w, weight_buf=buf, router_bias=bias, E=E, H=H, I=Il, K=K,
                 ep_first=e0 if ep_size > 1 else 0, ep_num=ne if ep_size > 1 else 0)


def algorithmic_bytes(E: int, H: int, I: int, distinct_experts: int, tokens: int, elt: int) -> int:
    """Bytes one layer must move: the selected experts' weights, the router,
    the input tokens and the fp32 output."""
    return distinct_experts * 3 * H * I * elt + E * H * elt + tokens * H * elt + tokens * H * 4
