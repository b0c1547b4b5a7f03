"""Decode-step driver: a stack of MoE layers replayed from one CUDA graph.

warp-route runs one layer per Python call and synchronises the device after
each (src/bindings.cpp:55,94,140); its README motivates the kernels with
decode-step latency (README.md:17).  `MoEStack` captures the whole stack of
layer calls for a fixed token count once and replays it every step:

    h_0 = x;   h_{l+1} = h_l + moe_l(h_l)   (residual add, in the layer dtype)

Each moe_l is this package's fused layer (`fused_moe_routed`: the streaming
kernel for one token, the grouped tcgen05 path for a batch), optionally
followed by a sum over ranks (`all_reduce`, e.g. torch.distributed.all_reduce
on an NCCL group: it is captured into the same graph) for tensor- or
expert-parallel shards.  Inputs and outputs live in static device buffers;
`step(x)` copies x in, replays, and returns the output buffer.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional

import torch

from .functional import fused_moe_routed


@dataclass
class StackLayer:
    """One layer's (shard of) weights: gate_w [E, H], the packed weight_buf,
    an optional fp32 router bias [E] and the expert-parallel shard."""
    gate_w: torch.Tensor
    weight_buf: torch.Tensor
    router_bias: Optional[torch.Tensor] = None
    ep_first_expert: int = 0
    ep_num_local: int = 0


class MoEStack:
    def __init__(self, layers: List[StackLayer], num_experts: int, hidden_dim: int,
                 intermediate_dim: int, top_k: int, tokens: int,
                 all_reduce: Optional[Callable[[torch.Tensor], None]] = None):
        if not layers:
            raise ValueError("MoEStack needs at least one layer")
        self.layers = layers
        self.E, self.H, self.I, self.K = num_experts, hidden_dim, intermediate_dim, top_k
        self.T = tokens
        self.all_reduce = all_reduce
        dev = layers[0].gate_w.device
        self.dtype = layers[0].gate_w.dtype
        shape = (hidden_dim,) if tokens == 1 else (tokens, hidden_dim)
        self.x_in = torch.zeros(shape, dtype=self.dtype, device=dev)
        self.h = [torch.zeros(shape, dtype=self.dtype, device=dev) for _ in range(2)]
        self.stream = torch.cuda.Stream(device=dev)
        self.graph: Optional[torch.cuda.CUDAGraph] = None

    def _layer(self, L: StackLayer, h: torch.Tensor) -> torch.Tensor:
        out, _, _ = fused_moe_routed(h, L.gate_w, L.weight_buf, self.E, self.H, self.I, self.K,
                                     router_bias=L.router_bias,
                                     ep_first_expert=L.ep_first_expert,
                                     ep_num_local=L.ep_num_local)
        if self.all_reduce is not None:
            self.all_reduce(out)
        return out

    def _forward(self) -> torch.Tensor:
        h = self.x_in
        for i, L in enumerate(self.layers):
            out = self._layer(L, h)
            nxt = self.h[i & 1]
            torch.add(h.float(), out, out=out)
            nxt.copy_(out)
            h = nxt
        return h

    def eager(self, x: torch.Tensor) -> torch.Tensor:
        """The same stack without a graph (for checking and for the first call)."""
        self.x_in.copy_(x)
        return self._forward().clone()

    def capture(self, warmup: int = 2) -> None:
        """Capture the stack into a CUDA graph (warm-up calls run first, on the
        capture stream, so the per-stream workspaces exist before capture)."""
        with torch.cuda.stream(self.stream):
            for _ in range(warmup):
                self._forward()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self.out = self._forward()
        self.graph = g

    def step(self, x: torch.Tensor) -> torch.Tensor:
        """One decode step: x -> the stack's output (a static buffer that the
        next step overwrites)."""
        if self.graph is None:
            self.capture()
        self.x_in.copy_(x)
        self.graph.replay()
        return self.out

    def close(self) -> None:
        """Release the graph (before destroying a process group it captured
        collectives of)."""
        self.graph = None
