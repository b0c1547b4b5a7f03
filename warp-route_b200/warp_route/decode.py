"""Decode-step driver: a stack of MoE layers replayed from one CUDA graph.

warp-route runs one layer per Python call and synchronises the device after
each (src/bindings.cpp:55,94,140); its README motivates the kernels with
decode-step latency (README.md:17).  `MoEStack` captures the whole stack of
layer calls for a fixed token count once and replays it every step:

    h_0 = x;   h_{l+1} = (h_l + moe_l(h_l)).to(dtype)   (residual, fp32 add, one rounding)

Each layer is ONE kernel launch chain of this package: `moe_decode_layer`
writes both the fp32 sum and the next layer's input from the layer's last
step (the streaming kernel for a token, the grouped tcgen05 path for a
batch), so consecutive layers follow each other with programmatic dependent
launch and no element-wise kernels in between.  Tensor- or expert-parallel
shards pass `comm` (a `PeerComm`): the ranks' partial outputs are summed in
the same kernel before the residual.  An external collective (`all_reduce`,
e.g. torch.distributed.all_reduce on NCCL, captured into the same graph)
still works; the residual is then added after it, as two extra kernels.
Inputs and outputs live in static device buffers; `step(x)` copies x in,
replays, and returns the output buffer.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional

import torch

from .functional import PeerComm, fused_moe_routed, moe_decode_layer


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
                 all_reduce: Optional[Callable[[torch.Tensor], None]] = None,
                 comm: Optional[PeerComm] = None):
        if not layers:
            raise ValueError("MoEStack needs at least one layer")
        if all_reduce is not None and comm is not None:
            raise ValueError("pass either comm (fused sum) or all_reduce (external), not both")
        self.layers = layers
        self.E, self.H, self.I, self.K = num_experts, hidden_dim, intermediate_dim, top_k
        self.T = tokens
        self.all_reduce = all_reduce
        self.comm = comm
        dev = layers[0].gate_w.device
        self.dtype = layers[0].gate_w.dtype
        shape = (hidden_dim,) if tokens == 1 else (tokens, hidden_dim)
        self.x_in = torch.zeros(shape, dtype=self.dtype, device=dev)
        self.h = [torch.zeros(shape, dtype=self.dtype, device=dev) for _ in range(2)]
        self.stream = torch.cuda.Stream(device=dev)
        self.graph: Optional[torch.cuda.CUDAGraph] = None

    def layer(self, i: int, h: torch.Tensor, nxt: torch.Tensor) -> torch.Tensor:
        """Layer i on input h: writes the next input into nxt and returns the
        layer's fp32 output (residual included)."""
        L = self.layers[i]
        if self.all_reduce is None:
            return moe_decode_layer(h, L.gate_w, L.weight_buf, self.E, self.H, self.I, self.K,
                                    next_x=nxt, comm=self.comm, router_bias=L.router_bias,
                                    ep_first_expert=L.ep_first_expert,
                                    ep_num_local=L.ep_num_local)
        out, _, _ = fused_moe_routed(h, L.gate_w, L.weight_buf, self.E, self.H, self.I, self.K,
                                     router_bias=L.router_bias,
                                     ep_first_expert=L.ep_first_expert,
                                     ep_num_local=L.ep_num_local)
        self.all_reduce(out)
        torch.add(h.float(), out, out=out)
        nxt.copy_(out)
        return out

    def _forward(self) -> torch.Tensor:
        h = self.x_in
        for i in range(len(self.layers)):
            nxt = self.h[i & 1]
            self.layer(i, h, nxt)
            h = nxt
        return h

    def eager(self, x: torch.Tensor) -> torch.Tensor:
        """The same stack without a graph (for checking and for the first call)."""
        self.x_in.copy_(x)
        return self._forward().clone()

    def capture(self, warmup: int = 2) -> None:
        """Capture the stack into a CUDA graph (warm-up calls run first, on the
        capture stream, so the per-stream workspaces exist before capture)."""
        # the capture stream's warm-up writes the same static buffers as any
        # call already queued on the caller's stream: run it after them
        self.stream.wait_stream(torch.cuda.current_stream())
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
