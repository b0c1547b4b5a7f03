"""Seeded CPU input generators that follow warp-route's own tests draw for draw.

Used by tests/golden/make_golden.py (which runs the reference's composition on
these inputs) and by the tests that check the oracle and the CUDA path against
the committed fixtures.  torch's CPU generator is deterministic for a given
torch version, and each fixture stores checksums of its inputs so a drift in
the generator shows up as a failed checksum, not as a parity failure.
"""
from __future__ import annotations

from typing import List, Tuple

import numpy as np
import torch

Experts = Tuple[List[torch.Tensor], List[torch.Tensor], List[torch.Tensor]]


def reference_test_inputs(E: int, H: int, I: int, seed: int = 42, experts: bool = True):
    """tests/test_python.py:55-60 with make_expert_tensors :40-48 (device=cpu):
    seed -> x*0.1, router*0.02; seed+1 -> all gate, all up, all down, *0.01.
    experts=False skips the (last-drawn) expert weights."""
    torch.manual_seed(seed)
    x = torch.randn(H, dtype=torch.float32) * 0.1
    gate_w = torch.randn(E, H, dtype=torch.float32) * 0.02
    if not experts:
        return x, gate_w, None
    torch.manual_seed(seed + 1)
    gate = [torch.randn(I, H, dtype=torch.float32) * 0.01 for _ in range(E)]
    up = [torch.randn(I, H, dtype=torch.float32) * 0.01 for _ in range(E)]
    down = [torch.randn(H, I, dtype=torch.float32) * 0.01 for _ in range(E)]
    return x, gate_w, (gate, up, down)


def reference_batched_inputs(E: int, H: int, I: int, B: int, seed: int = 42,
                             experts: bool = True):
    """tests/test_batched.py:9-23 (device=cpu), called with seed=42 as
    run_correctness does (:26-30): one stream for x, router and experts."""
    torch.manual_seed(seed)
    x = torch.randn(B, H, dtype=torch.float32) * 0.1
    gate_w = torch.randn(E, H, dtype=torch.float32) * 0.02
    if not experts:
        return x, gate_w, None
    gate = [torch.randn(I, H, dtype=torch.float32) * 0.01 for _ in range(E)]
    up = [torch.randn(I, H, dtype=torch.float32) * 0.01 for _ in range(E)]
    down = [torch.randn(H, I, dtype=torch.float32) * 0.01 for _ in range(E)]
    return x, gate_w, (gate, up, down)


def baseline_inputs(E: int, H: int, I: int, seed: int = 0, tokens: int = 1,
                    experts: bool = True):
    """The benchmark configurations' init: x~N(0,1), router~N(0,0.02),
    gate/up~N(0,1/sqrt(H)), down~N(0,1/sqrt(I)); draw order x, router,
    all gate, all up, all down."""
    torch.manual_seed(seed)
    shape = (H,) if tokens == 1 else (tokens, H)
    x = torch.randn(*shape, dtype=torch.float32)
    gate_w = torch.randn(E, H, dtype=torch.float32) * 0.02
    if not experts:
        return x, gate_w, None
    gate = [torch.randn(I, H, dtype=torch.float32) / H ** 0.5 for _ in range(E)]
    up = [torch.randn(I, H, dtype=torch.float32) / H ** 0.5 for _ in range(E)]
    down = [torch.randn(H, I, dtype=torch.float32) / I ** 0.5 for _ in range(E)]
    return x, gate_w, (gate, up, down)


def round_bf16(t: torch.Tensor) -> torch.Tensor:
    """Round to bf16 (nearest-even) and widen back to fp32."""
    return t.to(torch.bfloat16).to(torch.float32)


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    """Raw bf16 bits (uint16) of t rounded to bf16."""
    return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)


def pack_numpy(experts: Experts, bf16: bool = False, only=None) -> np.ndarray:
    """Packed [gate | up | down] buffer (uint8 bytes) in warp-route's layout
    (bf16=True rounds each weight to bf16).  `only`: the experts to fill in
    (the others stay zero), e.g. the selected ones when only they are read."""
    gate, up, down = experts
    E = len(gate)
    I, H = gate[0].shape
    elt = 2 if bf16 else 4
    raw = 3 * I * H * elt
    stride = (raw + 127) // 128 * 128
    buf = np.zeros(E * stride, np.uint8)
    for e in range(E):
        if only is not None and e not in only:
            continue
        parts = []
        for t in (gate[e], up[e], down[e]):
            a = bf16_bits(t) if bf16 else t.contiguous().numpy().astype(np.float32)
            parts.append(a.reshape(-1).view(np.uint8))
        blob = np.concatenate(parts)
        buf[e * stride:e * stride + blob.size] = blob
    return buf


def checksum(*arrays) -> float:
    """float64 sum of all inputs, used to detect generator drift."""
    s = 0.0
    for a in arrays:
        if isinstance(a, torch.Tensor):
            a = a.detach().to(torch.float64).numpy()
        s += float(np.asarray(a, np.float64).sum())
    return s
