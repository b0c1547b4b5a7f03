"""CPU: the Python boundary (warp_route.functional / warp_route._C) — imports,
argument errors with warp-route's messages, and the packed layout."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import inputs as gi
import oracle
import warp_route
from warp_route import functional as F


def test_extension_loads_without_gpu():
    _C = F._load_extension()
    for name in ("fused_moe_forward", "naive_moe_forward", "batched_fused_moe_forward",
                 "fused_moe_routed", "router_topk"):
        assert hasattr(_C, name)
    assert "sm_100a" in _C.version()


def test_public_names():
    for name in ("MoELayer", "fused_moe", "naive_moe", "batched_fused_moe", "fused_moe_batched",
                 "_pack_expert_weights"):
        assert hasattr(warp_route, name)
    assert F.fused_moe_batched is F.batched_fused_moe


def test_cpu_tensor_rejected_like_warp_route():
    x = torch.zeros(64)
    gw = torch.zeros(8, 64)
    wb = torch.zeros(10)
    with pytest.raises(RuntimeError, match="hidden must be a CUDA tensor"):
        F.fused_moe(x, gw, wb, 8, 64, 128, 2)
    with pytest.raises(RuntimeError, match="hidden must be a CUDA tensor"):
        F.naive_moe(x, gw, wb, 8, 64, 128, 2)


def test_batched_shape_errors_are_value_errors():
    # warp_route/functional.py:143-147 of warp-route
    with pytest.raises(ValueError, match="expects 2D input"):
        F.batched_fused_moe(torch.zeros(64), torch.zeros(8, 64), torch.zeros(1), 8, 64, 128, 2)
    with pytest.raises(ValueError, match="does not match hidden_dim"):
        F.batched_fused_moe(torch.zeros(2, 32), torch.zeros(8, 64), torch.zeros(1), 8, 64, 128, 2)


def test_moelayer_validates_top_k():
    with pytest.raises(ValueError):
        warp_route.MoELayer(4, 32, 64, top_k=5)
    layer = warp_route.MoELayer(4, 32, 64, top_k=4)  # top_k up to E is allowed now
    assert len(layer.gate_proj) == 4


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_pack_matches_oracle_layout(dtype):
    E, H, I = 3, 24, 40
    g = torch.Generator().manual_seed(0)
    gate = [torch.randn(I, H, generator=g).to(dtype) for _ in range(E)]
    up = [torch.randn(I, H, generator=g).to(dtype) for _ in range(E)]
    down = [torch.randn(H, I, generator=g).to(dtype) for _ in range(E)]
    buf = F._pack_expert_weights(gate, up, down, E, H, I)
    assert buf.dtype == dtype
    raw = buf.view(torch.uint8).numpy() if dtype == torch.float32 else \
        buf.view(torch.int16).numpy().view(np.uint8)
    to_np = (lambda t: t.numpy()) if dtype == torch.float32 else gi.bf16_bits
    ref = oracle.pack(np.stack([to_np(t) for t in gate]), np.stack([to_np(t) for t in up]),
                      np.stack([to_np(t) for t in down]))
    np.testing.assert_array_equal(raw, ref)


def test_moelayer_parameters_are_the_packed_buffer():
    """The expert parameters are views of the packed buffer: in-place writes
    (including through .data, the usual checkpoint-loading idiom, and
    load_state_dict) show up in it without a repack."""
    E, H, I = 2, 16, 32
    layer = warp_route.MoELayer(E, H, I, top_k=1)
    a = layer._pack_weights()
    assert layer._pack_weights() is a
    n = H * I
    stride = F._expert_stride_elems(H, I, 4)
    with torch.no_grad():
        layer.up_proj[1].add_(1.0)
    assert layer._pack_weights() is a
    assert torch.equal(a[stride + n:stride + 2 * n], layer.up_proj[1].detach().reshape(-1))
    w = torch.randn(I, H)
    layer.gate_proj[0].data.copy_(w)
    assert layer._pack_weights() is a and torch.equal(a[:n].view(I, H), w)
    sd = {k: v.clone() for k, v in layer.state_dict().items()}
    sd["down_proj.1"] = torch.full((H, I), 3.0)
    layer.load_state_dict(sd)
    assert layer._pack_weights() is a
    assert torch.equal(a[stride + 2 * n:stride + 3 * n], torch.full((H * I,), 3.0))
    # the stride padding stays zero
    assert stride == 3 * n  # 16 x 32 floats: already 128-byte aligned here


def test_moelayer_repacks_when_parameters_move():
    """A parameter that is no longer a view of the buffer (assigned a new
    tensor, or converted by module.to) makes the next pack rebuild the buffer
    from the parameters and re-point them at it."""
    E, H, I = 2, 16, 41  # expert blocks not a multiple of 128 bytes: padded strides
    layer = warp_route.MoELayer(E, H, I, top_k=2)
    a = layer._pack_weights()
    w = torch.randn(H, I)
    layer.down_proj[0].data = w.clone()
    b = layer._pack_weights()
    assert b is not a
    stride = F._expert_stride_elems(H, I, 4)
    n = H * I
    assert torch.equal(b[2 * n:3 * n].view(H, I), w)
    assert layer.down_proj[0].data_ptr() == b[2 * n:].data_ptr()
    assert layer._pack_weights() is b
    layer.to(torch.bfloat16)
    c = layer._pack_weights()
    assert c.dtype == torch.bfloat16 and c is not b
    assert torch.equal(c[2 * n:3 * n].view(H, I), w.to(torch.bfloat16))
    assert all(p.dtype == torch.bfloat16 for p in layer.parameters())
    # bf16 stride rounding: the padding between experts is zero
    sb = F._expert_stride_elems(H, I, 2)
    assert sb > 3 * n and torch.count_nonzero(c[3 * n:sb]) == 0
