"""GPU tests of the decode-step driver (warp_route.decode.MoEStack): the
graph replay equals the same stack run eagerly bit for bit, every step, for a
single token (streaming kernel) and a batch (grouped tcgen05 path); and the
chained stack follows the CPU oracle applied layer by layer."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from warp_route import synthetic
from warp_route.decode import MoEStack, StackLayer
from wr_testlib import host_array

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _stack(E, H, I, K, T, n_layers, seed=50):
    layers = []
    for li in range(n_layers):
        L = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=seed + li, layer=li,
                                 router_bias=True)
        layers.append(StackLayer(L.gate_w, L.weight_buf, L.router_bias))
    return MoEStack(layers, E, H, I, K, T)


@pytest.mark.parametrize("T", [1, 16])
def test_graph_replay_equals_eager(T):
    E, H, I, K = 8, 512, 1024, 2
    stack = _stack(E, H, I, K, T, 4)
    g = torch.Generator(device="cuda")
    g.manual_seed(T)
    shape = (H,) if T == 1 else (T, H)
    for step in range(3):
        x = torch.randn(shape, generator=g, device="cuda").to(torch.bfloat16)
        ref = stack.eager(x)
        got = stack.step(x).clone()
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"step {step}: graph replay differs from the eager stack"
        assert torch.isfinite(got.float()).all()
    stack.close()


def test_chain_follows_the_oracle():
    E, H, I, K, T = 8, 512, 1024, 2, 16
    n_layers = 3
    stack = _stack(E, H, I, K, T, n_layers, seed=70)
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
    got = stack.step(x).clone()
    torch.cuda.synchronize()
    # oracle: h <- bf16(h + moe(h)) per layer, on the host
    h = x.cpu()
    for L in stack.layers:
        wb = L.weight_buf.cpu().view(torch.uint8).numpy()
        out, _, _ = oracle.moe(host_array(h), host_array(L.gate_w), wb, E, H, I, K,
                               L.router_bias.cpu().numpy())
        h = (h.float() + torch.from_numpy(np.asarray(out))).to(torch.bfloat16)
    err = oracle.rel_l2(got.float().cpu().numpy(), h.float().numpy())
    assert err <= 1e-2, err
    stack.close()
