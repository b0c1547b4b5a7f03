"""GPU parity tests of the grouped tensor-core path that batched calls of two or
more bf16 tokens take (router -> per-expert token buckets -> tcgen05 grouped
GEMMs -> fixed-order combine), called through the C ABI.

Bar, as for the streaming path: expert indices bit-exact against the oracle's
router for every token; outputs within relative L2 error 1e-3 of the oracle.
At the benchmark shapes the oracle (single-threaded C) checks a sample of
tokens: every token's output depends only on that token, so the sampled rows
of the batch must equal the oracle run on those rows alone.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from warp_route import synthetic
from wr_testlib import abi_layer, host_array, oracle_inputs_from_device

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-3


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _router_ids(x, gate_w, K, bias):
    xa = host_array(x).reshape(-1, x.shape[-1])
    ba = None if bias is None else bias.detach().cpu().numpy().astype(np.float32)
    _, ids, w = oracle.router(np.ascontiguousarray(xa), host_array(gate_w), K, ba)
    return ids, w


def _check_rows(out, x, gate_w, wbuf, E, H, I, K, rows, bias=None, ep_first=0, ep_num=0):
    xs = x[rows].contiguous()
    xa, gwa, host, ba = oracle_inputs_from_device(xs, gate_w, wbuf, E, H, I, K, bias, ep_first,
                                                  ep_num)
    o_out, _, _ = oracle.moe(xa, gwa, host, E, H, I, K, ba, ep_first, ep_num)
    got = out[rows].cpu().numpy()
    err = oracle.rel_l2(got, o_out)
    assert err <= REL_L2_TOL, f"rel L2 {err:.3e} > {REL_L2_TOL}"
    return err


def _run(L, E, H, I, K, **kw):
    out, ids, w = abi_layer(L.x, L.gate_w, L.weight_buf, E, H, I, K, bias=L.router_bias, **kw)
    torch.cuda.synchronize()
    return out, ids, w


def _check_routing(ids, w, L, K):
    o_ids, o_w = _router_ids(L.x, L.gate_w, K, L.router_bias)
    np.testing.assert_array_equal(ids.cpu().numpy(), o_ids)
    np.testing.assert_allclose(w.cpu().numpy(), o_w, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("T", [2, 5, 16, 17, 40, 64, 130])
@pytest.mark.parametrize("bias", [False, True])
def test_small_shape_all_tokens(T, bias):
    E, H, I, K = 8, 1024, 2048, 2
    L = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=21, tokens=T,
                             router_bias=bias)
    out, ids, w = _run(L, E, H, I, K)
    _check_routing(ids, w, L, K)
    _check_rows(out, L.x, L.gate_w, L.weight_buf, E, H, I, K, list(range(T)), L.router_bias)


@pytest.mark.parametrize("T", [16, 64, 256])
def test_mixtral_batched_sweep_shape(T):
    """The batched-decode sweep's shape: Mixtral layer with a per-expert
    router bias N(0,1) skewing the load."""
    E, H, I, K = synthetic.SHAPES["mixtral"]
    L = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=4, tokens=T,
                             router_bias=True)
    out, ids, w = _run(L, E, H, I, K)
    _check_routing(ids, w, L, K)
    g = torch.Generator().manual_seed(T)
    rows = sorted(torch.randperm(T, generator=g)[:4].tolist())
    _check_rows(out, L.x, L.gate_w, L.weight_buf, E, H, I, K, rows, L.router_bias)
    assert torch.isfinite(out).all()


def test_deepseek_shape_batch_256_tokens():
    """64 experts, top_k 6, 1536 pairs: every bucketing warp's span holds
    pairs of many experts (ranks carried across warps)."""
    E, H, I, K = synthetic.SHAPES["deepseek"]
    T = 256
    L = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=62, tokens=T,
                             router_bias=True)
    out, ids, w = _run(L, E, H, I, K)
    _check_routing(ids, w, L, K)
    _check_rows(out, L.x, L.gate_w, L.weight_buf, E, H, I, K, [0, 1, 100, 191, 192, 255],
                L.router_bias)


def test_deepseek_shape_many_idle_experts():
    E, H, I, K = synthetic.SHAPES["deepseek"]
    T = 24  # 144 (token, expert) pairs over 64 experts: many experts get none
    L = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=8, tokens=T)
    out, ids, w = _run(L, E, H, I, K)
    _check_routing(ids, w, L, K)
    _check_rows(out, L.x, L.gate_w, L.weight_buf, E, H, I, K, [0, 7, 23])


def test_hot_expert_spans_several_token_tiles():
    """A bias that sends every token to the same expert: that expert's bucket
    holds 300 rows, three token tiles of the GEMMs."""
    E, H, I, K = 8, 1024, 1024, 2
    T = 300
    L = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=9, tokens=T)
    bias = torch.zeros(E, dtype=torch.float32, device="cuda")
    bias[5] = 50.0
    out, ids, w = abi_layer(L.x, L.gate_w, L.weight_buf, E, H, I, K, bias=bias)
    torch.cuda.synchronize()
    assert (ids[:, 0] == 5).all()
    o_ids, _ = _router_ids(L.x, L.gate_w, K, bias)
    np.testing.assert_array_equal(ids.cpu().numpy(), o_ids)
    _check_rows(out, L.x, L.gate_w, L.weight_buf, E, H, I, K, [0, 128, 129, 299], bias)


@pytest.mark.parametrize("E,H,I,T,rows", [
    # few K chunks: nearly every gate/up tile is cut between CTAs (partial
    # sums parked and added by the tile's last CTA); every token checked
    (4, 1024, 1536, 250, None),
    # more tiles than CTAs: whole tiles run in one CTA
    (8, 1024, 4096, 250, [0, 5, 127, 128, 129, 200, 249]),
    # 129 tokens: the second accumulator holds one token
    (4, 1024, 1536, 129, None),
])
def test_gate_up_tiles_above_128_tokens(E, H, I, T, rows):
    """Batches above 128 tokens: an expert's gate/up tile of up to 256 tokens
    streams its weights once, tokens 128.. from a second token slot into the
    second TMEM accumulator.  A bias sends every token to expert 2 first."""
    K = 2
    L = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=23, tokens=T)
    bias = torch.zeros(E, dtype=torch.float32, device="cuda")
    bias[2] = 50.0
    out, ids, w = abi_layer(L.x, L.gate_w, L.weight_buf, E, H, I, K, bias=bias)
    torch.cuda.synchronize()
    assert (ids[:, 0] == 2).all()
    o_ids, o_w = _router_ids(L.x, L.gate_w, K, bias)
    np.testing.assert_array_equal(ids.cpu().numpy(), o_ids)
    np.testing.assert_allclose(w.cpu().numpy(), o_w, rtol=2e-6, atol=1e-7)
    _check_rows(out, L.x, L.gate_w, L.weight_buf, E, H, I, K,
                list(range(T)) if rows is None else rows, bias)


@pytest.mark.parametrize("E,H,I,K,T", [
    (8, 1000, 1000, 2, 20),    # row tiles and K chunks with tails (TMA zero fill)
    (4, 64, 64, 2, 8),         # one K chunk, one row tile smaller than the MMA
    (64, 256, 128, 8, 40),     # the most experts, top_k 8: many small buckets
    (4, 512, 768, 4, 32),      # top_k == E: every expert takes every token
    (8, 512, 1024, 1, 48),     # top_k == 1
    (3, 256, 512, 2, 16),      # odd expert count, smallest grouped batch
])
def test_edge_shapes(E, H, I, K, T):
    L = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=13, tokens=T)
    out, ids, w = _run(L, E, H, I, K)
    _check_routing(ids, w, L, K)
    _check_rows(out, L.x, L.gate_w, L.weight_buf, E, H, I, K, list(range(T)))


@pytest.mark.parametrize("T,hot", [(64, False), (130, True)])
def test_expert_parallel_shards_sum_to_full(T, hot):
    """Four expert shards sum to the whole layer.  With `hot`, a bias sends
    every token to expert 1 first: shard 0 then holds a tile above 64 tokens
    (both accumulators, cost-weighted down split) beside small ones."""
    E, H, I, K = 8, 1024, 2048, 2
    bias = None
    if hot:
        bias = torch.zeros(E, dtype=torch.float32, device="cuda")
        bias[1] = 50.0
    full = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=17, tokens=T)
    ref, _, _ = abi_layer(full.x, full.gate_w, full.weight_buf, E, H, I, K, bias=bias)
    acc = torch.zeros_like(ref)
    for r in range(4):
        sh = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=17, tokens=T,
                                  ep_rank=r, ep_size=4)
        out, _, _ = abi_layer(sh.x, sh.gate_w, sh.weight_buf, E, H, I, K, bias=bias,
                              ep_first=sh.ep_first, ep_num=sh.ep_num)
        acc += out
    torch.cuda.synchronize()
    assert oracle.rel_l2(acc.cpu().numpy(), ref.cpu().numpy()) <= 1e-5


def test_tensor_parallel_slices_sum_to_full():
    E, H, I, K, T = 8, 1024, 2048, 2, 32
    full = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=19, tokens=T)
    ref, _, _ = _run(full, E, H, I, K)
    acc = torch.zeros_like(ref)
    for r in range(2):
        sh = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=19, tokens=T,
                                  tp_rank=r, tp_size=2)
        out, _, _ = abi_layer(sh.x, sh.gate_w, sh.weight_buf, E, H, sh.I, K)
        acc += out
    torch.cuda.synchronize()
    assert oracle.rel_l2(acc.cpu().numpy(), ref.cpu().numpy()) <= 1e-4


def test_deterministic_and_workspace_reusable():
    E, H, I, K, T = 8, 1024, 2048, 2, 64
    L = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=23, tokens=T,
                             router_bias=True)
    from warp_route import _abi
    import ctypes
    lib = _abi.load()
    d = _abi.desc(E, H, I, K, _abi.WR_DTYPE_BF16, 0, 0, L.router_bias.data_ptr())
    ws = torch.zeros(lib.wr_fused_moe_workspace_size(ctypes.byref(d), T), dtype=torch.uint8,
                     device="cuda")
    a, _, _ = abi_layer(L.x, L.gate_w, L.weight_buf, E, H, I, K, bias=L.router_bias, ws=ws)
    # a smaller batch through the same workspace in between
    small = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=29, tokens=20)
    abi_layer(small.x, small.gate_w, small.weight_buf, E, H, I, K, ws=ws)
    b, _, _ = abi_layer(L.x, L.gate_w, L.weight_buf, E, H, I, K, bias=L.router_bias, ws=ws)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("E,H,I,K,T", [
    (8, 512, 1024, 2, 20),     # the smallest shapes
    (8, 1000, 1000, 2, 37),    # row tiles and K chunks with tails (TMA zero fill)
    (4, 1024, 1536, 4, 64),    # top_k 4: experts with up to 64 tokens, one tile each
    (8, 1024, 2048, 2, 130),   # experts with several 64-token tiles
    (64, 256, 128, 8, 40),     # the most experts, top_k 8: many small buckets
    (8, 512, 1024, 2, 3),      # the smallest fp32 batch on the grouped path
])
def test_fp32_batches_grouped(E, H, I, K, T):
    """fp32 batches (warp-route's dtype) on the tensor cores: weights split
    into bf16 hi + lo in shared memory, tokens and activations likewise."""
    L = synthetic.make_layer(E, H, I, K, dtype=torch.float32, seed=31, tokens=T)
    out, ids, w = _run(L, E, H, I, K)
    _check_routing(ids, w, L, K)
    _check_rows(out, L.x, L.gate_w, L.weight_buf, E, H, I, K, list(range(T)))


def test_fp32_hot_expert_and_expert_shards():
    """fp32: a bias sends every token to expert 1 first (150 tokens: three
    token tiles, nearly every tile cut between CTAs), and four expert shards
    sum to the whole layer."""
    E, H, I, K, T = 8, 1024, 2048, 2, 150
    bias = torch.zeros(E, dtype=torch.float32, device="cuda")
    bias[1] = 50.0
    full = synthetic.make_layer(E, H, I, K, dtype=torch.float32, seed=41, tokens=T)
    ref, ids, _ = abi_layer(full.x, full.gate_w, full.weight_buf, E, H, I, K, bias=bias)
    torch.cuda.synchronize()
    assert (ids[:, 0] == 1).all()
    _check_rows(ref, full.x, full.gate_w, full.weight_buf, E, H, I, K, [0, 63, 64, 127, 149],
                bias)
    acc = torch.zeros_like(ref)
    for r in range(4):
        sh = synthetic.make_layer(E, H, I, K, dtype=torch.float32, seed=41, tokens=T,
                                  ep_rank=r, ep_size=4)
        out, _, _ = abi_layer(sh.x, sh.gate_w, sh.weight_buf, E, H, I, K, bias=bias,
                              ep_first=sh.ep_first, ep_num=sh.ep_num)
        acc += out
    torch.cuda.synchronize()
    assert oracle.rel_l2(acc.cpu().numpy(), ref.cpu().numpy()) <= 1e-5


def test_fp32_mixtral_shape_batch():
    """The Mixtral shape in fp32 at T = 16 with the sweep's router bias."""
    E, H, I, K = synthetic.SHAPES["mixtral"]
    T = 16
    L = synthetic.make_layer(E, H, I, K, dtype=torch.float32, seed=43, tokens=T,
                             router_bias=True)
    out, ids, w = _run(L, E, H, I, K)
    _check_routing(ids, w, L, K)
    _check_rows(out, L.x, L.gate_w, L.weight_buf, E, H, I, K, [0, 7, 15], L.router_bias)


def test_python_api_matches_c_abi():
    from warp_route import functional as F
    E, H, I, K, T = 8, 1024, 2048, 2, 48
    L = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=37, tokens=T)
    a, _, _ = _run(L, E, H, I, K)
    b = F.batched_fused_moe(L.x, L.gate_w, L.weight_buf, E, H, I, K)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_many_pairs_bucket_reads_global(dtype):
    """More (token, expert) pairs than the bucket kernel stages in shared
    memory (T * K > 5632): its passes read the routing from global memory;
    experts get hundreds of tokens (many token tiles each)."""
    E, H, I, K, T = 16, 256, 256, 8, 720  # 5760 pairs
    L = synthetic.make_layer(E, H, I, K, dtype=dtype, seed=61, tokens=T,
                             router_bias=True)
    out, ids, w = _run(L, E, H, I, K)
    _check_routing(ids, w, L, K)
    _check_rows(out, L.x, L.gate_w, L.weight_buf, E, H, I, K, [0, 1, 357, 719], L.router_bias)


@pytest.mark.parametrize("T", [6, 100])
def test_one_rank_allreduce_combine_matches_plain_combine(T):
    """The all-reducing combine step (one launch per 64 tokens), given a
    one-rank communicator, sums a single partial output and must equal the
    plain combine.  At T = 100 every token picks the same first expert, so
    its 100 rows form a tile above 64 tokens (both accumulators, the
    cost-weighted down split) and the step runs as two launches."""
    from warp_route import functional as F
    E, H, I, K = 8, 1024, 2048, 2
    L = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=67, tokens=T)
    bias = torch.zeros(E, dtype=torch.float32, device="cuda")
    bias[3] = 50.0
    ref = F.fused_moe_routed(L.x, L.gate_w, L.weight_buf, E, H, I, K, router_bias=bias)[0]
    _C = F._load_extension()
    comm = _C.comm_create(0, 1, H)
    try:
        for _ in range(2):  # the second call runs under the next epoch
            got = _C.fused_moe_allreduce(L.x, L.gate_w, L.weight_buf, E, H, I, K, comm, bias,
                                         0, 0)[0]
            torch.cuda.synchronize()
            assert oracle.rel_l2(got.cpu().numpy(), ref.cpu().numpy()) <= 1e-6
    finally:
        _C.comm_destroy(comm)
    _check_rows(ref, L.x, L.gate_w, L.weight_buf, E, H, I, K, [0, T - 1], bias)


def test_expert_shard_without_pairs_writes_zeros():
    """An expert-parallel shard that no token picks (a bias makes experts 0
    and 1 everyone's choice; this rank holds experts 6-7): no tiles at all,
    and the output is exactly zero."""
    E, H, I, K, T = 8, 1024, 2048, 2, 6
    bias = torch.zeros(E, dtype=torch.float32, device="cuda")
    bias[0] = bias[1] = 50.0
    sh = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=71, tokens=T,
                              ep_rank=3, ep_size=4)
    for _ in range(2):
        out, ids, _ = abi_layer(sh.x, sh.gate_w, sh.weight_buf, E, H, I, K, bias=bias,
                                ep_first=sh.ep_first, ep_num=sh.ep_num)
        torch.cuda.synchronize()
        assert set(ids.view(-1).tolist()) == {0, 1}
        assert torch.equal(out, torch.zeros_like(out))
