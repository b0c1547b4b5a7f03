"""GPU parity tests: the CUDA path, called through the C ABI, against the CPU
oracle (which is itself pinned to warp-route's own composition by
test_oracle_golden.py).

Bar: expert indices bit-exact; outputs within relative L2 error 1e-3 of the
oracle (the fp32-accumulating kernels land near 1e-6); router logits
bit-exact.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import inputs as gi
import oracle
from conftest import golden_inputs, golden_selected, load_golden
from warp_route import _abi, synthetic
from wr_testlib import abi_layer, host_array, oracle_inputs_from_device, ptr, stream_ptr

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-3  # the stated output tolerance (fp32 accumulation, fp32 output)
_, INDEX = load_golden()


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _check(out, ids, w, x, gate_w, wbuf, E, H, I, K, bias=None, ep_first=0, ep_num=0,
           golden_ids=None):
    xa, gwa, host, ba = oracle_inputs_from_device(x, gate_w, wbuf, E, H, I, K, bias, ep_first,
                                                  ep_num)
    o_out, o_ids, o_w = oracle.moe(xa, gwa, host, E, H, I, K, ba, ep_first, ep_num)
    if ids is not None:
        np.testing.assert_array_equal(ids.cpu().numpy(), o_ids)
        np.testing.assert_allclose(w.cpu().numpy(), o_w, rtol=2e-6, atol=1e-7)
    if golden_ids is not None:
        np.testing.assert_array_equal(o_ids, golden_ids)
    err = oracle.rel_l2(out.cpu().numpy().reshape(o_out.shape), o_out)
    assert err <= REL_L2_TOL, f"rel L2 {err:.3e} > {REL_L2_TOL}"
    return err


@pytest.mark.parametrize("meta", INDEX, ids=[m["name"] for m in INDEX])
def test_golden_cases_through_c_abi(golden, meta):
    z, _ = golden
    x, gw, ex = golden_inputs(meta)
    dt = torch.bfloat16 if meta["bf16"] else torch.float32
    E, H, I, K = meta["E"], meta["H"], meta["I"], meta["top_k"]
    xd = x.to(dt).cuda()
    gwd = gw.to(dt).cuda().contiguous()
    # the experts the reference selected are packed (the others stay zero: a
    # wrong selection reads zeros and fails the output check as well)
    wb = torch.from_numpy(gi.pack_numpy(ex, bf16=meta["bf16"],
                                        only=golden_selected(z, meta))).cuda().view(dt)
    xin = xd if meta["kind"] == "batched" else xd[0].contiguous()
    out, ids, w = abi_layer(xin, gwd, wb, E, H, I, K)
    torch.cuda.synchronize()
    # directly against the reference composition's own selection and output
    golden_ids = z[meta["name"] + "/ids"]
    np.testing.assert_array_equal(ids.cpu().numpy().reshape(golden_ids.shape), golden_ids)
    np.testing.assert_allclose(w.cpu().numpy().reshape(golden_ids.shape),
                               z[meta["name"] + "/weights"], rtol=1e-5, atol=1e-7)
    ref = z[meta["name"] + "/out"]
    assert oracle.rel_l2(out.cpu().numpy().reshape(ref.shape), ref) <= REL_L2_TOL
    # and against the oracle
    _check(out, ids, w, xin, gwd, wb, E, H, I, K, golden_ids=golden_ids)


@pytest.mark.parametrize("shape,dtype", [("tiny", torch.float32), ("mixtral", torch.bfloat16),
                                         ("deepseek", torch.bfloat16), ("dbrx", torch.bfloat16),
                                         ("mixtral", torch.float32)])
def test_benchmark_shapes_full_size(shape, dtype):
    E, H, I, K = synthetic.SHAPES[shape]
    L = synthetic.make_layer(E, H, I, K, dtype=dtype, seed=0)
    out, ids, w = abi_layer(L.x, L.gate_w, L.weight_buf, E, H, I, K)
    torch.cuda.synchronize()
    _check(out, ids, w, L.x, L.gate_w, L.weight_buf, E, H, I, K)


@pytest.mark.parametrize("T", [2, 3, 4, 5, 8, 13])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_token_batches(T, dtype):
    E, H, I, K = 8, 1024, 2048, 2
    L = synthetic.make_layer(E, H, I, K, dtype=dtype, seed=11, tokens=T)
    out, ids, w = abi_layer(L.x, L.gate_w, L.weight_buf, E, H, I, K)
    torch.cuda.synchronize()
    _check(out, ids, w, L.x, L.gate_w, L.weight_buf, E, H, I, K)


@pytest.mark.parametrize("E,H,I,K,dtype", [
    (8, 512, 1024, 8, torch.bfloat16),     # top_k == E
    (8, 512, 1024, 1, torch.float32),      # top_k == 1
    (3, 256, 512, 2, torch.float32),       # odd expert count
    (64, 256, 256, 6, torch.bfloat16),     # many small experts
    (5, 100, 52, 2, torch.float32),        # ragged shapes -> unaligned path
    (6, 200, 36, 3, torch.bfloat16),       # ragged bf16 (H % 8 != 0)
    (8, 21248, 256, 2, torch.bfloat16),    # largest H the streaming kernel keeps in smem
    (8, 21256, 256, 2, torch.bfloat16),    # one vector more: the naive path takes it
    (8, 8200, 512, 2, torch.bfloat16),     # gate/up rows split across stages
])
def test_edge_shapes(E, H, I, K, dtype):
    L = synthetic.make_layer(E, H, I, K, dtype=dtype, seed=5)
    out, ids, w = abi_layer(L.x, L.gate_w, L.weight_buf, E, H, I, K)
    torch.cuda.synchronize()
    _check(out, ids, w, L.x, L.gate_w, L.weight_buf, E, H, I, K)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_ties_go_to_lowest_index(dtype):
    E, H, I, K = 8, 512, 512, 3
    L = synthetic.make_layer(E, H, I, K, dtype=dtype, seed=3)
    gw = L.gate_w.clone()
    # experts 2, 5 and 6 get identical router rows: identical logits
    gw[5] = gw[2]
    gw[6] = gw[2]
    # make their logit the largest by aligning the row with x
    gw[2] = (L.x.float() * 0.05).to(dtype)
    gw[5] = gw[2]
    gw[6] = gw[2]
    out, ids, w = abi_layer(L.x, gw, L.weight_buf, E, H, I, K)
    torch.cuda.synchronize()
    assert ids.cpu().numpy().ravel().tolist() == [2, 5, 6]
    _check(out, ids, w, L.x, gw, L.weight_buf, E, H, I, K)


def test_router_bias():
    E, H, I, K = 16, 1024, 512, 4
    L = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=9, tokens=3, router_bias=True)
    out, ids, w = abi_layer(L.x, L.gate_w, L.weight_buf, E, H, I, K, bias=L.router_bias)
    torch.cuda.synchronize()
    _check(out, ids, w, L.x, L.gate_w, L.weight_buf, E, H, I, K, bias=L.router_bias)


def test_expert_parallel_shards_sum_to_full():
    E, H, I, K, N = 8, 1024, 1024, 2, 4
    full = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=21)
    ref, ids, _ = abi_layer(full.x, full.gate_w, full.weight_buf, E, H, I, K)
    acc = torch.zeros_like(ref)
    for r in range(N):
        sh = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=21, ep_rank=r, ep_size=N,
                                  x=full.x, gate_w=full.gate_w)
        part, pids, _ = abi_layer(sh.x, sh.gate_w, sh.weight_buf, E, H, I, K,
                                  ep_first=sh.ep_first, ep_num=sh.ep_num)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(pids.cpu().numpy(), ids.cpu().numpy())
        _check(part, None, None, sh.x, sh.gate_w, sh.weight_buf, E, H, I, K,
               ep_first=sh.ep_first, ep_num=sh.ep_num)
        acc += part
    assert oracle.rel_l2(acc.cpu().numpy(), ref.cpu().numpy()) < 1e-5


def test_tensor_parallel_slices_sum_to_full():
    E, H, I, K, N = 8, 2048, 4096, 2, 4
    full = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=22)
    ref, ids, _ = abi_layer(full.x, full.gate_w, full.weight_buf, E, H, I, K)
    acc = torch.zeros_like(ref)
    for r in range(N):
        sh = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=22, tp_rank=r, tp_size=N,
                                  x=full.x, gate_w=full.gate_w)
        part, pids, _ = abi_layer(sh.x, sh.gate_w, sh.weight_buf, E, H, I // N, K)
        np.testing.assert_array_equal(pids.cpu().numpy(), ids.cpu().numpy())
        acc += part
    torch.cuda.synchronize()
    assert oracle.rel_l2(acc.cpu().numpy(), ref.cpu().numpy()) < 1e-5


def test_deterministic_and_workspace_reusable():
    E, H, I, K = 8, 4096, 14336, 2
    L = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=1)
    lib = _abi.load()
    d = _abi.desc(E, H, I, K, _abi.WR_DTYPE_BF16)
    ws = torch.zeros(lib.wr_fused_moe_workspace_size(ctypes.byref(d), 1), dtype=torch.uint8,
                     device="cuda")
    outs = [abi_layer(L.x, L.gate_w, L.weight_buf, E, H, I, K, ws=ws)[0] for _ in range(3)]
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    # the grid-barrier words reset themselves after every call
    words = ws[:12].view(torch.int32).cpu().tolist()
    assert words == [0, 0, 0]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_naive_entry_point(dtype):
    E, H, I, K = 8, 512, 1024, 2
    L = synthetic.make_layer(E, H, I, K, dtype=dtype, seed=4)
    out, _, _ = abi_layer(L.x, L.gate_w, L.weight_buf, E, H, I, K, naive=True)
    torch.cuda.synchronize()
    _check(out, None, None, L.x, L.gate_w, L.weight_buf, E, H, I, K)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("H", [4096, 2048, 100])
def test_router_logits_bit_exact(dtype, H):
    E, K, T = 64, 6, 32
    g = torch.Generator(device="cuda").manual_seed(H)
    x = torch.randn(T, H, generator=g, device="cuda").to(dtype)
    gw = (torch.randn(E, H, generator=g, device="cuda") * 0.02).to(dtype)
    lib = _abi.load()
    d = _abi.desc(E, H, 1, K, 1 if dtype == torch.bfloat16 else 0)
    logits = torch.empty(T, E, dtype=torch.float32, device="cuda")
    ids = torch.empty(T, K, dtype=torch.int32, device="cuda")
    w = torch.empty(T, K, dtype=torch.float32, device="cuda")
    _abi.check(lib.wr_router_topk(ctypes.byref(d), T, ptr(x), ptr(gw), ptr(logits), ptr(ids),
                                  ptr(w), stream_ptr()))
    torch.cuda.synchronize()
    o_logits, o_ids, o_w = oracle.router(host_array(x), host_array(gw), K)
    np.testing.assert_array_equal(logits.cpu().numpy(), o_logits)  # bit for bit
    np.testing.assert_array_equal(ids.cpu().numpy(), o_ids)
    np.testing.assert_allclose(w.cpu().numpy(), o_w, rtol=2e-6, atol=1e-7)


def test_empty_batch_is_a_no_op():
    E, H, I, K = 8, 256, 512, 2
    L = synthetic.make_layer(E, H, I, K, dtype=torch.float32, seed=2, tokens=2)
    lib = _abi.load()
    d = _abi.desc(E, H, I, K, 0)
    st = lib.wr_batched_fused_moe(ctypes.byref(d), 0, ptr(L.x), ptr(L.gate_w), ptr(L.weight_buf),
                                  L.weight_buf.numel() * 4, None, None, None, None, 0, stream_ptr())
    assert st == _abi.WR_OK


@pytest.mark.parametrize("mode", ["tp", "ep"])
def test_one_rank_allreduce_tail_matches_plain_layer(mode):
    """The all-reduce fused into the streaming kernel's tail, given a one-rank
    communicator: every CTA stores its rows as tagged words into the mailbox
    and polls them back, so the output must equal the plain single-token
    layer's (the sum of one source adds 0).  Shards as the 8-GPU runs hold
    them: a tensor-parallel slice of the Mixtral shape (I / 8) and an
    expert-parallel set of the DeepSeek shape (8 of 64 experts).  Three calls
    in a row cover both mailbox parities and the epoch advancing."""
    from warp_route import functional as F
    if mode == "tp":
        E, H, I, K = synthetic.SHAPES["mixtral"]
        sh = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=83, tp_rank=3,
                                  tp_size=8)
    else:
        E, H, I, K = synthetic.SHAPES["deepseek"]
        sh = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=83, ep_rank=2,
                                  ep_size=8)
    _C = F._load_extension()
    comm = _C.comm_create(0, 1, H)
    try:
        gen = torch.Generator(device="cuda")
        gen.manual_seed(5)
        for _ in range(3):
            x = torch.randn(H, generator=gen, device="cuda").to(torch.bfloat16)
            ref, ref_ids, _ = F.fused_moe_routed(x, sh.gate_w, sh.weight_buf, E, H, sh.I, K,
                                                 ep_first_expert=sh.ep_first,
                                                 ep_num_local=sh.ep_num)
            got, ids, _ = _C.fused_moe_allreduce(x, sh.gate_w, sh.weight_buf, E, H, sh.I, K,
                                                 comm, None, sh.ep_first, sh.ep_num)
            torch.cuda.synchronize()
            assert torch.equal(ids, ref_ids)
            assert torch.equal(got, ref), "one-rank all-reduce changed the output"
        assert F._load_extension().workspace_status(x) == 0
    finally:
        _C.comm_destroy(comm)
    # and the shard itself against the oracle
    _check(got, None, None, x, sh.gate_w, sh.weight_buf, E, H, sh.I, K, ep_first=sh.ep_first,
           ep_num=sh.ep_num)
