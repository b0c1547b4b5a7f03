"""wr_fused_moe_noalloc: the single-token layer for callers that cannot
allocate device memory, using the library's built-in 1 MiB scratch.

Its results must match wr_fused_moe's (same kernels, caller workspace) on
consecutive calls, since every call reuses the same scratch.  The file name
makes pytest collect it last, so the GPU test also runs after everything else
the suite has launched; it passes alone in a fresh process too.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from warp_route import _abi, synthetic
from wr_testlib import dtype_code, ptr, stream_ptr

REL_L2_TOL = 1e-3  # the output tolerance the parity tests use
SCRATCH_BYTES = 1 << 20


def _desc(E, H, I, K, dtype_code_):
    return _abi.desc(E, H, I, K, dtype_code_)


def _run_regular(lib, d, x, gate_w, wbuf, K):
    H = x.shape[0]
    out = torch.full((H,), float("nan"), dtype=torch.float32, device=x.device)
    ids = torch.full((K,), -1, dtype=torch.int32, device=x.device)
    w = torch.full((K,), float("nan"), dtype=torch.float32, device=x.device)
    need = lib.wr_fused_moe_workspace_size(ctypes.byref(d), 1)
    ws = torch.zeros(need, dtype=torch.uint8, device=x.device)
    wbytes = wbuf.numel() * wbuf.element_size()
    _abi.check(lib.wr_fused_moe(ctypes.byref(d), ptr(x), ptr(gate_w), ptr(wbuf), wbytes,
                                ptr(out), ptr(ids), ptr(w), ptr(ws), ws.numel(), stream_ptr()))
    _abi.check(lib.wr_workspace_status(ptr(ws), stream_ptr()))
    return out, ids, w


def _run_noalloc(lib, d, x, gate_w, wbuf, K):
    H = x.shape[0]
    out = torch.full((H,), float("nan"), dtype=torch.float32, device=x.device)
    ids = torch.full((K,), -1, dtype=torch.int32, device=x.device)
    w = torch.full((K,), float("nan"), dtype=torch.float32, device=x.device)
    wbytes = wbuf.numel() * wbuf.element_size()
    _abi.check(lib.wr_fused_moe_noalloc(ctypes.byref(d), ptr(x), ptr(gate_w), ptr(wbuf), wbytes,
                                        ptr(out), ptr(ids), ptr(w), stream_ptr()))
    # no bounded wait inside the call gave up
    _abi.check(lib.wr_fused_moe_noalloc_status(stream_ptr()))
    return out, ids, w


def _rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a64, b64 = a.double(), b.double()
    den = torch.linalg.vector_norm(b64).item()
    return torch.linalg.vector_norm(a64 - b64).item() / (den if den > 0 else 1.0)


@pytest.mark.gpu
@pytest.mark.parametrize("E,H,I,K,dtype", [
    (8, 512, 1024, 2, torch.float32),        # tiny
    (8, 514, 1000, 2, torch.float32),        # unaligned: the multi-kernel path
    (64, 2048, 1408, 6, torch.bfloat16),     # deepseek shape
    (8, 4096, 14336, 2, torch.bfloat16),     # mixtral shape
])
def test_noalloc_matches_fused_on_consecutive_calls(E, H, I, K, dtype):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    lib = _abi.load()
    L = synthetic.make_layer(E, H, I, K, dtype=dtype, seed=11)
    d = _desc(E, H, I, K, dtype_code(L.x))
    assert lib.wr_fused_moe_workspace_size(ctypes.byref(d), 1) <= SCRATCH_BYTES
    g = torch.Generator(device="cuda")
    g.manual_seed(1234)
    xs = [L.x, torch.randn(H, generator=g, device="cuda", dtype=torch.float32).to(dtype)]
    # two calls in a row on the shared scratch, each checked against the
    # regular entry point on the same token
    results = [_run_noalloc(lib, d, x, L.gate_w, L.weight_buf, K) for x in xs]
    torch.cuda.synchronize()
    for x, (out, ids, w) in zip(xs, results):
        r_out, r_ids, r_w = _run_regular(lib, d, x, L.gate_w, L.weight_buf, K)
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        np.testing.assert_array_equal(ids.cpu().numpy(), r_ids.cpu().numpy())
        np.testing.assert_allclose(w.cpu().numpy(), r_w.cpu().numpy(), rtol=2e-6, atol=1e-7)
        err = _rel_l2(out, r_out)
        assert err <= REL_L2_TOL, f"rel L2 {err:.3e} > {REL_L2_TOL}"
    # the two tokens differ, so the second call did not reuse the first's result
    assert not torch.equal(results[0][0], results[1][0])


def test_noalloc_rejects_layers_beyond_the_scratch():
    """A layer whose workspace exceeds the built-in scratch is refused before
    anything touches the GPU (the pointers here are host dummies)."""
    lib = _abi.load()
    E, H, I, K = 8, 256, 40000, 8
    d = _desc(E, H, I, K, _abi.WR_DTYPE_F32)
    assert lib.wr_fused_moe_workspace_size(ctypes.byref(d), 1) > SCRATCH_BYTES
    dummy = (ctypes.c_float * 16)()
    p = ctypes.cast(dummy, ctypes.c_void_p)
    wbytes = lib.wr_total_weight_bytes(E, H, I, 4)
    st = lib.wr_fused_moe_noalloc(ctypes.byref(d), p, p, p, wbytes, p, None, None, None)
    assert st == _abi.WR_ERR_UNSUPPORTED
    msg = lib.wr_last_error_string().decode()
    assert "scratch" in msg and str(SCRATCH_BYTES) in msg


def test_noalloc_reports_bad_arguments_like_fused():
    lib = _abi.load()
    dummy = (ctypes.c_float * 16)()
    p = ctypes.cast(dummy, ctypes.c_void_p)
    bad = _desc(8, 512, 1024, 0, _abi.WR_DTYPE_F32)  # top_k 0
    assert lib.wr_fused_moe_noalloc(ctypes.byref(bad), p, p, p, 1 << 30, p, None, None,
                                    None) == _abi.WR_ERR_INVALID
    assert "top_k" in lib.wr_last_error_string().decode()
    d = _desc(8, 512, 1024, 2, _abi.WR_DTYPE_F32)
    assert lib.wr_fused_moe_noalloc(ctypes.byref(d), p, p, p, 16, p, None, None,
                                    None) == _abi.WR_ERR_TOO_SMALL
    assert lib.wr_fused_moe_noalloc(ctypes.byref(d), None, p, p, 1 << 30, p, None, None,
                                    None) == _abi.WR_ERR_INVALID
