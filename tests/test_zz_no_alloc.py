"""spock_chunk_prefill_noalloc: the chunk prefill for callers that cannot
allocate device memory at call time (a host framework's pool allocator or a
hard memory budget they do not own, code that must not trigger the device
synchronisation that cudaMalloc/cudaFree can cause, plugins that get only the
caller's buffers and no context). Its staging lives in a fixed array inside
the library, so its results must equal the context-based entry point's.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test."""
import ctypes

import numpy as np
import pytest
import torch

import spock_b200
from tests.golden.gen import chunk_inputs
from tests.util import max_rel

pytestmark = pytest.mark.gpu
TOL = 1e-3  # the parity bar of the chunk-prefill tests


def _call_noalloc(q, k, v, g, b, out, st, use_l2=False):
    B, H, S, K = q.shape
    d = spock_b200.ChunkDesc(B, H, S, K, v.shape[-1], 64, spock_b200._dtype_code(q.dtype),
                             spock_b200._dtype_code(out.dtype), int(use_l2), 0)
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = spock_b200.lib().spock_chunk_prefill_noalloc(ctypes.byref(d), p(q), p(k), p(v), p(g), p(b), None,
                                                      p(out), p(st), stream)
    return rc


def test_noalloc_matches_context_entry_point_twice(cuda_ok):
    dev = torch.device("cuda", 0)
    for call, (S, seed) in enumerate([(300, 21), (130, 22)]):  # two calls in a row, different sizes
        q, k, v, g, b = (torch.from_numpy(x).to(dev) for x in chunk_inputs(4, S, seed=seed, batch=2))
        out = torch.full((2, 4, S, 128), float("nan"), device=dev)
        st = torch.full((2, 4, 128, 128), float("nan"), device=dev)
        rc = _call_noalloc(q, k, v, g, b, out, st)
        assert rc == spock_b200.SPOCK_OK, spock_b200.lib().spock_last_error(None)
        ref_out, ref_st = spock_b200.chunk_prefill(q, k, v, g, b)  # fp32 inputs: staged in ctx scratch
        torch.cuda.synchronize()
        assert max_rel(out.cpu().numpy(), ref_out.cpu().numpy()) <= TOL, call
        assert max_rel(st.cpu().numpy(), ref_st.cpu().numpy()) <= TOL, call


def test_noalloc_l2norm_staging(cuda_ok):
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(5)
    q, k, v = (torch.from_numpy(rng.standard_normal((1, 2, 100, 128), dtype=np.float32)).to(dev).half()
               for _ in range(3))
    g = torch.from_numpy(rng.uniform(-1, -0.01, (1, 2, 100)).astype(np.float32)).to(dev)
    b = torch.from_numpy(rng.uniform(0, 1, (1, 2, 100)).astype(np.float32)).to(dev)
    out = torch.empty((1, 2, 100, 128), device=dev)
    st = torch.empty((1, 2, 128, 128), device=dev)
    assert _call_noalloc(q, k, v, g, b, out, st, use_l2=True) == spock_b200.SPOCK_OK
    ref_out, ref_st = spock_b200.chunk_prefill(q, k, v, g, b, out_dtype=torch.float32, use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert max_rel(out.cpu().numpy(), ref_out.cpu().numpy()) <= TOL
    assert max_rel(st.cpu().numpy(), ref_st.cpu().numpy()) <= TOL


def test_noalloc_rejects_sizes_beyond_its_fixed_scratch(cuda_ok):
    dev = torch.device("cuda", 0)
    x = torch.zeros((1, 16, 1025, 128), device=dev)  # 16400 token-heads > 16384
    s = torch.zeros((1, 16, 1025), device=dev)
    out = torch.empty_like(x)
    st = torch.empty((1, 16, 128, 128), device=dev)
    rc = _call_noalloc(x, x, x, s, s, out, st)
    assert rc == spock_b200.SPOCK_ERR_INVALID
    assert b"exceeds the fixed scratch" in spock_b200.lib().spock_last_error(None)
