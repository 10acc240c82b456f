"""spock_chunk_prefill_noalloc: the chunk prefill for callers that cannot
allocate device memory at call time (a host framework's pool allocator or a
hard memory budget they do not own, code that must not trigger the device
synchronisation that cudaMalloc/cudaFree can cause, plugins that get only the
caller's buffers and no context). Its staging lives in a fixed array inside
the library, so its results must equal the context-based entry point's and
meet the same oracle bar, and a bounded wait that gives up must reach the
caller through spock_noalloc_sync.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
import spock_b200
from tests.golden.gen import chunk_inputs
from tests.util import max_rel

pytestmark = pytest.mark.gpu
TOL = 1e-3  # the parity bar of the chunk-prefill tests
DEV = torch.device("cuda", 0)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _call_noalloc(q, k, v, g, b, out, st, use_l2=False):
    B, H, S, K = q.shape
    d = spock_b200.ChunkDesc(B, H, S, K, v.shape[-1], 64, spock_b200._dtype_code(q.dtype),
                             spock_b200._dtype_code(out.dtype), int(use_l2), 0)
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    return spock_b200.lib().spock_chunk_prefill_noalloc(ctypes.byref(d), p(q), p(k), p(v), p(g), p(b), None,
                                                        p(out), p(st), _stream())


def _noalloc_sync():
    return spock_b200.lib().spock_noalloc_sync(_stream())


def _oracle(q, k, v, g, b, l2=False):
    outs, sts = zip(*(oracle.chunk_rule(q[i], k[i], v[i], g[i], b[i], use_qk_l2norm=l2, threads=8)
                      for i in range(q.shape[0])))
    return np.stack(outs), np.stack(sts)


def _inputs(H, S, seed, batch, dtype=torch.float32):
    q, k, v, g, b = chunk_inputs(H, S, seed=seed, batch=batch)
    if dtype != torch.float32:  # the oracle sees the values the kernel sees
        q, k, v = (torch.from_numpy(x).to(dtype).float().numpy() for x in (q, k, v))
    host = (q, k, v, g, b)
    dev = tuple(torch.from_numpy(np.ascontiguousarray(x)).to(DEV) for x in host)
    dev = tuple(t.to(dtype) for t in dev[:3]) + dev[3:]
    return host, dev


def test_noalloc_matches_context_entry_point_twice(cuda_ok):
    for call, (S, seed) in enumerate([(300, 21), (130, 22)]):  # two calls in a row, different sizes
        _, (q, k, v, g, b) = _inputs(4, S, seed, 2)
        out = torch.full((2, 4, S, 128), float("nan"), device=DEV)
        st = torch.full((2, 4, 128, 128), float("nan"), device=DEV)
        rc = _call_noalloc(q, k, v, g, b, out, st)
        assert rc == spock_b200.SPOCK_OK, spock_b200.lib().spock_last_error(None)
        assert _noalloc_sync() == spock_b200.SPOCK_OK
        ref_out, ref_st = spock_b200.chunk_prefill(q, k, v, g, b)  # fp32 inputs: staged in ctx scratch
        torch.cuda.synchronize()
        assert max_rel(out.cpu().numpy(), ref_out.cpu().numpy()) <= TOL, call
        assert max_rel(st.cpu().numpy(), ref_st.cpu().numpy()) <= TOL, call


def test_noalloc_at_its_limit_fp32_matches_oracle(cuda_ok):
    """Exactly 16384 token-heads of fp32 input: all six staged tensors
    (q, k, v and v's low half) fill the fixed array."""
    (hq, hk, hv, hg, hb), (q, k, v, g, b) = _inputs(16, 1024, 31, 1)
    out = torch.full((1, 16, 1024, 128), float("nan"), device=DEV)
    st = torch.full((1, 16, 128, 128), float("nan"), device=DEV)
    assert _call_noalloc(q, k, v, g, b, out, st) == spock_b200.SPOCK_OK, spock_b200.lib().spock_last_error(None)
    assert _noalloc_sync() == spock_b200.SPOCK_OK
    ro, rs = _oracle(hq, hk, hv, hg, hb)
    assert max_rel(out.cpu().numpy(), ro) <= TOL and max_rel(st.cpu().numpy(), rs) <= TOL


def test_noalloc_unstaged_bf16_matches_oracle(cuda_ok):
    """bf16 inputs need no staging (any size): the pipelined kernel reads them directly."""
    (hq, hk, hv, hg, hb), (q, k, v, g, b) = _inputs(16, 600, 32, 2, torch.bfloat16)
    out = torch.empty((2, 16, 600, 128), device=DEV)
    st = torch.empty((2, 16, 128, 128), device=DEV)
    assert _call_noalloc(q, k, v, g, b, out, st) == spock_b200.SPOCK_OK
    assert _noalloc_sync() == spock_b200.SPOCK_OK
    ro, rs = _oracle(hq, hk, hv, hg, hb)
    assert max_rel(out.cpu().numpy(), ro) <= TOL and max_rel(st.cpu().numpy(), rs) <= TOL


def test_noalloc_l2norm_staging(cuda_ok):
    rng = np.random.default_rng(5)
    hq, hk, hv = (rng.standard_normal((1, 2, 100, 128), dtype=np.float32) for _ in range(3))
    hq, hk, hv = (torch.from_numpy(x).half().float().numpy() for x in (hq, hk, hv))
    hg = rng.uniform(-1, -0.01, (1, 2, 100)).astype(np.float32)
    hb = rng.uniform(0, 1, (1, 2, 100)).astype(np.float32)
    q, k, v = (torch.from_numpy(x).to(DEV).half() for x in (hq, hk, hv))
    g, b = torch.from_numpy(hg).to(DEV), torch.from_numpy(hb).to(DEV)
    out = torch.empty((1, 2, 100, 128), device=DEV)
    st = torch.empty((1, 2, 128, 128), device=DEV)
    assert _call_noalloc(q, k, v, g, b, out, st, use_l2=True) == spock_b200.SPOCK_OK
    assert _noalloc_sync() == spock_b200.SPOCK_OK
    ro, rs = _oracle(hq, hk, hv, hg, hb, l2=True)
    assert max_rel(out.cpu().numpy(), ro) <= TOL and max_rel(st.cpu().numpy(), rs) <= TOL


def test_noalloc_second_call_allocates_nothing(cuda_ok):
    """The first call on a device may commit the fixed array (lazy module
    loading); a later call must leave the device's free memory unchanged."""
    _, (q, k, v, g, b) = _inputs(4, 200, 33, 1)
    out = torch.empty((1, 4, 200, 128), device=DEV)
    st = torch.empty((1, 4, 128, 128), device=DEV)
    assert _call_noalloc(q, k, v, g, b, out, st) == spock_b200.SPOCK_OK
    assert _noalloc_sync() == spock_b200.SPOCK_OK
    free0, _ = torch.cuda.mem_get_info(0)
    assert _call_noalloc(q, k, v, g, b, out, st) == spock_b200.SPOCK_OK
    assert _noalloc_sync() == spock_b200.SPOCK_OK
    free1, _ = torch.cuda.mem_get_info(0)
    assert free1 == free0, (free0, free1)


def test_noalloc_timeout_reaches_the_caller(cuda_ok):
    """A bounded wait that gives up writes the fixed array's error word;
    spock_noalloc_sync reports it once, clears it, and later calls work."""
    L = spock_b200.lib()
    assert L.spock_selftest_wait_timeout(None, 64, _stream()) == spock_b200.SPOCK_OK
    assert _noalloc_sync() == spock_b200.SPOCK_ERR_TIMEOUT
    assert b"bounded wait gave up" in L.spock_last_error(None)
    assert _noalloc_sync() == spock_b200.SPOCK_OK
    (hq, hk, hv, hg, hb), (q, k, v, g, b) = _inputs(2, 90, 34, 1)
    out = torch.empty((1, 2, 90, 128), device=DEV)
    st = torch.empty((1, 2, 128, 128), device=DEV)
    assert _call_noalloc(q, k, v, g, b, out, st) == spock_b200.SPOCK_OK
    assert _noalloc_sync() == spock_b200.SPOCK_OK
    ro, rs = _oracle(hq, hk, hv, hg, hb)
    assert max_rel(out.cpu().numpy(), ro) <= TOL and max_rel(st.cpu().numpy(), rs) <= TOL


def test_noalloc_rejects_sizes_beyond_its_fixed_scratch(cuda_ok):
    x = torch.zeros((1, 16, 1025, 128), device=DEV)  # 16400 token-heads > 16384
    s = torch.zeros((1, 16, 1025), device=DEV)
    out = torch.empty_like(x)
    st = torch.empty((1, 16, 128, 128), device=DEV)
    rc = _call_noalloc(x, x, x, s, s, out, st)
    assert rc == spock_b200.SPOCK_ERR_INVALID
    assert b"exceeds the fixed scratch" in spock_b200.lib().spock_last_error(None)
