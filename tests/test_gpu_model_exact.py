"""Exact-order model path (spock_model_desc.exact = 1) against the CPU
restatement of the reference's decode shaders (oracle/model.cpp), bit for bit:
every final-normed hidden state and every greedy token must be identical, at
every position, with no margin rule.

The oracle's prefill is token-serial (the reference's decode semantics); the
GPU's exact prefill runs layer-major but walks each DeltaNet layer's prompt
through the recurrence token by token, so the two must agree exactly.

The config-3/4 geometry tests use BASELINE's model: 24 layers (18 DeltaNet +
6 attention), vocab 248320, a 512-token prompt and 128 greedy tokens."""
import os

import numpy as np
import pytest
import torch

import oracle
import spock_b200
from tests.golden.gen import model_weights

pytestmark = pytest.mark.gpu
THREADS = os.cpu_count() or 8


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def _serial_oracle(cpu, prompt, n_new):
    """prompt [B,P] token by token, then n_new greedy tokens. Returns (tokens
    [B,n_new], hidden [n_new][B,1024] bits): token 0 follows the prompt."""
    B, P = prompt.shape
    cpu.reset(B)
    for t in range(P - 1):
        cpu.step(prompt[:, t], threads=THREADS)
    tok = prompt[:, P - 1]
    toks, hids = [], []
    for _ in range(n_new):
        tok, hid, _ = cpu.step(tok, threads=THREADS)
        toks.append(tok.copy())
        hids.append(hid.copy())
    return np.stack(toks, 1), hids


@pytest.fixture(scope="module")
def small_weights():
    return model_weights(4, 32000, seed=3)


def test_exact_teacher_forced_steps_small(cuda_ok, small_weights):
    """4 layers, batch 3 (small-batch projections), 8 teacher-forced steps."""
    m = spock_b200.Model(4, 32000, max_batch=3, max_seq=64, exact=True)
    m.set_weights(small_weights)
    cpu = oracle.Model(small_weights, 4, 32000, 64)
    toks = np.random.default_rng(0).integers(0, 32000, (8, 3)).astype(np.int32)
    m.reset(3)
    cpu.reset(3)
    try:
        for t in range(8):
            g_tok, g_hid = m.step(torch.from_numpy(toks[t]).cuda())
            torch.cuda.synchronize()
            c_tok, c_hid, _ = cpu.step(toks[t], threads=THREADS)
            assert np.array_equal(_bits(g_hid), c_hid), t
            assert np.array_equal(g_tok.cpu().numpy(), c_tok), t
    finally:
        m.close()


@pytest.mark.parametrize("B,rows", [(12, [0, 7, 11]), (96, [0, 50, 95])])
def test_exact_batched_projection_paths_small(cuda_ok, small_weights, B, rows):
    """Batches above 8 take the register-tiled projections (12: 64-row tiles
    with padding; 96: 128-row tiles); rows are independent sequences."""
    m = spock_b200.Model(4, 32000, max_batch=B, max_seq=64, exact=True)
    m.set_weights(small_weights)
    cpu = oracle.Model(small_weights, 4, 32000, 64)
    toks = np.random.default_rng(B).integers(0, 32000, (4, B)).astype(np.int32)
    m.reset(B)
    cpu.reset(len(rows))
    try:
        for t in range(4):
            g_tok, g_hid = m.step(torch.from_numpy(toks[t]).cuda())
            torch.cuda.synchronize()
            c_tok, c_hid, _ = cpu.step(toks[t, rows], threads=THREADS)
            assert np.array_equal(_bits(g_hid)[rows], c_hid), t
            assert np.array_equal(g_tok.cpu().numpy()[rows], c_tok), t
    finally:
        m.close()


def test_exact_prefill_and_generate_small(cuda_ok, small_weights):
    """Layer-major exact prefill of a 70-token prompt (batch 2) and 12
    graph-replayed greedy tokens equal the oracle's token-serial run."""
    m = spock_b200.Model(4, 32000, max_batch=2, max_seq=96, exact=True)
    m.set_weights(small_weights)
    cpu = oracle.Model(small_weights, 4, 32000, 96)
    prompt = np.random.default_rng(7).integers(0, 32000, (2, 70)).astype(np.int32)
    try:
        m.reset(2)
        tok, hid = m.prefill(torch.from_numpy(prompt).cuda())
        torch.cuda.synchronize()
        ref_tok, ref_hid = _serial_oracle(cpu, prompt, 13)
        assert np.array_equal(tok.cpu().numpy(), ref_tok[:, 0])
        assert np.array_equal(_bits(hid), ref_hid[0])
        m.reset(2)
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            out = m.generate(torch.from_numpy(prompt).cuda(), 13, stream=s)
        s.synchronize()
        m.sync()
        assert np.array_equal(out.cpu().numpy(), ref_tok)
    finally:
        m.close()


@pytest.fixture(scope="module")
def full_weights():
    return model_weights(24, 248320, seed=11)


def test_exact_config3_and_config4_batch1(cuda_ok, full_weights):
    """BASELINE configs 3 and 4 at batch 1: prefill of a 512-token prompt
    (final-normed hidden of its last token and the first greedy token), then
    128 greedy tokens, all bit-identical to the oracle."""
    P, N = 512, 128
    prompt = np.random.default_rng(0).integers(0, 248320, (1, P)).astype(np.int32)
    m = spock_b200.Model(24, 248320, max_batch=1, max_seq=P + N + 8, exact=True)
    m.set_weights(full_weights)
    cpu = oracle.Model(full_weights, 24, 248320, P + N + 8)
    try:
        m.reset(1)
        tok, hid = m.prefill(torch.from_numpy(prompt).cuda())
        torch.cuda.synchronize()
        ref_tok, ref_hid = _serial_oracle(cpu, prompt, N)
        assert np.array_equal(_bits(hid), ref_hid[0])          # config 3: final-layer hidden
        assert int(tok.cpu()[0]) == int(ref_tok[0, 0])          # config 3: first greedy token
        m.reset(1)
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            out = m.generate(torch.from_numpy(prompt).cuda(), N, stream=s)
        s.synchronize()
        m.sync()
        mism = np.nonzero(out.cpu().numpy()[0] != ref_tok[0])[0]
        assert mism.size == 0, f"first mismatch at token {mism[:1]}"  # config 4: all 128 tokens
    finally:
        m.close()


def test_exact_config4_batch256_rows(cuda_ok, full_weights):
    """BASELINE config 4's 256 concurrent sequences (512-token prompts, 128
    greedy tokens each) on one GPU; two of the sequences are replayed on the
    oracle and must match at every position."""
    B, P, N, rows = 256, 512, 128, [0, 201]
    prompts = np.random.default_rng(1).integers(0, 248320, (B, P)).astype(np.int32)
    m = spock_b200.Model(24, 248320, max_batch=B, max_seq=P + N + 8, exact=True)
    m.set_weights(full_weights)
    try:
        m.reset(B)
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            out = m.generate(torch.from_numpy(prompts).cuda(), N, stream=s)
        s.synchronize()
        m.sync()
        out = out.cpu().numpy()
    finally:
        m.close()
    cpu = oracle.Model(full_weights, 24, 248320, P + N + 8)
    ref_tok, _ = _serial_oracle(cpu, prompts[rows], N)
    assert np.array_equal(out[rows], ref_tok)
