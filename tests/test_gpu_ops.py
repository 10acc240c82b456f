"""Per-op parity of the decode glue through the C ABI (spock_rms_norm,
spock_matvec, spock_argmax, spock_attention_decode) against the CPU
restatement of each shader (oracle/model.cpp, oracle/decode_ops.cpp).

Exact-order kernels must equal the restatement bit for bit. The fast kernels
accumulate the projections on tensor cores (and the attention with an online
softmax), so their fp16 results may differ by a rounding: <= 2 fp16 ulp or
<= 2^-10 absolute (the decode tests' policy)."""
import numpy as np
import pytest
import torch

import oracle
import spock_b200
from tests.util import close16, fp16_ulp_diff

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def _h(a, sd, rng):
    return (rng.standard_normal(a).astype(np.float32) * sd).astype(np.float16)


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def test_rms_norm_matches_shader_restatement(cuda_ok):
    rng = np.random.default_rng(1)
    x, w = _h((9, 1024), 1.0, rng), _h(1024, 0.1, rng)
    y = spock_b200.rms_norm(_dev(x), _dev(w))
    torch.cuda.synchronize()
    ref = np.stack([oracle.rms_norm(x[r].view(np.uint16), w.view(np.uint16)) for r in range(9)])
    assert np.array_equal(_bits(y), ref)


def _oracle_rows(W, X):
    return np.stack([oracle.matvec(W.view(np.uint16), X[r].view(np.uint16)) for r in range(X.shape[0])])


@pytest.mark.parametrize("exact", [True, False])
@pytest.mark.parametrize("rows", [1, 5, 40, 200])
def test_matvec_epilogues(cuda_ok, exact, rows):
    """STORE, RESIDUAL and SILU_GATE (gate/up rows interleaved by 16) on the
    qkv/out/MLP shapes, across the small-batch (<= 8 rows) and batched paths."""
    rng = np.random.default_rng(rows)
    check = (lambda a, b: np.array_equal(a, b)) if exact else (lambda a, b: close16(a, b))
    # STORE: in-projection of a DeltaNet layer (8224 x 1024)
    W, X = _h((8224, 1024), 0.02, rng), _h((rows, 1024), 1.0, rng)
    y = spock_b200.matvec(_dev(W), _dev(X), spock_b200.MV_STORE, exact=exact)
    torch.cuda.synchronize()
    ref = _oracle_rows(W, X)
    assert check(_bits(y), ref), int(fp16_ulp_diff(_bits(y), ref).max())
    # RESIDUAL: out-projection (1024 x 2048) added onto h
    W2, X2, H = _h((1024, 2048), 0.02, rng), _h((rows, 2048), 1.0, rng), _h((rows, 1024), 1.0, rng)
    h = _dev(H)
    spock_b200.matvec(_dev(W2), _dev(X2), spock_b200.MV_RESIDUAL, residual=h, exact=exact, out=h)
    torch.cuda.synchronize()
    ref = np.stack([oracle.residual_add(H[r].view(np.uint16), m) for r, m in enumerate(_oracle_rows(W2, X2))])
    assert check(_bits(h), ref)
    # SILU_GATE: gate and up (3584 x 1024 each), interleaved in groups of 16 rows
    G, U = _h((3584, 1024), 0.02, rng), _h((3584, 1024), 0.02, rng)
    Wgu = np.stack([G.reshape(224, 16, 1024), U.reshape(224, 16, 1024)], 1).reshape(7168, 1024)
    y = spock_b200.matvec(_dev(Wgu), _dev(X), spock_b200.MV_SILU_GATE, exact=exact)
    torch.cuda.synchronize()
    ref = np.stack([oracle.silu_gate(g, u) for g, u in zip(_oracle_rows(G, X), _oracle_rows(U, X))])
    assert check(_bits(y), ref), int(fp16_ulp_diff(_bits(y), ref).max())


def _ref_rows(W, X):
    """fp16 bits of fp16(W @ x) per row, from a float64 product on the GPU."""
    w = torch.from_numpy(W.view(np.float16)).to(DEV).double()
    x = torch.from_numpy(X.view(np.float16)).to(DEV).double()
    return (x @ w.T).half().cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("rows", [512, 1000])
def test_matvec_prefill_row_counts(cuda_ok, rows):
    """The fast path at prefill row counts (a 512-token prompt, and a ragged
    1000): the persistent GEMM's 256-row units, its K-split plans for the
    1024-output projections, and the partial last unit. The products are
    checked against a float64 product rounded to fp16 (the oracle's
    sequential sums are too slow at these sizes; both round the same exact
    value), the residual add and SwiGLU with the oracle's element rules, all
    within the fast path's 2-ulp policy."""
    rng = np.random.default_rng(rows)
    X = _h((rows, 1024), 1.0, rng)
    W = _h((8224, 1024), 0.02, rng)
    y = spock_b200.matvec(_dev(W), _dev(X), spock_b200.MV_STORE)
    torch.cuda.synchronize()
    got, ref = _bits(y), _ref_rows(W.view(np.uint16), X.view(np.uint16))
    assert close16(got, ref), int(fp16_ulp_diff(got, ref).max())
    X2, H = _h((rows, 3584), 1.0, rng), _h((rows, 1024), 1.0, rng)
    W2 = _h((1024, 3584), 0.02, rng)
    h = _dev(H)
    spock_b200.matvec(_dev(W2), _dev(X2), spock_b200.MV_RESIDUAL, residual=h, out=h)
    torch.cuda.synchronize()
    mv = _ref_rows(W2.view(np.uint16), X2.view(np.uint16))
    ref = np.stack([oracle.residual_add(H[r].view(np.uint16), mv[r]) for r in range(rows)])
    # The projection's fp16 rounding may differ by up to 2 ulps of the
    # projection, which the residual add keeps in absolute terms (where the
    # sum cancels, that is many ulps of the small result): allow 2 ulps of
    # the projection plus one rounding of the sum.
    f = lambda b: b.view(np.float16).astype(np.float32)
    ulp = lambda b: np.spacing(np.abs(b.view(np.float16))).astype(np.float32)
    err = np.abs(f(_bits(h)) - f(ref))
    assert np.all(err <= 2 * ulp(mv) + ulp(ref)), float((err - 2 * ulp(mv) - ulp(ref)).max())
    G, U = _h((3584, 1024), 0.02, rng), _h((3584, 1024), 0.02, rng)
    Wgu = np.stack([G.reshape(224, 16, 1024), U.reshape(224, 16, 1024)], 1).reshape(7168, 1024)
    y = spock_b200.matvec(_dev(Wgu), _dev(X), spock_b200.MV_SILU_GATE)
    torch.cuda.synchronize()
    g_, u_ = _ref_rows(G.view(np.uint16), X.view(np.uint16)), _ref_rows(U.view(np.uint16), X.view(np.uint16))
    ref = np.stack([oracle.silu_gate(a, b) for a, b in zip(g_, u_)])
    assert close16(_bits(y), ref), int(fp16_ulp_diff(_bits(y), ref).max())


@pytest.mark.parametrize("exact", [True, False])
@pytest.mark.parametrize("rows", [1, 3, 12])
def test_lm_head_argmax_full_vocab(cuda_ok, exact, rows):
    """The tied LM head at the model's real vocab (248320 x 1024) with the
    argmax epilogue. Exact: the token equals the restatement's. Fast: the
    chosen token's logit is the maximum within one fp16 rounding."""
    g = torch.Generator(device=DEV).manual_seed(rows)
    E = (torch.randn(248320, 1024, device=DEV, generator=g) * 0.02).half()
    X = torch.randn(rows, 1024, device=DEV, generator=g).half()
    tok = spock_b200.matvec(E, X, spock_b200.MV_ARGMAX, exact=exact).cpu().numpy()
    En, Xn = E.cpu().numpy(), X.cpu().numpy()
    for r in range(rows):
        logits = oracle.matvec(En.view(np.uint16), Xn[r].view(np.uint16))
        if exact:
            assert tok[r] == oracle.argmax(logits), r
        else:
            lf = logits.view(np.float16).astype(np.float32)
            assert lf[tok[r]] >= lf.max() - 2 * np.spacing(np.float16(lf.max())), r


@pytest.mark.parametrize("exact", [True, False])
def test_argmax_epilogue_planted_ties(cuda_ok, exact):
    """Duplicate weight rows give exactly equal logits: the lowest index must win
    (argmax.comp's strict '>'), in every 128-row tile position."""
    rng = np.random.default_rng(5)
    W = _h((4096, 1024), 0.02, rng)
    X = _h((2, 1024), 1.0, rng)
    best = int(np.argmax(W.astype(np.float32) @ X[0].astype(np.float32)))
    W[[300, 2000, 4095]] = W[best]  # three more copies of the winning row
    W[[best, 300, 2000, 4095]] *= np.float16(1.5)  # keep the copies on top
    want = min(best, 300)
    tok = spock_b200.matvec(_dev(W), _dev(X[:1]), spock_b200.MV_ARGMAX, exact=exact).cpu().numpy()
    logits = oracle.matvec(W.view(np.uint16), X[0].view(np.uint16))
    assert oracle.argmax(logits) == want
    assert tok[0] == want


def test_argmax_standalone_planted_ties(cuda_ok):
    rng = np.random.default_rng(2)
    L = _h((4, 248320), 1.0, rng)
    L[0, [5, 99, 248319]] = np.float16(9.0)           # tie at the top: index 5
    L[1, [248318, 248319]] = np.float16(9.0)          # tie in the last positions
    L[2, :] = np.float16(-0.0)
    L[2, 17] = np.float16(0.0)                        # +0 == -0: the first zero wins
    L[3, 131071:131075] = np.float16(11.0)            # a tie across a thread stride boundary
    got = spock_b200.argmax(_dev(L)).cpu().numpy()
    ref = [oracle.argmax(L[r].view(np.uint16)) for r in range(4)]
    assert list(got) == ref == [5, 248318, 0, 131071]


@pytest.mark.parametrize("exact", [True, False])
def test_attention_decode(cuda_ok, exact):
    """split_q_gate + per-head q/k norm + RoPE + KV store + attention + sigmoid
    gate for three sequences at positions 0, 7 and 300 (earlier positions of
    the cache hold random keys and values)."""
    rng = np.random.default_rng(9)
    max_seq, pos = 320, np.array([0, 7, 300], np.int32)
    proj = _h((3, 5120), 1.0, rng)
    qn, kn = _h(256, 0.1, rng), _h(256, 0.1, rng)
    cache = _h((3, max_seq, 2, 2, 256), 1.0, rng)
    kv = _dev(cache)
    out = spock_b200.attention_decode(_dev(proj), _dev(qn), _dev(kn), _dev(pos), kv, exact=exact)
    torch.cuda.synchronize()
    got, got_kv = _bits(out), _bits(kv)
    for r in range(3):
        ref, ref_cache = oracle.attention_decode(proj[r].view(np.uint16), qn.view(np.uint16), kn.view(np.uint16),
                                                 cache[r].view(np.uint16), pos[r])
        assert np.array_equal(got_kv[r], ref_cache), r  # K (normed, rotated) and V rows stored exactly
        if exact:
            assert np.array_equal(got[r], ref), r
        else:
            assert close16(got[r], ref), (r, int(fp16_ulp_diff(got[r], ref).max()))


@pytest.mark.parametrize("exact", [True, False])
def test_attention_prefill(cuda_ok, exact):
    """The layer-major prefill's attention for 2 sequences x 70 prompt tokens
    (3 query tiles of the tcgen05 kernel, 2-3 KV tiles each), the second
    sequence continuing after 40 cached positions: every row against the
    oracle's token-serial attention over the same cache."""
    rng = np.random.default_rng(12)
    B, T, max_seq = 2, 70, 128
    pos = np.array([0, 40], np.int32)
    proj = _h((B, T, 5120), 1.0, rng)
    qn, kn = _h(256, 0.1, rng), _h(256, 0.1, rng)
    cache = _h((B, max_seq, 2, 2, 256), 1.0, rng)
    kv = _dev(cache)
    out = spock_b200.attention_prefill(_dev(proj), _dev(qn), _dev(kn), _dev(pos), kv, exact=exact)
    torch.cuda.synchronize()
    got = _bits(out)
    worst = 0
    for b in range(B):
        c = cache[b].view(np.uint16)
        for t in range(T):
            ref, c = oracle.attention_decode(proj[b, t].view(np.uint16), qn.view(np.uint16), kn.view(np.uint16), c,
                                             pos[b] + t)
            if exact:
                assert np.array_equal(got[b, t], ref), (b, t)
            else:
                assert close16(got[b, t], ref), (b, t, int(fp16_ulp_diff(got[b, t], ref).max()))
            worst = max(worst, int(fp16_ulp_diff(got[b, t], ref).max()))
        assert np.array_equal(_bits(kv)[b, :pos[b] + T], c[:pos[b] + T]), b
