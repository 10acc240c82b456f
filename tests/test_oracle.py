"""The CPU oracle pinned against the reference: its compiled run_deltanet_chunk_rule
(oracle/_ref), its torch unit test's case, its probe geometry, and its captured
decode fixture."""
import os

import numpy as np
import pytest

import oracle
from tests.golden.gen import chunk_inputs

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _need_ref():
    if oracle.ref_lib() is None:
        pytest.skip("reference sources not present: oracle/_ref not built")


@pytest.mark.parametrize("S,init", [(104, False), (1, False), (64, True), (65, True), (200, False)])
def test_oracle_bitexact_vs_reference(S, init):
    _need_ref()
    H = 4
    q, k, v, g, b = chunk_inputs(H, S, seed=S)
    st0 = np.random.default_rng(1).standard_normal((H, 128, 128)).astype(np.float32) if init else None
    o1, s1 = oracle.chunk_rule(q, k, v, g, b, initial_state=st0, threads=4)
    o2, s2 = oracle.chunk_rule(q, k, v, g, b, initial_state=st0, use_reference=True)
    assert np.array_equal(o1, o2) and np.array_equal(s1, s2)


def test_oracle_l2norm_path_bitexact():
    _need_ref()
    rng = np.random.default_rng(3)
    q, k, v = (rng.standard_normal((2, 70, 128), dtype=np.float32) for _ in range(3))
    g = rng.uniform(-1, -0.01, (2, 70)).astype(np.float32)
    b = rng.uniform(0, 1, (2, 70)).astype(np.float32)
    r1 = oracle.chunk_rule(q, k, v, g, b, use_qk_l2norm=True)
    r2 = oracle.chunk_rule(q, k, v, g, b, use_qk_l2norm=True, use_reference=True)
    assert all(np.array_equal(x, y) for x, y in zip(r1, r2))


def test_unit_case_golden():
    d = np.load(os.path.join(GOLD, "chunk_unit.npz"))
    o, s = oracle.chunk_rule(d["q"], d["k"], d["v"], d["g"], d["beta"], chunk_size=int(d["chunk"]),
                             use_qk_l2norm=True, initial_state=d["init"])
    # the reference's own bar (tests/run_deltanet_chunk_unit.py:176-179)
    assert np.abs(o - d["torch_out"]).max() <= 1e-5
    assert np.abs(s - d["torch_state"]).max() <= 1e-5
    assert np.array_equal(o, d["ref_out"]) and np.array_equal(s, d["ref_state"])


def test_probe_golden():
    d = np.load(os.path.join(GOLD, "chunk_probe_h4.npz"))
    o, s = oracle.chunk_rule(d["q"], d["k"], d["v"], d["g"], d["beta"])
    assert np.array_equal(o, d["ref_out"]) and np.array_equal(s, d["ref_state"])


def test_decode_recurrent_golden():
    p = os.path.join(GOLD, "decode_layer0")
    rd = lambda n, t: np.fromfile(os.path.join(p, n), t)
    out, _ = oracle.recurrent_raw(rd("dn_q_2048.fp16", np.uint16), rd("dn_k_2048.fp16", np.uint16),
                                  rd("dn_v_2048.fp16", np.uint16),
                                  rd("dn_recurrent_state_pre_262176.f32", np.float32))
    assert np.array_equal(out, rd("dn_core_2048.fp16", np.uint16))


def test_oracle_rejects_zero_fields():
    q = np.zeros((1, 1, 128), np.float32)
    with pytest.raises(RuntimeError):
        oracle.chunk_rule(q, q, q, np.zeros((1, 1), np.float32), np.zeros((1, 1), np.float32), chunk_size=0)


def test_oracle_threads_do_not_change_results():
    q, k, v, g, b = chunk_inputs(8, 130, seed=5)
    r1 = oracle.chunk_rule(q, k, v, g, b, threads=1)
    r8 = oracle.chunk_rule(q, k, v, g, b, threads=8)
    assert all(np.array_equal(x, y) for x, y in zip(r1, r8))


def _fixture(name, dtype=np.uint16):
    return np.fromfile(os.path.join(GOLD, "decode_layer0", name), dtype)


def test_silu_gate_golden():
    """silu_gate.comp pinned on the reference's captured layer-0 MLP tensors."""
    out = oracle.silu_gate(_fixture("mlp_gate_3584.fp16"), _fixture("mlp_up_3584.fp16"))
    assert np.array_equal(out, _fixture("mlp_product_3584.fp16"))


def test_residual_adds_golden():
    """residual_add.comp pinned twice: h + mixer -> mixer_residual, then + down -> post_mlp."""
    mixed = oracle.residual_add(_fixture("input_hidden_1024.fp16"), _fixture("mixer_output_1024.fp16"))
    assert np.array_equal(mixed, _fixture("mixer_residual_1024.fp16"))
    post = oracle.residual_add(mixed, _fixture("down_output_1024.fp16"))
    assert np.array_equal(post, _fixture("post_mlp_1024.fp16"))


def test_beta_golden():
    """beta = sigmoid(b) of the g/beta phase, pinned on the captured b and the
    beta half of the captured g/beta tail (g also needs A_log / dt_bias weights,
    which are not among the fixtures). GLSL leaves exp()'s precision to the
    implementation and the oracle evaluates it in double, so the bar is one
    fp32 ulp; 14 of the 16 values are bit-identical."""
    gb = _fixture("dn_g_beta_32.u32", np.uint32).view(np.float32)
    b = _fixture("dn_b_16.fp16")
    _, beta = oracle.gbeta(np.zeros(16, np.uint16), b, np.zeros((16, 2), np.float32))
    ulps = np.abs(beta.view(np.int32).astype(np.int64) - gb[16:].view(np.int32).astype(np.int64))
    assert ulps.max() <= 1 and (ulps == 0).sum() >= 14, ulps


def test_matvec_is_sequential_per_row():
    """The oracle's matvec (vectorised across rows for speed) equals a plain
    sequential fp32 loop per row, as matvec.comp:28-41 computes it."""
    rng = np.random.default_rng(3)
    W = (rng.standard_normal((13, 1024)) * 0.02).astype(np.float16)
    x = rng.standard_normal(1024).astype(np.float16)
    got = oracle.matvec(W.view(np.uint16), x.view(np.uint16))
    for r in range(13):
        s = np.float32(0)
        for j in range(1024):
            s = np.float32(s + np.float32(np.float32(W[r, j]) * np.float32(x[j])))
        assert got[r] == np.float16(s).view(np.uint16), r
