"""Parity of the fused decode-step kernel (through the C ABI) with the CPU
restatement of deltanet_conv_l2_qk.comp + deltanet_recurrent_gbeta_norm_gate.comp,
and of the raw recurrent mode with the reference's captured layer-0 fixture.
fp16 outputs use the reference's ULP policy (diary/0089: opt-in N-ULP tolerance,
never a sign flip); exp() may differ from the host libm by an ulp."""
import os

import numpy as np
import pytest
import torch

import oracle
import spock_b200
from tests.golden.gen import decode_inputs
from tests.util import close16, fp16_ulp_diff, max_rel

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "decode_layer0")
ULP = 2


def gpu_step(d):
    dev = torch.device("cuda", 0)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    h16 = lambda a: T(a.view(np.int16))
    layer = spock_b200.DeltaNetLayer(h16(d["conv_w"]), T(d["a_log_bias"]), T(d["norm_w"]))
    qkv, cs, st = h16(d["qkv"]), h16(d["conv_state"]), T(d["state"])
    core = torch.empty((qkv.shape[0], 2048), dtype=torch.int16, device=dev)
    out = spock_b200.deltanet_decode_step(layer, qkv, cs, st, h16(d["a"]), h16(d["b"]), h16(d["z"]),
                                          core_raw=core)
    torch.cuda.synchronize()
    u16 = lambda t: t.cpu().view(torch.int16).numpy().view(np.uint16)
    return u16(out), u16(qkv), u16(cs), st.cpu().numpy(), u16(core)


def cpu_step(d):
    qkv, cs = oracle.conv_l2_qk(d["qkv"], d["conv_state"], d["conv_w"])
    out, st = oracle.rec_norm_gate(qkv, d["state"], d["a"], d["b"], d["a_log_bias"], d["z"], d["norm_w"])
    return out, qkv, cs, st


@pytest.mark.parametrize("batch", [1, 64])
def test_fused_decode_step_matches_oracle(cuda_ok, batch):
    d = decode_inputs(batch, seed=batch)
    go, gqkv, gcs, gst, _ = gpu_step(d)
    co, cqkv, ccs, cst = cpu_step(d)
    assert np.array_equal(gcs, ccs)                       # conv state: pure data movement
    assert fp16_ulp_diff(gqkv, cqkv).max() <= 1           # conv + SiLU + L2 (exp ulp)
    assert max_rel(gst, cst) <= 1e-5                      # fp32 state
    assert close16(go, co), (fp16_ulp_diff(go, co).max(), int((fp16_ulp_diff(go, co) > ULP).sum()))


def test_decode_two_steps_carry_state(cuda_ok):
    d = decode_inputs(4, seed=3)
    _, _, gcs, gst, _ = gpu_step(d)
    _, _, ccs, cst = cpu_step(d)
    d2 = dict(d, conv_state=gcs, state=gst, qkv=decode_inputs(4, seed=4)["qkv"])
    go, _, _, gst2, _ = gpu_step(d2)
    co, _, _, cst2 = cpu_step(dict(d2, conv_state=ccs, state=cst))
    assert max_rel(gst2, cst2) <= 1e-5
    assert close16(go, co)


def test_recurrent_raw_matches_reference_fixture(cuda_ok):
    rd = lambda n, t: np.fromfile(os.path.join(GOLD, n), t)
    st = rd("dn_recurrent_state_pre_262176.f32", np.float32)
    g, beta = st[-32:-16].copy(), st[-16:].copy()
    dev = torch.device("cuda", 0)
    h16 = lambda a: torch.from_numpy(a.view(np.int16)).to(dev).reshape(1, -1)
    state = torch.from_numpy(st[:-32].copy()).to(dev).reshape(1, 16, 128, 128)
    out = spock_b200.deltanet_recurrent(h16(rd("dn_q_2048.fp16", np.uint16)), h16(rd("dn_k_2048.fp16", np.uint16)),
                                        h16(rd("dn_v_2048.fp16", np.uint16)),
                                        torch.from_numpy(g).to(dev).reshape(1, 16),
                                        torch.from_numpy(beta).to(dev).reshape(1, 16), state)
    torch.cuda.synchronize()
    got = out.cpu().view(torch.int16).numpy().view(np.uint16).ravel()
    assert fp16_ulp_diff(got, rd("dn_core_2048.fp16", np.uint16)).max() <= 1
