"""Regenerates the golden fixtures in this directory (run once, in a checkout
that has the reference at REF; the GPU box never runs this).

  chunk_unit.npz      the reference's own chunk-rule unit case
                      (tests/run_deltanet_chunk_unit.py:104-116: torch seed 0,
                      H=2 S=5 K=3 V=2 C=4, g~N*0.2-0.3, beta=sigmoid(N),
                      init_state~0.1N), expected outputs from the reference's
                      torch restatement of HF torch_chunk_gated_delta_rule
                      (that file :19-92) AND from the reference's compiled C++
                      run_deltanet_chunk_rule (oracle/_ref).
  chunk_probe_h4.npz  the GPU chunk-prefill probe geometry
                      (apps/spock-deltanet-chunk-prefill-probe.cpp:215-250):
                      xorshift32 inputs with its seeds and ranges, H=4 of its 16
                      heads, S=104, C=64, K=V=128, outputs of oracle/_ref.
  decode_layer0/      the reference's captured layer-0 decode fixtures for the
                      recurrent probe (CMakeLists.txt:144), copied verbatim:
                      q,k,v fp16 [2048], state_pre f32 [16*128*128 + 32]
                      (g and beta in the tail), expected raw output fp16 [2048];
                      and the weight-free glue fixtures of the same step
                      (mlp gate/up -> product, residual adds, b -> beta).
"""
import importlib.util
import os
import shutil
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# the reference checkout: $SPOCK_REFERENCE, else a checkout named "reference"
# beside this repository
REF = os.environ.get("SPOCK_REFERENCE") or os.path.abspath(
    os.path.join(os.path.dirname(__file__), "..", "..", "..", "reference"))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import oracle  # noqa: E402
from tests.golden.gen import probe_inputs  # noqa: E402


def unit_case():
    import torch
    spec = importlib.util.spec_from_file_location("ref_unit", os.path.join(REF, "tests", "run_deltanet_chunk_unit.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    torch.manual_seed(0)
    H, S, K, V, C = 2, 5, 3, 2, 4
    q = torch.randn(1, S, H, K)
    k = torch.randn(1, S, H, K)
    v = torch.randn(1, S, H, V)
    g = torch.randn(1, S, H) * 0.2 - 0.3
    beta = torch.sigmoid(torch.randn(1, S, H))
    init = torch.randn(1, H, K, V) * 0.1
    exp_out, exp_state = m.torch_chunk_gated_delta_rule(q, k, v, g, beta, chunk_size=C, initial_state=init,
                                                        output_final_state=True, use_qk_l2norm_in_kernel=True)
    hm = lambda x: x[0].transpose(0, 1).contiguous().numpy()  # [S,H,..] -> [H,S,..]
    d = dict(q=hm(q), k=hm(k), v=hm(v), g=g[0].T.contiguous().numpy(), beta=beta[0].T.contiguous().numpy(),
             init=init[0].numpy(), chunk=np.int64(C),
             torch_out=hm(exp_out), torch_state=exp_state[0].numpy())
    ro, rs = oracle.chunk_rule(d["q"], d["k"], d["v"], d["g"], d["beta"], chunk_size=C, use_qk_l2norm=True,
                               initial_state=d["init"], use_reference=True)
    d["ref_out"], d["ref_state"] = ro, rs
    np.savez(os.path.join(HERE, "chunk_unit.npz"), **d)


def probe_case():
    q, k, v, g, b = probe_inputs(heads=4)
    ro, rs = oracle.chunk_rule(q, k, v, g, b, chunk_size=64, use_qk_l2norm=False, use_reference=True)
    np.savez(os.path.join(HERE, "chunk_probe_h4.npz"), q=q, k=k, v=v, g=g, beta=b, ref_out=ro, ref_state=rs)


def decode_case():
    dst = os.path.join(HERE, "decode_layer0")
    os.makedirs(dst, exist_ok=True)
    for name in ["dn_q_2048.fp16", "dn_k_2048.fp16", "dn_v_2048.fp16", "dn_g_beta_32.u32",
                 "dn_recurrent_state_pre_262176.f32", "dn_core_2048.fp16",
                 # weight-free glue fixtures: silu_gate.comp, residual_add.comp, and
                 # the beta = sigmoid(b) half of the g/beta computation
                 "mlp_gate_3584.fp16", "mlp_up_3584.fp16", "mlp_product_3584.fp16",
                 "input_hidden_1024.fp16", "mixer_output_1024.fp16", "mixer_residual_1024.fp16",
                 "down_output_1024.fp16", "post_mlp_1024.fp16", "dn_b_16.fp16"]:
        shutil.copyfile(os.path.join(REF, "tests", "data", "layer0_step1_" + name), os.path.join(dst, name))


if __name__ == "__main__":
    oracle.build()
    unit_case()
    probe_case()
    decode_case()
    print("golden fixtures written to", HERE)
