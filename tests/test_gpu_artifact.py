"""Weight loading from a repacked text artifact (the reference's
text_repack_manifest.json + text_weights.bin) gives a model identical to one
fed the same tensors role by role."""
import json
import os
import subprocess

import numpy as np
import pytest
import torch

import spock_b200
from tests.golden.gen import model_weights, write_repack_artifact

pytestmark = pytest.mark.gpu
LAYERS, VOCAB = 4, 32000
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def weights():
    return model_weights(LAYERS, VOCAB, seed=5)


def test_artifact_matches_role_uploads(cuda_ok, weights, tmp_path):
    write_repack_artifact(str(tmp_path), weights)
    a = spock_b200.Model(LAYERS, VOCAB, max_batch=2, max_seq=16)
    b = spock_b200.Model(LAYERS, VOCAB, max_batch=2, max_seq=16)
    try:
        a.load_artifact(str(tmp_path))
        b.set_weights(weights)
        a.reset(2)
        b.reset(2)
        tok = torch.tensor([7, 31000], dtype=torch.int32, device="cuda")
        ta, tb = tok, tok
        for _ in range(3):
            ta, ha = a.step(ta)
            tb, hb = b.step(tb)
            torch.cuda.synchronize()
            assert torch.equal(ta, tb)
            assert torch.equal(ha.view(torch.int16), hb.view(torch.int16))
    finally:
        a.close()
        b.close()


def test_artifact_missing_role_is_reported(cuda_ok, weights, tmp_path):
    write_repack_artifact(str(tmp_path), weights, drop=("layer.2.delta_norm",))
    m = spock_b200.Model(LAYERS, VOCAB, max_batch=1, max_seq=16)
    try:
        with pytest.raises(spock_b200.SpockError, match="layer.2.delta_norm"):
            m.load_artifact(str(tmp_path))
    finally:
        m.close()


def test_spock_decode_cli_loads_artifact(cuda_ok, weights, tmp_path):
    write_repack_artifact(str(tmp_path / "art"), weights)
    toks = tmp_path / "prompt.txt"
    toks.write_text("9419 11 1814 0\n")
    exe = os.path.join(HERE, "..", "spock_b200", "bin", "spock-decode")
    r = subprocess.run([exe, "--tokens", str(toks), "--max-new-tokens", "4", "--layers", str(LAYERS), "--vocab",
                        str(VOCAB), "--repack-dir", str(tmp_path / "art")], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    out = json.loads(r.stdout)
    assert out["generated_count"] == 4 and len(out["generated_tokens"]) == 4
    # same tokens as the library path with the same weights
    m = spock_b200.Model(LAYERS, VOCAB, max_batch=1, max_seq=16)
    try:
        m.set_weights(weights)
        m.reset(1)
        stream = torch.cuda.Stream()
        with torch.cuda.stream(stream):
            gen = m.generate(torch.tensor([[9419, 11, 1814, 0]], dtype=torch.int32, device="cuda"), 4, stream=stream)
        stream.synchronize()
        assert gen.cpu().numpy().ravel().tolist() == out["generated_tokens"]
    finally:
        m.close()
