"""The reference's CLIs rebuilt over the C ABI: spock-deltanet-chunk (JSON in/out,
apps/spock-deltanet-chunk.cpp), spock-decode and spock-bench (apps/spock-*.cpp).
The flag/exit-code checks need no GPU; the runs are marked gpu."""
import json
import os
import subprocess

import numpy as np
import pytest

import oracle
import spock_b200
from tests.golden.gen import chunk_inputs
from tests.util import max_rel

BIN = os.path.join(os.path.dirname(spock_b200.__file__), "bin")


@pytest.fixture(scope="module", autouse=True)
def built():
    spock_b200.build()


def run(name, *args, timeout=600):
    return subprocess.run([os.path.join(BIN, name), *args], capture_output=True, text=True, timeout=timeout)


@pytest.mark.parametrize("name", ["spock-deltanet-chunk", "spock-decode", "spock-bench"])
def test_help(name):
    r = run(name, "--help")
    assert r.returncode == 0 and "usage" in r.stdout


def test_chunk_cli_usage_errors(tmp_path):
    assert run("spock-deltanet-chunk").returncode == 2
    r = run("spock-deltanet-chunk", "--input", str(tmp_path / "missing.json"))
    assert r.returncode == 1 and "cannot open" in r.stderr
    bad = tmp_path / "bad.json"
    bad.write_text('{"num_heads": 0, "sequence_length": 1, "key_dim": 128, "value_dim": 128,'
                   ' "query": [], "key": [], "value": [], "g": [], "beta": []}')
    r = run("spock-deltanet-chunk", "--input", str(bad))
    assert r.returncode == 1 and "must be non-zero" in r.stderr


def test_bench_cli_unknown_mode():
    assert run("spock-bench", "--mode", "nope").returncode == 2


@pytest.mark.gpu
def test_chunk_cli_matches_oracle(cuda_ok, tmp_path):
    q, k, v, g, b = chunk_inputs(2, 70, seed=4)
    doc = dict(num_heads=2, sequence_length=70, key_dim=128, value_dim=128, chunk_size=64, use_qk_l2norm=False,
               query=q.ravel().tolist(), key=k.ravel().tolist(), value=v.ravel().tolist(), g=g.ravel().tolist(),
               beta=b.ravel().tolist())
    p = tmp_path / "in.json"
    p.write_text(json.dumps(doc))
    r = run("spock-deltanet-chunk", "--input", str(p))
    assert r.returncode == 0, r.stderr
    out = json.loads(r.stdout)
    ro, rs = oracle.chunk_rule(q, k, v, g, b)
    assert max_rel(np.array(out["core_attn_out"]), ro.ravel()) <= 1e-3
    assert max_rel(np.array(out["final_state"]), rs.ravel()) <= 1e-3


@pytest.mark.gpu
def test_decode_and_bench_cli_small_model(cuda_ok, tmp_path):
    t = tmp_path / "tok.txt"
    t.write_text("1 2 3 4 5")
    r = run("spock-decode", "--tokens", str(t), "--max-new-tokens", "4", "--layers", "4", "--vocab", "32000")
    assert r.returncode == 0, r.stdout + r.stderr
    d = json.loads(r.stdout)
    assert d["prompt_tokens"] == [1, 2, 3, 4, 5] and d["generated_count"] == 4
    assert all(0 <= x < 32000 for x in d["generated_tokens"])
    r = run("spock-bench", "--mode", "correctness", "--layers", "4", "--vocab", "32000", "--runs", "2", "--warmup", "0")
    assert r.returncode == 0, r.stdout + r.stderr
    assert json.loads(r.stdout)["ok"] is True


def test_bench_cli_config_usage_errors():
    """--config outside 0..4 or more GPUs than present is a usage error (exit 2)."""
    assert run("spock-bench", "--config", "7").returncode == 2
    assert run("spock-bench", "--config", "2", "--gpus", "4096").returncode == 2


@pytest.mark.gpu
@pytest.mark.parametrize("cfg", [0, 1, 2])
def test_bench_cli_configs(cuda_ok, cfg):
    """spock-bench --config N on one GPU prints one JSON line with a positive rate."""
    r = run("spock-bench", "--config", str(cfg), "--gpus", "1", "--runs", "2", "--warmup", "1")
    assert r.returncode == 0, r.stdout + r.stderr
    d = json.loads(r.stdout)
    assert d["config"] == cfg and d["gpus"] == 1 and d["rate"] > 0 and d["ms_per_step"] > 0
