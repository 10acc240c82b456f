"""Multi-process paths on CPU (gloo, world_size 2): bench.py's reference arm
under torchrun (rank 0 alone prints; other ranks exit 0 without work) and the
max-over-ranks reduction the GPU arm uses for timing."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _torchrun(args, nproc=2, port=29517, timeout=600):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr", "127.0.0.1", "--master-port", str(port)] + args
    env = dict(os.environ, OMP_NUM_THREADS="1")
    return subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=timeout, env=env)


def test_reference_arm_under_torchrun_rank0_prints_once():
    r = _torchrun(["bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["cpu_baseline"]["cores"] >= 1


def test_max_over_ranks_gloo(tmp_path):
    script = tmp_path / "mor.py"
    script.write_text(
        "import os, sys, torch.distributed as dist\n"
        f"sys.path.insert(0, {ROOT!r})\n"
        "import bench\n"
        "dist.init_process_group('gloo')\n"
        "r = dist.get_rank()\n"
        "v = bench.max_over_ranks(float(10 + r), dist.get_world_size())\n"
        "assert v == 11.0, v\n"
        "bench.barrier(2)\n"
        "print('ok', r)\n"
        "dist.destroy_process_group()\n")
    r = _torchrun([str(script)], port=29518, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.count("ok") == 2


def test_sequence_partition_gloo(tmp_path):
    """bench.py's strong-scaling split: on 2 gloo ranks, every one of the 64
    config-2 sequences (and config 4's 256, and a ragged 7) is owned by exactly
    one rank, in contiguous blocks, and the union is all of them."""
    script = tmp_path / "part.py"
    script.write_text(
        "import os, sys, torch, torch.distributed as dist\n"
        f"sys.path.insert(0, {ROOT!r})\n"
        "import bench\n"
        "dist.init_process_group('gloo')\n"
        "r, ws = dist.get_rank(), dist.get_world_size()\n"
        "for total in (64, 256, 7):\n"
        "    first, n = bench.shard(total, ws, r)\n"
        "    mine = torch.zeros(total, dtype=torch.int64)\n"
        "    mine[first:first + n] = 1\n"
        "    dist.all_reduce(mine)\n"
        "    assert torch.equal(mine, torch.ones(total, dtype=torch.int64)), (total, mine)\n"
        "    lo = torch.tensor([first]); dist.all_reduce(lo, op=dist.ReduceOp.MIN)\n"
        "    assert lo.item() == 0\n"
        "print('ok', r)\n"
        "dist.destroy_process_group()\n")
    r = _torchrun([str(script)], port=29519, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.count("ok") == 2
