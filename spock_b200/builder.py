"""Builds libspock_b200.so in-tree with nvcc for sm_100a (no JIT cache)."""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
SOURCES = ["capi.cu", "decode_step.cu", "chunk_prefill.cu", "chunk_pipeline.cu", "gemm.cu", "model_kernels.cu", "prefill.cu",
           "exact.cu", "ops.cu", "attn_tc.cu", "model.cu"]
# per-file flags: the exact-order kernels must not contract a*b+c into fma
EXTRA = {"exact.cu": ["--fmad=false"]}
LIB = os.path.join(HERE, "libspock_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]


def _stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(HERE, "..", "include", "spock_b200.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d) and not d.endswith(".o"))


def build(force=False, verbose=False):
    """Compiles every CUDA source for sm_100a and links the C-ABI library."""
    if not force and not _stale():
        return LIB
    objs = []
    for src in SOURCES:
        obj = os.path.join(CSRC, src.replace(".cu", ".o"))
        cmd = [NVCC] + FLAGS + EXTRA.get(src, []) + (["-Xptxas", "-v"] if verbose else []) + [
            "-c", os.path.join(CSRC, src), "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or r.returncode:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode:
            raise RuntimeError("nvcc failed on " + src)
        objs.append(obj)
    cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB] + objs
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("link failed")
    return LIB


APPS = {"spock-deltanet-chunk": "spock_deltanet_chunk.cpp", "spock-decode": "spock_decode.cpp",
        "spock-bench": "spock_bench.cpp"}
BIN = os.path.join(HERE, "bin")


def build_apps(force=False, verbose=False):
    """The reference's CLIs over the C ABI, linked against libspock_b200.so."""
    os.makedirs(BIN, exist_ok=True)
    for name, src in APPS.items():
        out = os.path.join(BIN, name)
        srcp = os.path.join(HERE, "apps", src)
        deps = [srcp, LIB] + [os.path.join(HERE, "apps", f) for f in os.listdir(os.path.join(HERE, "apps"))]
        if not force and os.path.exists(out) and all(os.path.getmtime(d) <= os.path.getmtime(out) for d in deps):
            continue
        cmd = [NVCC, "-O2", "-std=c++17", "-x", "cu", srcp, "-o", out, "-L" + HERE, "-lspock_b200",
               "-Xlinker", "-rpath,$ORIGIN/..", "-gencode", "arch=compute_100a,code=sm_100a"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or r.returncode:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode:
            raise RuntimeError("nvcc failed on " + src)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    build_apps(force="--force" in sys.argv, verbose="-v" in sys.argv)
