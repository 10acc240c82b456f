"""Seeded synthetic input generators shared by tests, smoke() and bench.py.

probe_inputs restates the deterministic generator of the reference's GPU
chunk-prefill probe (apps/spock-deltanet-chunk-prefill-probe.cpp:215-270):
xorshift32 (13/17/5) per array with fixed seeds, mapped to [lo, hi], q and k
L2-normalised per (head, token) with eps 1e-6 inside the sqrt, head-major
layouts. The BASELINE configs use numpy's PCG64 (default_rng) instead.
"""
import numpy as np

PROBE_SEEDS = dict(q=0xDEADBEEF, k=0xCAFEBABE, v=0xDECAFBAD, g=0xABADCAFE, beta=0xBEEFCACE)
PROBE_RANGES = dict(q=(-1.0, 1.0), k=(-1.0, 1.0), v=(-20.0, 20.0), g=(-9.0, -1e-6), beta=(0.0, 1.0))


def xorshift32_stream(n, seed):
    out = np.empty(n, np.uint32)
    s = np.uint32(seed)
    # vectorised in blocks is not possible (serial recurrence); plain loop on uint32
    s = int(seed) & 0xFFFFFFFF
    for i in range(n):
        s ^= (s << 13) & 0xFFFFFFFF
        s ^= s >> 17
        s ^= (s << 5) & 0xFFFFFFFF
        out[i] = s
    return out


def bounded_rand(n, lo, hi, seed):
    t = xorshift32_stream(n, seed).astype(np.float32) * np.float32(1.0 / 4294967296.0)
    return (np.float32(lo) + t * (np.float32(hi) - np.float32(lo))).astype(np.float32)


def l2norm_rows(x, eps=1e-6):
    x = x.astype(np.float32)
    nrm = np.sqrt((x.astype(np.float32) ** 2).sum(-1, dtype=np.float32, keepdims=True) + np.float32(eps))
    return (x / nrm).astype(np.float32)


def probe_inputs(heads=16, seq=104, k_dim=128, v_dim=128, full_heads=16):
    """The probe draws all 16 heads; `heads` keeps the first few of them."""
    H = full_heads
    q = bounded_rand(H * seq * k_dim, *PROBE_RANGES["q"], PROBE_SEEDS["q"]).reshape(H, seq, k_dim)
    k = bounded_rand(H * seq * k_dim, *PROBE_RANGES["k"], PROBE_SEEDS["k"]).reshape(H, seq, k_dim)
    v = bounded_rand(H * seq * v_dim, *PROBE_RANGES["v"], PROBE_SEEDS["v"]).reshape(H, seq, v_dim)
    g = bounded_rand(H * seq, *PROBE_RANGES["g"], PROBE_SEEDS["g"]).reshape(H, seq)
    b = bounded_rand(H * seq, *PROBE_RANGES["beta"], PROBE_SEEDS["beta"]).reshape(H, seq)
    q, k = l2norm_rows(q), l2norm_rows(k)
    return q[:heads].copy(), k[:heads].copy(), v[:heads].copy(), g[:heads].copy(), b[:heads].copy()


def chunk_inputs(heads, seq, k_dim=128, v_dim=128, seed=0, batch=None):
    """BASELINE configs 0/2: q,k ~ N(0,1) then L2-normalised per (head, token);
    v ~ N(0,1); g ~ U(-1,-0.01); beta ~ U(0,1). fp32, head-major [.., H, S, D]."""
    rng = np.random.default_rng(seed)
    lead = (heads,) if batch is None else (batch, heads)
    q = l2norm_rows(rng.standard_normal(lead + (seq, k_dim), dtype=np.float32))
    k = l2norm_rows(rng.standard_normal(lead + (seq, k_dim), dtype=np.float32))
    v = rng.standard_normal(lead + (seq, v_dim), dtype=np.float32)
    g = rng.uniform(-1.0, -0.01, lead + (seq,)).astype(np.float32)
    b = rng.uniform(0.0, 1.0, lead + (seq,)).astype(np.float32)
    return q, k, v, g, b


def f16bits(x):
    return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


def decode_inputs(batch, heads=16, k_dim=128, v_dim=128, ks=4, seed=0):
    """BASELINE config 1 per sequence: state ~ N(0,0.02) fp32; conv cache fp16
    (the reference's [conv_dim][4] slot layout) ~ N(0,1); conv weight ~ N(0,0.02);
    qkv ~ N(0,1); a, b ~ N(0,1); A_log ~ U(-2,1); dt_bias ~ N(0,0.1) (fp16-rounded,
    the reference reads it from fp16); z ~ N(0,1); norm weight ~ N(0,0.1) + 1."""
    rng = np.random.default_rng(seed)
    conv_dim = heads * (2 * k_dim + v_dim)
    d = dict(
        state=(rng.standard_normal((batch, heads, k_dim, v_dim), dtype=np.float32) * 0.02).astype(np.float32),
        conv_state=f16bits(rng.standard_normal((batch, conv_dim, ks), dtype=np.float32)),
        conv_w=f16bits(rng.standard_normal((conv_dim, ks), dtype=np.float32) * 0.02),
        qkv=f16bits(rng.standard_normal((batch, conv_dim), dtype=np.float32)),
        a=f16bits(rng.standard_normal((batch, heads), dtype=np.float32)),
        b=f16bits(rng.standard_normal((batch, heads), dtype=np.float32)),
        z=f16bits(rng.standard_normal((batch, heads * v_dim), dtype=np.float32)),
        norm_w=(1.0 + 0.1 * rng.standard_normal(v_dim, dtype=np.float32)).astype(np.float32),
    )
    a_log = rng.uniform(-2, 1, heads).astype(np.float32)
    dt = np.float16(rng.standard_normal(heads, dtype=np.float32) * 0.1).astype(np.float32)
    d["a_log_bias"] = np.stack([a_log, dt], 1).astype(np.float32)
    return d


def model_weights(layers=24, vocab=248320, seed=0):
    """Random-init weights in the Qwen3.5-0.8B layout under the reference's role
    names: fp16 matrices ~ N(0, 0.02), (1+w) RMSNorm weights
    w ~ N(0, 0.1) fp16, A_log ~ U(-2, 1) fp32, dt_bias ~ N(0, 0.1) fp16, conv
    weight ~ N(0, 0.02) fp16, gated-norm weight 1 + N(0, 0.1) fp32. Matrices as
    uint16 fp16 bits [out][in]."""
    rng = np.random.default_rng(seed)

    def mat(o, i, sd=0.02):
        return (rng.standard_normal((o, i), dtype=np.float32) * sd).astype(np.float16).view(np.uint16)

    def vec16(n, sd=0.1):
        return (rng.standard_normal(n, dtype=np.float32) * sd).astype(np.float16).view(np.uint16)

    w = {"embedding": mat(vocab, 1024), "final_norm": vec16(1024)}
    for i in range(layers):
        p = f"layer.{i}."
        w[p + "input_norm"] = vec16(1024)
        w[p + "post_norm"] = vec16(1024)
        w[p + "mlp_gate"] = mat(3584, 1024)
        w[p + "mlp_up"] = mat(3584, 1024)
        w[p + "mlp_down"] = mat(1024, 3584)
        if i % 4 == 3:
            w[p + "attn_q"] = mat(4096, 1024)
            w[p + "attn_k"] = mat(512, 1024)
            w[p + "attn_v"] = mat(512, 1024)
            w[p + "attn_q_norm"] = vec16(256)
            w[p + "attn_k_norm"] = vec16(256)
            w[p + "attn_o"] = mat(1024, 2048)
        else:
            w[p + "delta_in_proj_qkv"] = mat(6144, 1024)
            w[p + "delta_in_proj_z"] = mat(2048, 1024)
            w[p + "delta_in_proj_a"] = mat(16, 1024)
            w[p + "delta_in_proj_b"] = mat(16, 1024)
            w[p + "delta_conv"] = mat(6144, 4)
            w[p + "delta_norm"] = (1.0 + 0.1 * rng.standard_normal(128, dtype=np.float32)).astype(np.float32)
            w[p + "delta_a_log"] = rng.uniform(-2, 1, 16).astype(np.float32)
            w[p + "delta_dt_bias"] = vec16(16)
            w[p + "delta_out_proj"] = mat(1024, 2048)
    return w


def write_repack_artifact(path, weights, drop=(), alignment=256):
    """Writes `weights` (role -> array) as a repacked text artifact in the format
    the reference's tools/repack_text_weights.py produces and
    src/runtime/weight_loader.cpp reads: text_weights.bin with each tensor at an
    `alignment`-aligned offset, and text_repack_manifest.json listing role_path,
    offset, nbytes, dtype and shape. Roles in `drop` are left out."""
    import json
    import os
    os.makedirs(path, exist_ok=True)
    tensors, off = [], 0
    with open(os.path.join(path, "text_weights.bin"), "wb") as f:
        for role, arr in weights.items():
            if role in drop:
                continue
            arr = np.ascontiguousarray(arr)
            pad = (-off) % alignment
            f.write(b"\0" * pad)
            off += pad
            f.write(arr.tobytes())
            rp = {"embedding": "global.token_embedding", "final_norm": "global.final_norm"}.get(role, role)
            tensors.append({"role_path": rp, "name": rp, "file": "text_weights.bin", "offset": off,
                            "nbytes": int(arr.nbytes), "dtype": "fp32" if arr.dtype == np.float32 else "fp16",
                            "shape": list(arr.shape)})
            off += arr.nbytes
    manifest = {"schema_version": 1, "artifact": {"format": "spock-text-repacked-weights"},
                "packing": {"alignment": alignment, "byte_order": "little", "weights_file": "text_weights.bin"},
                "tensors": tensors}
    with open(os.path.join(path, "text_repack_manifest.json"), "w") as f:
        json.dump(manifest, f)
