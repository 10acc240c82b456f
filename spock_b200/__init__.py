"""spock_b200: B200 (sm_100a) Gated DeltaNet hot path behind a C ABI.

Host-side mirror of spock's DeltaNet entry points over libspock_b200.so
(include/spock_b200.h). PyTorch provides device memory and streams only; every
computation runs in this package's own CUDA kernels. There is no CPU fallback:
if the library or a B200 is missing, calls raise SpockError.

Reference interfaces mirrored here:
  DeltaNetChunkConfig / Inputs / Outputs, run_deltanet_chunk_rule
      src/runtime/deltanet_chunk.hpp:8-40 (same field names, layouts and the
      same "fields must be non-zero" / size-mismatch errors)
  chunk_prefill        batched device-tensor form used by
                       DecodeSession::gpu_chunk_prefill_from_gpu_collect
                       (src/runtime/vk_session.cpp:4466-4828)
  deltanet_decode_step fused conv_l2_qk + recurrent_gbeta_norm_gate
                       (src/runtime/vk_session.cpp:2878-2883, 3213-3218)
"""
import ctypes
import os
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libspock_b200.so")

SPOCK_OK = 0
SPOCK_ERR_INVALID = -1
SPOCK_ERR_UNSUPPORTED = -2
SPOCK_ERR_CUDA = -3
SPOCK_ERR_ALLOC = -4
SPOCK_ERR_TIMEOUT = -5
F32, F16, BF16 = 0, 1, 2

EXPORTED = ["spock_create", "spock_destroy", "spock_last_error", "spock_sync",
            "spock_kernel_launch_count", "spock_selftest_wait_timeout", "spock_chunk_prefill", "spock_chunk_last_to_fp16",
            "spock_deltanet_decode_step", "spock_deltanet_recurrent", "spock_chunk_prefill_noalloc",
            "spock_model_create", "spock_model_destroy", "spock_model_last_error", "spock_model_set_weight",
            "spock_model_reset", "spock_model_step", "spock_model_generate", "spock_model_load_artifact",
            "spock_model_prefill", "spock_noalloc_sync", "spock_model_sync",
            "spock_rms_norm", "spock_matvec", "spock_argmax", "spock_attention_decode", "spock_attention_prefill"]


class SpockError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class ChunkDesc(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int64), ("num_heads", ctypes.c_int64), ("seq_len", ctypes.c_int64),
                ("key_dim", ctypes.c_int64), ("value_dim", ctypes.c_int64), ("chunk_size", ctypes.c_int64),
                ("dtype_in", ctypes.c_int32), ("dtype_out", ctypes.c_int32),
                ("use_qk_l2norm", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class DnLayer(ctypes.Structure):
    _fields_ = [("num_heads", ctypes.c_int32), ("key_dim", ctypes.c_int32), ("value_dim", ctypes.c_int32),
                ("conv_kernel", ctypes.c_int32), ("conv_weight", ctypes.c_void_p),
                ("a_log_bias", ctypes.c_void_p), ("norm_weight", ctypes.c_void_p),
                ("eps", ctypes.c_float), ("reserved", ctypes.c_int32)]


_LIB = None


def build(force=False):
    from . import builder as _b
    lib_path = _b.build(force=force)
    _b.build_apps(force=force)
    return lib_path


def lib():
    """Loads libspock_b200.so (building it in-tree when absent or stale)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
        L.spock_create.argtypes = [ctypes.c_int, ctypes.POINTER(vp)]
        L.spock_destroy.argtypes = [vp]
        L.spock_last_error.argtypes = [vp]
        L.spock_last_error.restype = ctypes.c_char_p
        L.spock_sync.argtypes = [vp, vp]
        L.spock_kernel_launch_count.restype = ctypes.c_uint64
        L.spock_selftest_wait_timeout.argtypes = [vp, ctypes.c_uint32, vp]
        L.spock_chunk_prefill.argtypes = [vp, ctypes.POINTER(ChunkDesc)] + [vp] * 9
        L.spock_chunk_prefill_noalloc.argtypes = [ctypes.POINTER(ChunkDesc)] + [vp] * 9
        L.spock_noalloc_sync.argtypes = [vp]
        L.spock_rms_norm.argtypes = [vp, vp, vp, vp, i64, i32, ctypes.c_float, vp]
        L.spock_matvec.argtypes = [vp, i32, i32, vp, i32, i32, vp, i64, vp, vp, vp]
        L.spock_argmax.argtypes = [vp, vp, i64, i64, vp, vp]
        L.spock_attention_decode.argtypes = [vp, i32, vp, vp, vp, ctypes.c_float, ctypes.c_float, vp, vp, i32, i64,
                                             vp, vp]
        L.spock_attention_prefill.argtypes = [vp, i32, vp, vp, vp, ctypes.c_float, ctypes.c_float, vp, vp, i32, i64,
                                              i32, vp, vp]
        L.spock_chunk_last_to_fp16.argtypes = [vp, i64, i64, i64, i64, vp, vp, vp]
        L.spock_deltanet_decode_step.argtypes = [vp, ctypes.POINTER(DnLayer), i64] + [vp] * 9
        L.spock_deltanet_recurrent.argtypes = [vp, i64, i32, i32, i32] + [vp] * 8
        _LIB = L
    return _LIB


def _ptr(t):
    if t is None:
        return None
    import torch
    if not t.is_cuda:
        raise SpockError(SPOCK_ERR_INVALID, "expected a CUDA tensor")
    if not t.is_contiguous():
        raise SpockError(SPOCK_ERR_INVALID, "expected a contiguous tensor")
    return ctypes.c_void_p(t.data_ptr())


def _dtype_code(dt):
    import torch
    return {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}[dt]


class Context:
    """One per GPU (spock_ctx). Replaces VulkanDevice (src/runtime/vk_device.hpp:29-117)."""

    _by_device = {}

    def __init__(self, device=0):
        L = lib()
        h = ctypes.c_void_p()
        rc = L.spock_create(int(device), ctypes.byref(h))
        if rc != SPOCK_OK:
            raise SpockError(rc, L.spock_last_error(None).decode())
        self.h = h
        self.device = device

    @classmethod
    def get(cls, device=0):
        if device not in cls._by_device:
            cls._by_device[device] = Context(device)
        return cls._by_device[device]

    def check(self, rc):
        if rc != SPOCK_OK:
            raise SpockError(rc, lib().spock_last_error(self.h).decode())

    def sync(self, stream=None):
        self.check(lib().spock_sync(self.h, _stream(stream)))

    def selftest_wait_timeout(self, polls=256, stream=None):
        """Launches the failure-detection self-test (a bounded device wait that
        must give up); the following sync() raises SpockError(SPOCK_ERR_TIMEOUT)."""
        self.check(lib().spock_selftest_wait_timeout(self.h, int(polls), _stream(stream)))

    def close(self):
        if self.h:
            lib().spock_destroy(self.h)
            self.h = None


def _stream(stream):
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


def chunk_prefill(q, k, v, g, beta, initial_state=None, out_dtype=None, use_qk_l2norm=False,
                  chunk_size=64, out=None, final_state=None, ctx=None, stream=None):
    """Batched chunked gated delta rule on device tensors.

    q, k [B,H,S,K] and v [B,H,S,V] (fp32/fp16/bf16, same dtype); g, beta [B,H,S]
    fp32; initial_state [B,H,K,V] fp32 or None. Returns (core_attn_out [B,H,S,V]
    in out_dtype (default: q's dtype), final_state [B,H,K,V] fp32).
    """
    import torch
    B, H, S, K = q.shape
    V = v.shape[-1]
    out_dtype = out_dtype or q.dtype
    ctx = ctx or Context.get(q.device.index or 0)
    if out is None:
        out = torch.empty((B, H, S, V), dtype=out_dtype, device=q.device)
    if final_state is None:
        final_state = torch.empty((B, H, K, V), dtype=torch.float32, device=q.device)
    d = ChunkDesc(B, H, S, K, V, chunk_size, _dtype_code(q.dtype), _dtype_code(out_dtype),
                  int(bool(use_qk_l2norm)), 0)
    ctx.check(lib().spock_chunk_prefill(ctx.h, ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v), _ptr(g),
                                        _ptr(beta), _ptr(initial_state), _ptr(out), _ptr(final_state),
                                        _stream(stream)))
    return out, final_state


def chunk_last_to_fp16(core_out, ctx=None, stream=None):
    """Last token of core_attn_out [B,H,S,V] fp32 -> fp16 [B,H*V] by truncation (FTZ)."""
    import torch
    B, H, S, V = core_out.shape
    ctx = ctx or Context.get(core_out.device.index or 0)
    out = torch.empty((B, H * V), dtype=torch.float16, device=core_out.device)
    ctx.check(lib().spock_chunk_last_to_fp16(ctx.h, B, H, S, V, _ptr(core_out), _ptr(out), _stream(stream)))
    return out


MV_STORE, MV_RESIDUAL, MV_SILU_GATE, MV_ARGMAX = 0, 1, 2, 3


def rms_norm(x, w, eps=1e-6, out=None, ctx=None, stream=None):
    """rms_norm.comp on fp16 rows x [rows, 1024] with (1+w) weights w [1024] fp16."""
    import torch
    ctx = ctx or Context.get(x.device.index or 0)
    out = torch.empty_like(x) if out is None else out
    ctx.check(lib().spock_rms_norm(ctx.h, _ptr(x), _ptr(w), _ptr(out), x.shape[0], x.shape[1], eps, _stream(stream)))
    return out


def matvec(w, x, epilogue=MV_STORE, residual=None, exact=False, out=None, ctx=None, stream=None):
    """matvec.comp over rows x [rows, in] with fp16 W [out(, x2 for SILU_GATE), in] and a fused epilogue;
    ARGMAX returns int32 token ids [rows]."""
    import torch
    ctx = ctx or Context.get(x.device.index or 0)
    rows, n_in = x.shape
    n_out = w.shape[0] // 2 if epilogue == MV_SILU_GATE else w.shape[0]
    if out is None:
        out = (torch.empty(rows, dtype=torch.int32, device=x.device) if epilogue == MV_ARGMAX
               else torch.empty((rows, n_out), dtype=torch.float16, device=x.device))
    ctx.check(lib().spock_matvec(ctx.h, int(epilogue), int(bool(exact)), _ptr(w), n_out, n_in, _ptr(x), rows,
                                 _ptr(out), _ptr(residual), _stream(stream)))
    return out


def argmax(logits, ctx=None, stream=None):
    """argmax.comp per row of fp16 logits [rows, n] -> int32 [rows] (lowest index among ties)."""
    import torch
    ctx = ctx or Context.get(logits.device.index or 0)
    out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    ctx.check(lib().spock_argmax(ctx.h, _ptr(logits), logits.shape[0], logits.shape[1], _ptr(out), _stream(stream)))
    return out


def attention_decode(proj, q_norm, k_norm, pos, kv_cache, eps=1e-6, theta=1e7, exact=False, ctx=None, stream=None):
    """One gated-attention decode token per sequence: proj [rows, 5120] fp16, pos int32 [rows],
    kv_cache [rows, max_seq, 2, 2, 256] fp16 (row pos written) -> out [rows, 2048] fp16."""
    import torch
    ctx = ctx or Context.get(proj.device.index or 0)
    rows = proj.shape[0]
    out = torch.empty((rows, 2048), dtype=torch.float16, device=proj.device)
    ctx.check(lib().spock_attention_decode(ctx.h, int(bool(exact)), _ptr(proj), _ptr(q_norm), _ptr(k_norm), eps, theta,
                                           _ptr(pos), _ptr(kv_cache), kv_cache.shape[1], rows, _ptr(out),
                                           _stream(stream)))
    return out


def attention_prefill(proj, q_norm, k_norm, pos, kv_cache, eps=1e-6, theta=1e7, exact=False, ctx=None, stream=None):
    """Gated attention over `len` prompt tokens per sequence: proj [batch, len, 5120] fp16, pos int32 [batch]
    (first prompt position), kv_cache [batch, max_seq, 2, 2, 256] fp16 -> out [batch, len, 2048] fp16."""
    import torch
    ctx = ctx or Context.get(proj.device.index or 0)
    B, T = proj.shape[0], proj.shape[1]
    out = torch.empty((B, T, 2048), dtype=torch.float16, device=proj.device)
    ctx.check(lib().spock_attention_prefill(ctx.h, int(bool(exact)), _ptr(proj), _ptr(q_norm), _ptr(k_norm), eps,
                                            theta, _ptr(pos), _ptr(kv_cache), kv_cache.shape[1], B, T, _ptr(out),
                                            _stream(stream)))
    return out


@dataclass
class DeltaNetLayer:
    """Per-layer constants (spock_dn_layer). Tensors are device tensors."""
    conv_weight: object   # fp16 [conv_dim, conv_kernel]
    a_log_bias: object    # fp32 [num_heads, 2]
    norm_weight: object   # fp32 [value_dim]
    num_heads: int = 16
    key_dim: int = 128
    value_dim: int = 128
    conv_kernel: int = 4
    eps: float = 1e-6

    def c_struct(self):
        return DnLayer(self.num_heads, self.key_dim, self.value_dim, self.conv_kernel,
                       _ptr(self.conv_weight), _ptr(self.a_log_bias), _ptr(self.norm_weight),
                       self.eps, 0)


def deltanet_decode_step(layer, qkv, conv_state, state, a, b, z, out=None, core_raw=None, ctx=None,
                         stream=None):
    """One decode token through a DeltaNet mixer core; qkv, conv_state, state updated in place."""
    import torch
    B = qkv.shape[0]
    ctx = ctx or Context.get(qkv.device.index or 0)
    if out is None:
        out = torch.empty((B, layer.num_heads * layer.value_dim), dtype=torch.float16, device=qkv.device)
    st = layer.c_struct()
    ctx.check(lib().spock_deltanet_decode_step(ctx.h, ctypes.byref(st), B, _ptr(qkv), _ptr(conv_state),
                                               _ptr(state), _ptr(a), _ptr(b), _ptr(z), _ptr(out),
                                               _ptr(core_raw), _stream(stream)))
    return out


def deltanet_recurrent(q, k, v, g, beta, state, num_heads=16, key_dim=128, value_dim=128, ctx=None,
                       stream=None):
    """Unfused recurrent update (deltanet_recurrent.comp contract); state updated in place."""
    import torch
    B = q.shape[0]
    ctx = ctx or Context.get(q.device.index or 0)
    out = torch.empty((B, num_heads * value_dim), dtype=torch.float16, device=q.device)
    ctx.check(lib().spock_deltanet_recurrent(ctx.h, B, num_heads, key_dim, value_dim, _ptr(q), _ptr(k),
                                             _ptr(v), _ptr(g), _ptr(beta), _ptr(state), _ptr(out),
                                             _stream(stream)))
    return out


# ---- reference-shaped API (host vectors in, host vectors out) ----------------

@dataclass
class DeltaNetChunkConfig:
    num_heads: int = 0
    sequence_length: int = 0
    key_dim: int = 0
    value_dim: int = 0
    chunk_size: int = 64
    use_qk_l2norm: bool = True


@dataclass
class DeltaNetChunkInputs:
    query: List[float] = field(default_factory=list)   # [head][token][dim]
    key: List[float] = field(default_factory=list)
    value: List[float] = field(default_factory=list)
    g: List[float] = field(default_factory=list)       # [head][token]
    beta: List[float] = field(default_factory=list)
    initial_state: List[float] = field(default_factory=list)  # [head][key][value] or empty


@dataclass
class DeltaNetChunkOutputs:
    core_attn_out: np.ndarray = None   # flat [head][token][value]
    final_state: np.ndarray = None     # flat [head][key][value]


def run_deltanet_chunk_rule(config: DeltaNetChunkConfig, inputs: DeltaNetChunkInputs,
                            device=0) -> DeltaNetChunkOutputs:
    """Drop-in for spock::runtime::run_deltanet_chunk_rule on the GPU (fp32 in, fp32 out)."""
    import torch
    c = config
    if min(c.num_heads, c.sequence_length, c.key_dim, c.value_dim, c.chunk_size) <= 0:
        raise SpockError(SPOCK_ERR_INVALID, "DeltaNet chunk config fields must be non-zero")
    H, S, K, V = c.num_heads, c.sequence_length, c.key_dim, c.value_dim

    def checked(x, n, name):
        a = np.asarray(x, dtype=np.float32).reshape(-1)
        if a.size != n:
            raise SpockError(SPOCK_ERR_INVALID, f"{name} size mismatch: expected {n}, got {a.size}")
        return a

    dev = torch.device("cuda", device)
    t = lambda a, shape: torch.from_numpy(a.reshape(shape)).to(dev)
    q = t(checked(inputs.query, H * S * K, "query"), (1, H, S, K))
    k = t(checked(inputs.key, H * S * K, "key"), (1, H, S, K))
    v = t(checked(inputs.value, H * S * V, "value"), (1, H, S, V))
    g = t(checked(inputs.g, H * S, "g"), (1, H, S))
    b = t(checked(inputs.beta, H * S, "beta"), (1, H, S))
    init = None
    if len(inputs.initial_state):
        init = t(checked(inputs.initial_state, H * K * V, "initial_state"), (1, H, K, V))
    out, st = chunk_prefill(q, k, v, g, b, initial_state=init, out_dtype=torch.float32,
                            use_qk_l2norm=c.use_qk_l2norm, chunk_size=c.chunk_size)
    return DeltaNetChunkOutputs(out.reshape(-1).cpu().numpy(), st.reshape(-1).cpu().numpy())


# ---- full-model decode session ------------------------------------------------

class ModelDesc(ctypes.Structure):
    _fields_ = [("num_layers", ctypes.c_int32), ("vocab", ctypes.c_int32), ("max_batch", ctypes.c_int32),
                ("max_seq", ctypes.c_int32), ("rms_eps", ctypes.c_float), ("rope_theta", ctypes.c_float),
                ("exact", ctypes.c_int32), ("reserved", ctypes.c_int32)]


def _model_lib():
    L = lib()
    if not getattr(L, "_model_types", False):
        vp = ctypes.c_void_p
        L.spock_model_create.argtypes = [vp, ctypes.POINTER(ModelDesc), ctypes.POINTER(vp)]
        L.spock_model_destroy.argtypes = [vp]
        L.spock_model_last_error.argtypes = [vp]
        L.spock_model_last_error.restype = ctypes.c_char_p
        L.spock_model_set_weight.argtypes = [vp, ctypes.c_char_p, vp, ctypes.c_size_t]
        L.spock_model_load_artifact.argtypes = [vp, ctypes.c_char_p]
        L.spock_model_reset.argtypes = [vp, ctypes.c_int32]
        L.spock_model_step.argtypes = [vp, vp, vp, vp, vp]
        L.spock_model_generate.argtypes = [vp, vp, ctypes.c_int32, ctypes.c_int32, vp, vp]
        L.spock_model_prefill.argtypes = [vp, vp, ctypes.c_int32, vp, vp, vp]
        L.spock_model_sync.argtypes = [vp, vp]
        L._model_types = True
    return L


class Model:
    """Qwen3.5-0.8B-layout decode session on one GPU (spock_model): the B200
    form of DecodeSession (src/runtime/vk_session.hpp:22-46) for a batch of
    independent sequences. Weights are uploaded by the reference's role names."""

    def __init__(self, num_layers=24, vocab=248320, max_batch=1, max_seq=2048, eps=1e-6, theta=1e7,
                 ctx=None, device=0, exact=False):
        self.L = _model_lib()
        self.ctx = ctx or Context.get(device)
        self.device = device
        self.exact = bool(exact)
        d = ModelDesc(num_layers, vocab, max_batch, max_seq, eps, theta, int(bool(exact)), 0)
        h = ctypes.c_void_p()
        rc = self.L.spock_model_create(self.ctx.h, ctypes.byref(d), ctypes.byref(h))
        if rc != SPOCK_OK:
            raise SpockError(rc, "spock_model_create failed")
        self.h = h
        self.max_batch = max_batch

    def _check(self, rc):
        if rc != SPOCK_OK:
            raise SpockError(rc, self.L.spock_model_last_error(self.h).decode())

    def set_weights(self, weights):
        for role, arr in weights.items():
            arr = np.ascontiguousarray(arr)
            self._check(self.L.spock_model_set_weight(self.h, role.encode(), arr.ctypes.data, arr.nbytes))

    def load_artifact(self, repack_dir):
        """Loads a repacked text artifact (text_repack_manifest.json + text_weights.bin)."""
        self._check(self.L.spock_model_load_artifact(self.h, os.fsencode(repack_dir)))

    def sync(self, stream=None):
        """Waits for the stream; raises SpockError(SPOCK_ERR_TIMEOUT) when one of this
        model's kernels reported a bounded wait that gave up (spock_model_sync)."""
        self._check(self.L.spock_model_sync(self.h, _stream(stream)))

    def reset(self, batch):
        self.batch = batch
        self._check(self.L.spock_model_reset(self.h, batch))

    def step(self, tokens, stream=None):
        """tokens: int32 CUDA tensor [batch] -> (next tokens [batch], final-normed hidden fp16 [batch,1024])."""
        import torch
        out = torch.empty_like(tokens)
        hid = torch.empty((tokens.shape[0], 1024), dtype=torch.float16, device=tokens.device)
        self._check(self.L.spock_model_step(self.h, _ptr(tokens), _ptr(out), _ptr(hid), _stream(stream)))
        return out, hid

    def prefill(self, prompt, stream=None):
        """prompt: int32 CUDA tensor [batch, len] -> (next tokens [batch], final-normed hidden of the
        last prompt token fp16 [batch, 1024]). Layer-major: every layer over the whole prompt."""
        import torch
        prompt = prompt.contiguous()
        out = torch.empty((prompt.shape[0],), dtype=torch.int32, device=prompt.device)
        hid = torch.empty((prompt.shape[0], 1024), dtype=torch.float16, device=prompt.device)
        self._check(self.L.spock_model_prefill(self.h, _ptr(prompt), prompt.shape[1], _ptr(out), _ptr(hid),
                                               _stream(stream)))
        return out, hid

    def generate(self, prompt, n_new, stream=None):
        """prompt: int32 CUDA tensor [batch, len] -> greedy tokens [batch, n_new] (layer-major prefill,
        then graph-replayed decode steps)."""
        import torch
        out = torch.empty((prompt.shape[0], n_new), dtype=torch.int32, device=prompt.device)
        self._check(self.L.spock_model_generate(self.h, _ptr(prompt), prompt.shape[1], n_new, _ptr(out),
                                                _stream(stream)))
        return out

    def close(self):
        if self.h:
            self.L.spock_model_destroy(self.h)
            self.h = None
