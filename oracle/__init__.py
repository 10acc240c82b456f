"""ctypes bindings for the CPU oracle (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm import this package; the product library (spock_b200) never does.

  liboracle.so          restatement of the reference algorithms (oracle/*.cpp)
  _ref/libref_chunk.so  the reference's own run_deltanet_chunk_rule
                        (src/runtime/deltanet_chunk.cpp), built from its sources
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_i64 = ctypes.c_int64


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _ptr(a, t):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(t)


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        _LIB = ctypes.CDLL(path)
        _LIB.oracle_chunk_rule.restype = ctypes.c_int
        _LIB.oracle_chunk_rule.argtypes = [_i64] * 5 + [ctypes.c_int] + [_f32p] * 8 + [ctypes.c_int]
        _LIB.oracle_conv_l2_qk.argtypes = [ctypes.c_int] * 5 + [_u16p, _u16p, _u16p, ctypes.c_int]
        _LIB.oracle_rec_norm_gate.argtypes = [ctypes.c_int] * 4 + [ctypes.c_float] * 2 + [
            _u16p, _u16p, _f32p, _u16p, _f32p, _u16p, _f32p, _u16p, ctypes.c_int]
        vp = ctypes.c_void_p
        _LIB.oracle_model_create.restype = vp
        _LIB.oracle_model_create.argtypes = [ctypes.c_int] * 3 + [ctypes.c_float] * 2
        _LIB.oracle_model_destroy.argtypes = [vp]
        _LIB.oracle_model_set.argtypes = [vp, ctypes.c_char_p, vp]
        _LIB.oracle_model_reset.argtypes = [vp, ctypes.c_int]
        _LIB.oracle_model_step.argtypes = [vp, vp, vp, vp, vp, ctypes.c_int]
        _LIB.oracle_recurrent_raw.argtypes = [ctypes.c_int] * 3 + [ctypes.c_float] + [
            _u16p, _u16p, _u16p, _f32p, _u16p]
        _LIB.oracle_silu_gate.argtypes = [_i64, _u16p, _u16p, _u16p]
        _LIB.oracle_matvec.argtypes = [_u16p, _u16p, ctypes.c_int, ctypes.c_int, _u16p, ctypes.c_int]
        _LIB.oracle_rms_norm.argtypes = [_u16p, _u16p, ctypes.c_float, _u16p]
        _LIB.oracle_argmax.argtypes = [_u16p, ctypes.c_int]
        _LIB.oracle_argmax.restype = ctypes.c_int
        _LIB.oracle_attention_decode.argtypes = [_u16p, _u16p, _u16p, ctypes.c_float, ctypes.c_float, _u16p,
                                                 ctypes.c_int, _u16p]
        _LIB.oracle_residual_add.argtypes = [_i64, _u16p, _u16p, _u16p]
        _LIB.oracle_gbeta.argtypes = [ctypes.c_int, _u16p, _u16p, _f32p, _f32p, _f32p]
    return _LIB


def ref_lib():
    """The reference's own chunk rule, or None when it was never built."""
    global _REF
    if _REF is None:
        path = os.path.join(HERE, "_ref", "libref_chunk.so")
        if not os.path.exists(path):
            try:
                build()
            except Exception:
                pass
        if not os.path.exists(path):
            return None
        _REF = ctypes.CDLL(path)
        _REF.ref_chunk_rule.restype = ctypes.c_int
        _REF.ref_chunk_rule.argtypes = [_i64] * 5 + [ctypes.c_int] + [_f32p] * 8
        _REF.ref_chunk_rule_batched.restype = ctypes.c_int
        _REF.ref_chunk_rule_batched.argtypes = [_i64] * 6 + [_f32p] * 7 + [ctypes.c_int]
    return _REF


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def chunk_rule(q, k, v, g, beta, chunk_size=64, use_qk_l2norm=False, initial_state=None,
               threads=1, use_reference=False):
    """q,k [H,S,K], v [H,S,V], g,beta [H,S] -> (core_attn_out [H,S,V], final_state [H,K,V])."""
    q, k, v, g, beta = map(_f32, (q, k, v, g, beta))
    H, S, K = q.shape
    V = v.shape[2]
    init = None if initial_state is None else _f32(initial_state)
    out = np.zeros((H, S, V), np.float32)
    st = np.zeros((H, K, V), np.float32)
    args = [H, S, K, V, chunk_size, int(use_qk_l2norm)] + [
        _ptr(x, _f32p) for x in (q, k, v, g, beta)] + [_ptr(init, _f32p), _ptr(out, _f32p), _ptr(st, _f32p)]
    if use_reference:
        r = ref_lib()
        if r is None:
            raise RuntimeError("reference chunk rule not built (oracle/_ref)")
        rc = r.ref_chunk_rule(*args)
    else:
        rc = lib().oracle_chunk_rule(*(args + [threads]))
    if rc != 0:
        raise RuntimeError("chunk rule rejected its inputs")
    return out, st


def conv_l2_qk(qkv, conv_state, conv_w, num_heads=16, key_dim=128, threads=1):
    """In-place on copies. qkv [B,conv_dim] u16 (fp16 bits), conv_state [B,conv_dim,ks]."""
    qkv = np.ascontiguousarray(qkv, np.uint16).copy()
    cs = np.ascontiguousarray(conv_state, np.uint16).copy()
    w = np.ascontiguousarray(conv_w, np.uint16)
    B, D = qkv.shape
    ks = cs.shape[2]
    rc = lib().oracle_conv_l2_qk(B, D, ks, num_heads * key_dim, num_heads, _ptr(qkv, _u16p),
                                 _ptr(cs, _u16p), _ptr(w, _u16p), threads)
    assert rc == 0
    return qkv, cs


def rec_norm_gate(qkv, state, a, b, a_log_bias, z, norm_w, num_heads=16, k_dim=128, v_dim=128,
                  eps=1e-6, threads=1):
    """qkv [B,conv_dim] (post conv/L2) u16; state [B,H,K,V] f32 (copied); a,b [B,H] u16;
    a_log_bias [H,2] f32; z [B,H*V] u16; norm_w [V] f32 -> (out [B,H*V] u16, new state)."""
    qkv = np.ascontiguousarray(qkv, np.uint16)
    st = _f32(state).copy()
    a = np.ascontiguousarray(a, np.uint16)
    b = np.ascontiguousarray(b, np.uint16)
    alb = _f32(a_log_bias)
    z = np.ascontiguousarray(z, np.uint16)
    w = _f32(norm_w)
    B = qkv.shape[0]
    out = np.zeros((B, num_heads * v_dim), np.uint16)
    rc = lib().oracle_rec_norm_gate(B, num_heads, k_dim, v_dim, 1.0 / np.sqrt(np.float32(k_dim)),
                                    eps, _ptr(a, _u16p), _ptr(b, _u16p), _ptr(alb, _f32p),
                                    _ptr(qkv, _u16p), _ptr(st, _f32p), _ptr(z, _u16p),
                                    _ptr(w, _f32p), _ptr(out, _u16p), threads)
    assert rc == 0
    return out, st


def recurrent_raw(q, k, v, state_with_tail, num_heads=16, k_dim=128, v_dim=128):
    q, k, v = (np.ascontiguousarray(x, np.uint16) for x in (q, k, v))
    st = _f32(state_with_tail).copy()
    out = np.zeros(num_heads * v_dim, np.uint16)
    lib().oracle_recurrent_raw(num_heads, k_dim, v_dim, float(np.float32(1.0) / np.sqrt(np.float32(k_dim))),
                               _ptr(q, _u16p), _ptr(k, _u16p), _ptr(v, _u16p), _ptr(st, _f32p),
                               _ptr(out, _u16p))
    return out, st


def _u16(a):
    return np.ascontiguousarray(a, dtype=np.uint16)


def matvec(W, x, threads=8):
    """matvec.comp: fp16 W [out][in] (bits) times fp16 x [in] -> fp16 [out], each dot sequential."""
    W, x = _u16(W), _u16(x)
    out = np.zeros(W.shape[0], np.uint16)
    lib().oracle_matvec(_ptr(W, _u16p), _ptr(x, _u16p), W.shape[0], W.shape[1], _ptr(out, _u16p), threads)
    return out


def rms_norm(x, w, eps=1e-6):
    """rms_norm.comp on one 1024-wide fp16 row (bits)."""
    x, w = _u16(x), _u16(w)
    y = np.zeros(1024, np.uint16)
    lib().oracle_rms_norm(_ptr(x, _u16p), _ptr(w, _u16p), eps, _ptr(y, _u16p))
    return y


def argmax(logits):
    """argmax.comp on fp16 logits (bits): lowest index among equal maxima."""
    logits = _u16(logits)
    return int(lib().oracle_argmax(_ptr(logits, _u16p), logits.size))


def attention_decode(proj, q_norm, k_norm, cache, pos, eps=1e-6, theta=1e7):
    """One gated-attention token of one sequence: proj [5120], cache [max_seq, 2, 2, 256]
    (a copy; row pos written) -> (gated [2048], updated cache). All fp16 bits."""
    proj, qn, kn = _u16(proj), _u16(q_norm), _u16(k_norm)
    cache = _u16(cache).copy()
    out = np.zeros(2048, np.uint16)
    lib().oracle_attention_decode(_ptr(proj, _u16p), _ptr(qn, _u16p), _ptr(kn, _u16p), eps, theta,
                                  _ptr(cache, _u16p), int(pos), _ptr(out, _u16p))
    return out, cache


def silu_gate(gate, up):
    """silu_gate.comp: fp16 bits in, fp16 bits out."""
    gate, up = _u16(gate), _u16(up)
    out = np.zeros_like(gate)
    lib().oracle_silu_gate(gate.size, _ptr(gate, _u16p), _ptr(up, _u16p), _ptr(out, _u16p))
    return out


def residual_add(a, b):
    """residual_add.comp: fp16(a + b) on fp16 bits."""
    a, b = _u16(a), _u16(b)
    out = np.zeros_like(a)
    lib().oracle_residual_add(a.size, _ptr(a, _u16p), _ptr(b, _u16p), _ptr(out, _u16p))
    return out


def gbeta(a, b, a_log_bias):
    """Phase 1 of deltanet_recurrent_gbeta_norm_gate.comp: (g [H], beta [H]) fp32."""
    a, b = _u16(a), _u16(b)
    alb = _f32(a_log_bias)
    H = a.size
    g = np.zeros(H, np.float32)
    beta = np.zeros(H, np.float32)
    lib().oracle_gbeta(H, _ptr(a, _u16p), _ptr(b, _u16p), _ptr(alb, _f32p), _ptr(g, _f32p), _ptr(beta, _f32p))
    return g, beta


class Model:
    """CPU restatement of one full-model decode step (oracle/model.cpp).
    `weights` maps reference role names to numpy arrays (kept alive here)."""

    def __init__(self, weights, layers, vocab, max_seq, eps=1e-6, theta=1e7):
        self.L = lib()
        self.h = self.L.oracle_model_create(layers, vocab, max_seq, eps, theta)
        self.keep = {}
        for role, arr in weights.items():
            arr = np.ascontiguousarray(arr)
            self.keep[role] = arr
            self.L.oracle_model_set(self.h, role.encode(), arr.ctypes.data)

    def reset(self, batch):
        self.batch = batch
        self.L.oracle_model_reset(self.h, batch)

    def step(self, tokens, threads=8):
        tok = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(self.batch, np.int32)
        hid = np.zeros((self.batch, 1024), np.uint16)
        margin = np.zeros(self.batch, np.float32)
        rc = self.L.oracle_model_step(self.h, tok.ctypes.data, out.ctypes.data, hid.ctypes.data,
                                      margin.ctypes.data, threads)
        assert rc == 0
        return out, hid, margin

    def __del__(self):
        try:
            self.L.oracle_model_destroy(self.h)
        except Exception:
            pass
