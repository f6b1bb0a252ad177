"""Test infrastructure — NOT part of the product.

ctypes bindings for the CPU checker libraries:
  * oracle/liboracle.so         — the FP64 restatement (oracle.h), always built;
  * oracle/_ref/libwelvet_ref.so — the reference's own MHA host code, codecs and
    soft-double shaders compiled for the CPU (built only where the reference
    sources are present; absent on GPU boxes unless shipped prebuilt).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs
import this module.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libwelvet_ref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


class OracleCfg(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "d_model", "num_heads", "num_kv_heads", "head_dim", "max_seq_len",
        "mask", "pos", "softmax", "window", "prefix_len", "window_causal")] + [
        ("rope_theta", C.c_double), ("scale_override", C.c_double),
        ("per_sequence", C.c_int32)]


@dataclass
class MhaCfg:
    """Python view of welvet::mha::Config (include/welvet/mha.hpp:39-64)."""
    d_model: int
    num_heads: int
    num_kv_heads: int = 0
    head_dim: int = 0
    max_seq_len: int = 0
    mask: int = 1
    pos: int = 0
    softmax: int = 0
    window: int = 0
    prefix_len: int = 0
    window_causal: int = 1
    rope_theta: float = 10000.0
    scale_override: float = 0.0
    per_sequence: int = 0

    def resolved(self) -> "MhaCfg":
        """Defaults of validate() (src/layers/mha/mha.cpp:63-94)."""
        c = MhaCfg(**self.__dict__)
        if c.head_dim <= 0:
            c.head_dim = c.d_model // c.num_heads
        if c.num_kv_heads <= 0:
            c.num_kv_heads = c.num_heads
        if c.max_seq_len <= 0:
            c.max_seq_len = 512
        if c.mask == 0:
            c.mask = 1
        if c.rope_theta <= 0:
            c.rope_theta = 10000.0
        return c

    @property
    def q_dim(self) -> int:
        r = self.resolved()
        return r.num_heads * r.head_dim

    @property
    def kv_dim(self) -> int:
        r = self.resolved()
        return r.num_kv_heads * r.head_dim

    def to_c(self) -> OracleCfg:
        return OracleCfg(**self.__dict__)


class RefStatusC(C.Structure):
    _fields_ = [("code", C.c_int32), ("message", C.c_char * 256)]


def _load_oracle():
    lib = C.CDLL(ORACLE_SO)
    cfgp = C.POINTER(OracleCfg)
    lib.oracle_dense.argtypes = [_f32p, _f32p, _f32p, C.c_int64, C.c_int64, C.c_int64, C.c_int32]
    lib.oracle_attention.argtypes = [cfgp, C.c_int32, C.c_int32, _f32p, _f32p, _f32p, _f32p, C.c_int32]
    lib.oracle_attention.restype = C.c_int32
    lib.oracle_mha_forward.argtypes = [cfgp, C.c_int32, C.c_int32] + [_f32p] * 7 + [C.c_void_p] * 3 + [C.c_int32]
    lib.oracle_mha_forward.restype = C.c_int32
    lib.oracle_mha_decode.argtypes = [cfgp, C.c_int32, _i32p, C.c_int64, _f32p, _f32p] + [_f32p] * 7 + [C.c_void_p] * 2 + [C.c_int32]
    lib.oracle_mha_decode.restype = C.c_int32
    lib.oracle_mha_validate.argtypes = [cfgp, C.c_char_p, C.c_int32]
    lib.oracle_mha_validate.restype = C.c_int32
    lib.oracle_encode.argtypes = [C.c_int32, _f32p, C.c_int64, _u8p, C.POINTER(C.c_float)]
    lib.oracle_encode.restype = C.c_int64
    lib.oracle_decode.argtypes = [C.c_int32, _u8p, C.c_int64, C.c_float, _f32p]
    lib.oracle_roundtrip.argtypes = [C.c_int32, _f32p, C.c_int64, _f32p]
    lib.oracle_roundtrip.restype = C.c_int32
    lib.oracle_decode.restype = C.c_int32
    for name, a, r in (("oracle_bf16_encode", C.c_float, C.c_uint16), ("oracle_bf16_decode", C.c_uint16, C.c_float),
                       ("oracle_f16_encode", C.c_float, C.c_uint16), ("oracle_f16_decode", C.c_uint16, C.c_float),
                       ("oracle_e4m3_encode", C.c_float, C.c_uint8), ("oracle_e4m3_decode", C.c_uint8, C.c_float),
                       ("oracle_e5m2_encode", C.c_float, C.c_uint8), ("oracle_e5m2_decode", C.c_uint8, C.c_float),
                       ("oracle_nf4_level", C.c_int32, C.c_float)):
        f = getattr(lib, name)
        f.argtypes = [a]
        f.restype = r
    lib.oracle_fp8_rowscale_encode.argtypes = [_f32p, C.c_int64, C.c_int64, _u8p, _f32p]
    lib.oracle_fp8_rowscale_decode.argtypes = [_u8p, _f32p, C.c_int64, C.c_int64, _f32p]
    lib.oracle_nf4_block_encode.argtypes = [_f32p, C.c_int64, C.c_int32, _u8p, _f32p]
    lib.oracle_nf4_block_decode.argtypes = [_u8p, _f32p, C.c_int64, C.c_int32, _f32p]
    lib.oracle_mha_normalbp.argtypes = [cfgp, C.c_int32, C.c_int32] + [_f32p] * 6 + [C.c_int32, C.c_double,
                                        C.c_int32] + [_f32p] * 5 + [C.POINTER(C.c_double), C.c_int32]
    lib.oracle_mha_normalbp.restype = C.c_int32
    lib.oracle_act_value.argtypes = [C.c_float, C.c_int32]
    lib.oracle_act_value.restype = C.c_float
    lib.oracle_norm_forward.argtypes = [C.c_int32, C.c_int64, C.c_int32, C.c_double, _f32p, _f32p, _f32p,
                                        _f32p, _f32p]
    lib.oracle_norm_forward.restype = C.c_int32
    lib.oracle_swiglu_forward.argtypes = [C.c_int64, C.c_int32, C.c_int32] + [_f32p] * 6 + [C.c_int32]
    lib.oracle_swiglu_forward.restype = C.c_int32
    lib.oracle_embedding_forward.argtypes = [C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _f32p,
                                             _f32p, _f32p, _f32p]
    lib.oracle_embedding_forward.restype = C.c_int32
    return lib


_ORACLE = None
_REF = None


def oracle_lib():
    global _ORACLE
    if _ORACLE is None:
        _ORACLE = _load_oracle()
    return _ORACLE


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref_lib():
    global _REF
    if _REF is None:
        lib = C.CDLL(REF_SO)
        lib.ref_mha_forward_f32.argtypes = [C.c_int32] * 11 + [_f32p] * 5 + [_f32p, _f32p]
        lib.ref_mha_forward_f32.restype = RefStatusC
        lib.ref_mha_forward_cfg.argtypes = [C.c_int32] * 13 + [C.c_double, C.c_double, C.c_int32] + [_f32p] * 7
        lib.ref_mha_forward_cfg.restype = RefStatusC
        lib.ref_weight_roundtrip.argtypes = [C.c_int32, C.c_int32, C.c_int32, _f32p, _u8p,
                                             C.POINTER(C.c_int64), C.POINTER(C.c_float), _f32p]
        lib.ref_weight_roundtrip.restype = RefStatusC
        lib.ref_mha_normalbp_f32.argtypes = [C.c_int32] * 10 + [_f32p] * 6 + [C.c_int32, C.c_double] + \
            [_f32p] * 5 + [C.POINTER(C.c_double)]
        lib.ref_mha_normalbp_f32.restype = RefStatusC
        lib.ref_swiglu_forward_f32.argtypes = [C.c_int32] * 5 + [_f32p] * 6
        lib.ref_swiglu_forward_f32.restype = RefStatusC
        lib.ref_rmsnorm_forward_f32.argtypes = [C.c_int32] * 3 + [C.c_double, C.c_int32] + [_f32p] * 4
        lib.ref_rmsnorm_forward_f32.restype = RefStatusC
        lib.ref_layernorm_forward_f32.argtypes = [C.c_int32] * 3 + [C.c_double, C.c_int32] + [_f32p] * 5
        lib.ref_layernorm_forward_f32.restype = RefStatusC
        lib.ref_embedding_forward_f32.argtypes = [C.c_int32] * 8 + [_f32p] * 4
        lib.ref_embedding_forward_f32.restype = RefStatusC
        for name, a, r in (("ref_fp8e4m3_encode", C.c_float, C.c_uint8), ("ref_fp8e4m3_decode", C.c_uint8, C.c_float),
                           ("ref_fp8e5m2_encode", C.c_float, C.c_uint8), ("ref_fp8e5m2_decode", C.c_uint8, C.c_float),
                           ("ref_bf16_encode", C.c_float, C.c_uint16), ("ref_bf16_decode", C.c_uint16, C.c_float),
                           ("ref_f16_encode", C.c_float, C.c_uint16), ("ref_f16_decode", C.c_uint16, C.c_float)):
            f = getattr(lib, name)
            f.argtypes = [a]
            f.restype = r
        _REF = lib
    return _REF


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------- oracle calls
def dense(x, W, threads: int = 0) -> np.ndarray:
    x, W = _f32(x), _f32(W)
    M, K = x.shape
    N = W.shape[0]
    y = np.empty((M, N), np.float32)
    oracle_lib().oracle_dense(x, W, y, M, K, N, threads)
    return y


def attention(cfg: MhaCfg, batch: int, seq: int, q, k, v, threads: int = 0) -> np.ndarray:
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty((batch * seq, cfg.q_dim), np.float32)
    c = cfg.to_c()
    st = oracle_lib().oracle_attention(C.byref(c), batch, seq, q, k, v, out, threads)
    if st:
        raise ValueError(f"oracle_attention status {st}")
    return out


def mha_forward(cfg: MhaCfg, batch: int, seq: int, Wq, Wk, Wv, Wo, x, threads: int = 0,
                want_qkv: bool = False):
    """Returns (pre [B*T,qd], post [B*T,d]) and, with want_qkv, the FP32 q/k/v projections."""
    Wq, Wk, Wv, Wo, x = (_f32(a) for a in (Wq, Wk, Wv, Wo, x))
    M = batch * seq
    pre = np.empty((M, cfg.q_dim), np.float32)
    post = np.empty((M, cfg.d_model), np.float32)
    q = np.empty((M, cfg.q_dim), np.float32) if want_qkv else None
    k = np.empty((M, cfg.kv_dim), np.float32) if want_qkv else None
    v = np.empty((M, cfg.kv_dim), np.float32) if want_qkv else None
    ptr = (lambda a: a.ctypes.data if a is not None else None)
    c = cfg.to_c()
    st = oracle_lib().oracle_mha_forward(C.byref(c), batch, seq, Wq, Wk, Wv, Wo, x, pre, post,
                                         ptr(q), ptr(k), ptr(v), threads)
    if st:
        raise ValueError(f"oracle_mha_forward status {st}")
    return (pre, post, q, k, v) if want_qkv else (pre, post)


def mha_decode(cfg: MhaCfg, ctx_len, k_cache, v_cache, Wq, Wk, Wv, Wo, x_new, threads: int = 0):
    """k_cache/v_cache [B, S, kd] (rows < ctx_len[b] valid, keys after RoPE).
    Returns (pre [B,qd], post [B,d], k_new [B,kd], v_new [B,kd])."""
    ctx = np.ascontiguousarray(ctx_len, dtype=np.int32)
    kc, vc = _f32(k_cache), _f32(v_cache)
    B = ctx.shape[0]
    pre = np.empty((B, cfg.q_dim), np.float32)
    post = np.empty((B, cfg.d_model), np.float32)
    kn = np.empty((B, cfg.kv_dim), np.float32)
    vn = np.empty((B, cfg.kv_dim), np.float32)
    c = cfg.to_c()
    st = oracle_lib().oracle_mha_decode(C.byref(c), B, ctx, kc.shape[1], kc, vc, _f32(Wq), _f32(Wk),
                                        _f32(Wv), _f32(Wo), _f32(x_new), pre, post,
                                        kn.ctypes.data, vn.ctypes.data, threads)
    if st:
        raise ValueError(f"oracle_mha_decode status {st}")
    return pre, post, kn, vn


def encode(dtype: int, w) -> tuple[np.ndarray, float]:
    w = _f32(w).ravel()
    out = np.zeros(8 * max(1, w.size), np.uint8)
    s = C.c_float()
    n = oracle_lib().oracle_encode(dtype, w, w.size, out, C.byref(s))
    if n < 0:
        raise ValueError(f"oracle_encode: dtype {dtype} not covered")
    return out[:n].copy(), s.value


def decode(dtype: int, raw, n: int, scale: float) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    if raw.size == 0:
        raw = np.zeros(1, np.uint8)
    out = np.empty(n, np.float32)
    if oracle_lib().oracle_decode(dtype, raw, n, scale, out):
        raise ValueError(f"oracle_decode: dtype {dtype} not covered")
    return out


def fp8_rowscale(w):
    w = _f32(w)
    rows, cols = w.shape
    codes = np.empty((rows, cols), np.uint8)
    scales = np.empty(rows, np.float32)
    oracle_lib().oracle_fp8_rowscale_encode(w, rows, cols, codes, scales)
    dec = np.empty((rows, cols), np.float32)
    oracle_lib().oracle_fp8_rowscale_decode(codes, scales, rows, cols, dec)
    return codes, scales, dec


def nf4_block(w, block: int = 64):
    w = _f32(w)
    n = w.size
    packed = np.empty((n + 1) // 2, np.uint8)
    amax = np.empty((n + block - 1) // block, np.float32)
    oracle_lib().oracle_nf4_block_encode(w.ravel(), n, block, packed, amax)
    dec = np.empty(n, np.float32)
    oracle_lib().oracle_nf4_block_decode(packed, amax, n, block, dec)
    return packed, amax, dec.reshape(w.shape)


# ---------------------------------------------------------- reference calls
def ref_mha_forward(cfg: MhaCfg, batch: int, seq: int, Wq, Wk, Wv, Wo, x, dtype: int = 1):
    """Runs the reference's own mha::forward (CPU executor). Returns (code, msg, pre, post)."""
    lib = ref_lib()
    r = cfg
    M = batch * seq
    pre = np.zeros((M, cfg.q_dim), np.float32)
    post = np.zeros((M, cfg.d_model), np.float32)
    st = lib.ref_mha_forward_cfg(batch, seq, r.d_model, r.num_heads, r.num_kv_heads, r.head_dim,
                                 r.max_seq_len, r.mask, r.pos, r.softmax, r.window, r.prefix_len,
                                 r.window_causal, r.rope_theta, r.scale_override, dtype,
                                 _f32(Wq), _f32(Wk), _f32(Wv), _f32(Wo), _f32(x), pre, post)
    return st.code, st.message.decode(), pre, post


def roundtrip(dtype: int, w) -> np.ndarray:
    """decode(encode(w)) of the oracle port for FormatNone dtypes 0-33."""
    w = _f32(w)
    out = np.empty_like(w)
    st = oracle_lib().oracle_roundtrip(dtype, w, w.size, out)
    if st:
        raise ValueError(f"oracle_roundtrip: dtype {dtype} unsupported")
    return out


def ref_weight_roundtrip(dtype: int, w):
    w = _f32(w)
    rows, cols = w.shape
    cap = C.c_int64(16 * w.size + 16)
    native = np.zeros(cap.value, np.uint8)
    s = C.c_float()
    dec = np.empty_like(w)
    st = ref_lib().ref_weight_roundtrip(dtype, rows, cols, w, native, C.byref(cap), C.byref(s), dec)
    return st.code, st.message.decode(), native[:cap.value].copy(), s.value, dec


# ------------------------------------------------------------ block forwards
def norm_forward(layernorm: bool, x, gamma, beta=None, eps: float = 0.0):
    """RMSNorm / LayerNorm forward of the oracle on decoded weights: (pre, post)."""
    x = _f32(x)
    dim = x.shape[-1]
    rows = x.size // dim
    pre = np.empty_like(x)
    post = np.empty_like(x)
    b = _f32(beta if beta is not None else np.zeros(dim, np.float32))
    if oracle_lib().oracle_norm_forward(1 if layernorm else 0, rows, dim, eps, _f32(gamma), b, x, pre, post):
        raise ValueError("oracle_norm_forward: bad shape")
    return pre, post


def swiglu_forward(x, Gate, Up, Down, threads: int = 0):
    x = _f32(x)
    inter, d = np.shape(Gate)
    tokens = x.size // d
    pre = np.empty((tokens, inter), np.float32)
    post = np.empty((tokens, d), np.float32)
    if oracle_lib().oracle_swiglu_forward(tokens, d, inter, _f32(Gate), _f32(Up), _f32(Down), x, pre, post,
                                          threads):
        raise ValueError("oracle_swiglu_forward: bad shape")
    return pre, post


def embedding_forward(x, W, in_last: int = 1, act: int = -1):
    x = _f32(x)
    vocab, emb = np.shape(W)
    tokens = x.size // in_last
    pre = np.empty((tokens, emb), np.float32)
    post = np.empty((tokens, emb), np.float32)
    if oracle_lib().oracle_embedding_forward(tokens, vocab, emb, in_last, act, _f32(W), x, pre, post):
        raise ValueError("oracle_embedding_forward: bad shape")
    return pre, post


def ref_swiglu_forward(batch, seq, Gate, Up, Down, x, dtype=1):
    inter, d = np.shape(Gate)
    pre = np.zeros(batch * seq * inter, np.float32)
    post = np.zeros(batch * seq * d, np.float32)
    st = ref_lib().ref_swiglu_forward_f32(batch, seq, d, inter, dtype, _f32(Gate), _f32(Up), _f32(Down), _f32(x),
                                          pre, post)
    return st.code, st.message.decode(), pre, post


def ref_norm_forward(layernorm, batch, seq, dim, eps, gamma, x, beta=None, dtype=1):
    pre = np.zeros(batch * seq * dim, np.float32)
    post = np.zeros(batch * seq * dim, np.float32)
    if layernorm:
        st = ref_lib().ref_layernorm_forward_f32(batch, seq, dim, eps, dtype, _f32(gamma), _f32(beta), _f32(x),
                                                 pre, post)
    else:
        st = ref_lib().ref_rmsnorm_forward_f32(batch, seq, dim, eps, dtype, _f32(gamma), _f32(x), pre, post)
    return st.code, st.message.decode(), pre, post


def ref_embedding_forward(batch, vocab, emb, seq_len, in_rank, in_last, act, W, x, dtype=1):
    n = batch * seq_len if in_rank > 1 else seq_len
    pre = np.zeros(n * emb, np.float32)
    post = np.zeros(n * emb, np.float32)
    st = ref_lib().ref_embedding_forward_f32(batch, vocab, emb, seq_len, in_rank, in_last, act, dtype, _f32(W),
                                             _f32(x), pre, post)
    return st.code, st.message.decode(), pre, post


def ref_mha_normalbp(cfg: MhaCfg, batch, seq, Wq, Wk, Wv, Wo, x, grad_or_target, use_target, lr, dtype=1):
    """The reference's welvet_mha_normalbp_f32 (oracle/_ref): (code, msg, pre, post, dX, dW, W_after, loss)."""
    r = cfg.resolved()
    qd, kd, d = r.q_dim, r.kv_dim, r.d_model
    M = batch * seq
    pre = np.zeros(M * qd, np.float32)
    post = np.zeros(M * d, np.float32)
    dX = np.zeros(M * d, np.float32)
    nw = qd * d + 2 * kd * d + d * qd
    dW = np.zeros(nw, np.float32)
    Wa = np.zeros(nw, np.float32)
    loss = C.c_double(0.0)
    st = ref_lib().ref_mha_normalbp_f32(batch, seq, cfg.d_model, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                                        cfg.max_seq_len, cfg.mask, cfg.pos, dtype, _f32(Wq), _f32(Wk), _f32(Wv),
                                        _f32(Wo), _f32(x), _f32(grad_or_target), int(use_target), float(lr), pre,
                                        post, dX, dW, Wa, C.byref(loss))
    return st.code, st.message.decode(), pre, post, dX, dW, Wa, loss.value


def mha_normalbp(cfg: MhaCfg, batch, seq, Wq, Wk, Wv, Wo, x, grad_or_target, use_target, lr, sgd_f32=True,
                 threads=0):
    """The oracle's welvet_mha_normalbp_f32 on decoded weights: (code, pre, post, dX, dW, W_after, loss)."""
    r = cfg.resolved()
    qd, kd, d = r.q_dim, r.kv_dim, r.d_model
    M = batch * seq
    pre = np.zeros(M * qd, np.float32)
    post = np.zeros(M * d, np.float32)
    dX = np.zeros(M * d, np.float32)
    nw = qd * d + 2 * kd * d + d * qd
    dW = np.zeros(nw, np.float32)
    Wa = np.zeros(nw, np.float32)
    loss = C.c_double(0.0)
    c = cfg.to_c()
    code = oracle_lib().oracle_mha_normalbp(C.byref(c), batch, seq, _f32(Wq), _f32(Wk), _f32(Wv), _f32(Wo),
                                            _f32(x), _f32(grad_or_target), int(use_target), float(lr),
                                            1 if sgd_f32 else 0, pre, post, dX, dW, Wa, C.byref(loss), threads)
    return code, pre, post, dX, dW, Wa, loss.value
