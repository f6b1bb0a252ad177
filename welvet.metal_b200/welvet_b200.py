"""Python binding (ctypes) of libwelvet_b200.so — the B200 MHA forward path behind
the reference's C ABI (include/welvet_c.h) and its extension (include/welvet_b200.h).

Mirrors the reference's Python-facing plumbing (scripts/release_smoke.py drives the
same C ABI through ctypes): statuses are returned as `welvet_status` and raised as
WelvetError(code, message) with the reference's codes (1 invalid, 2 unsupported,
3 gap, 4 internal).

Host buffers are numpy arrays; device buffers are torch CUDA tensors (torch is only
the allocator/stream plumbing here). The library is loaded from lib/ next to this
file; if it is missing the import of any entry point raises — there is no fallback.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libwelvet_b200.so")

# Exported symbols declared in include/welvet_c.h and include/welvet_b200.h.
C_ABI_SYMBOLS = ("welvet_version", "welvet_runtime_identity", "welvet_metal_init",
                 "welvet_metal_available", "welvet_mha_forward_f32", "welvet_mha_normalbp_f32",
                 "welvet_swiglu_forward_f32",
                 "welvet_rmsnorm_forward_f32", "welvet_layernorm_forward_f32", "welvet_embedding_forward_f32",
                 "welvet_model_abi_version", "welvet_model_mount", "welvet_model_forward",
                 "welvet_model_train_credit", "welvet_model_dense_proxy", "welvet_model_forward_pair",
                 "welvet_model_backward", "welvet_model_apply_sgd", "welvet_model_train_mse",
                 "welvet_model_export_weights", "welvet_model_sync", "welvet_model_release",
                 "welvet_metal_blob_free")
EXT_SYMBOLS = ("welvet_b200_mha_config_default", "welvet_b200_mha_mount", "welvet_b200_mha_release",
               "welvet_b200_mha_forward", "welvet_b200_mha_forward_rows", "welvet_b200_mha_check",
               "welvet_b200_kv_create",
               "welvet_b200_kv_release", "welvet_b200_kv_fill", "welvet_b200_mha_prefill",
               "welvet_b200_mha_decode", "welvet_b200_comm_unique_id", "welvet_b200_comm_attach",
               "welvet_b200_gemm", "welvet_b200_split_tf32", "welvet_b200_attention",
               "welvet_b200_codec_roundtrip", "welvet_b200_codec_encode", "welvet_b200_codec_decode",
               "welvet_b200_fp8_rowscale_encode", "welvet_b200_fp8_rowscale_decode",
               "welvet_b200_nf4_block_encode", "welvet_b200_nf4_block_decode",
               "welvet_b200_fill_synthetic", "welvet_b200_device_check", "welvet_b200_launch_count",
               "welvet_b200_profile_enable", "welvet_b200_profile_read",
               "welvet_b200_decode_attention_static", "welvet_b200_swiglu_mount", "welvet_b200_swiglu_forward",
               "welvet_b200_swiglu_forward_host", "welvet_b200_swiglu_release", "welvet_b200_norm_forward",
               "welvet_b200_embedding_forward", "welvet_b200_wait_probe", "welvet_b200_mha_set_output_mode",
               "welvet_b200_attention_tf32")
PROFILE_SLOTS = ("gemm_qkv", "attn_prefill", "gemm_o", "attn_decode", "gemm_qkv_decode", "gemm_o_decode",
                 "allreduce", "other", "gemm_gate_up", "gemm_down", "norm", "embedding", "attn_bwd", "gemm_grad")

DTYPES = {"float64": 0, "float32": 1, "float16": 2, "bfloat16": 3, "fp8e4m3": 4, "fp8e5m2": 5, "nf4": 26}


class WelvetError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"welvet status {code}: {message}")
        self.code = code
        self.message = message


class Status(C.Structure):
    _fields_ = [("code", C.c_int32), ("message", C.c_char * 256)]


class MhaConfig(C.Structure):
    """welvet_b200_mha_config (include/welvet_b200.h)."""
    _fields_ = [(n, C.c_int32) for n in (
        "d_model", "num_heads", "num_kv_heads", "head_dim", "max_seq_len",
        "mask", "pos", "softmax", "window", "prefix_len", "window_causal")] + [
        ("rope_theta", C.c_double), ("scale_override", C.c_double)] + [
        (n, C.c_int32) for n in ("seq_mode", "precision", "weight_format", "head_begin",
                                 "head_count", "device")]

    @classmethod
    def make(cls, d_model, num_heads, num_kv_heads=0, **kw) -> "MhaConfig":
        c = cls()
        lib().welvet_b200_mha_config_default(C.byref(c), d_model, num_heads, num_kv_heads)
        for k, v in kw.items():
            if not hasattr(c, k):
                raise AttributeError(k)
            setattr(c, k, v)
        return c

    def resolved(self):
        hd = self.head_dim if self.head_dim > 0 else self.d_model // self.num_heads
        nk = self.num_kv_heads if self.num_kv_heads > 0 else self.num_heads
        return hd, nk


_LIB = None
_vp = C.c_void_p


def lib():
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(LIB_PATH):
        raise FileNotFoundError(f"{LIB_PATH} is missing: build it with welvet.metal_b200/build.py "
                                "(there is no CPU fallback)")
    L = C.CDLL(LIB_PATH)
    L.welvet_version.restype = C.c_char_p
    L.welvet_runtime_identity.restype = C.c_char_p
    L.welvet_metal_init.restype = Status
    L.welvet_metal_available.restype = C.c_int32
    L.welvet_mha_forward_f32.argtypes = [C.c_int32] * 11 + [_vp] * 7
    L.welvet_mha_normalbp_f32.argtypes = [C.c_int32] * 11 + [_vp] * 6 + [C.c_int32, C.c_double] + [_vp] * 5 + \
        [C.POINTER(C.c_double)]
    L.welvet_mha_normalbp_f32.restype = Status
    L.welvet_swiglu_forward_f32.argtypes = [C.c_int32] * 6 + [_vp] * 6
    L.welvet_rmsnorm_forward_f32.argtypes = [C.c_int32] * 3 + [C.c_double, C.c_int32, C.c_int32] + [_vp] * 4
    L.welvet_layernorm_forward_f32.argtypes = [C.c_int32] * 3 + [C.c_double, C.c_int32, C.c_int32] + [_vp] * 5
    L.welvet_embedding_forward_f32.argtypes = [C.c_int32] * 9 + [_vp] * 4
    for name in ("welvet_swiglu_forward_f32", "welvet_rmsnorm_forward_f32", "welvet_layernorm_forward_f32",
                 "welvet_embedding_forward_f32"):
        getattr(L, name).restype = Status
    L.welvet_b200_swiglu_mount.argtypes = [C.c_int32] * 5 + [_vp] * 3 + [C.c_int32, C.POINTER(_vp)]
    L.welvet_b200_swiglu_forward.argtypes = [_vp, C.c_int64, _vp, _vp, _vp, _vp]
    L.welvet_b200_swiglu_forward_host.argtypes = [_vp, C.c_int64, _vp, _vp, _vp]
    L.welvet_b200_swiglu_release.argtypes = [_vp]
    L.welvet_b200_swiglu_release.restype = None
    L.welvet_b200_norm_forward.argtypes = [C.c_int32, C.c_int64, C.c_int32, C.c_double, _vp, _vp, _vp, _vp, _vp,
                                           C.c_int32, _vp]
    L.welvet_b200_embedding_forward.argtypes = [C.c_int64] + [C.c_int32] * 4 + [_vp] * 3 + [C.c_int32, _vp]
    for name in ("welvet_b200_swiglu_mount", "welvet_b200_swiglu_forward", "welvet_b200_swiglu_forward_host",
                 "welvet_b200_norm_forward", "welvet_b200_embedding_forward"):
        getattr(L, name).restype = Status
    L.welvet_mha_forward_f32.restype = Status
    cfgp = C.POINTER(MhaConfig)
    L.welvet_b200_mha_config_default.argtypes = [cfgp, C.c_int32, C.c_int32, C.c_int32]
    L.welvet_b200_mha_config_default.restype = None
    L.welvet_b200_mha_mount.argtypes = [cfgp, C.c_int32, _vp, _vp, _vp, _vp, C.c_int32, C.POINTER(_vp)]
    L.welvet_b200_mha_release.argtypes = [_vp]
    L.welvet_b200_mha_release.restype = None
    L.welvet_b200_mha_forward.argtypes = [_vp, C.c_int32, C.c_int32, _vp, _vp, _vp, C.c_int32, _vp]
    L.welvet_b200_mha_forward_rows.argtypes = [_vp, C.c_int32, C.c_int32, _vp, _vp]
    L.welvet_b200_mha_check.argtypes = [_vp]
    L.welvet_b200_kv_create.argtypes = [_vp, C.c_int32, C.c_int32, C.POINTER(_vp)]
    L.welvet_b200_kv_release.argtypes = [_vp]
    L.welvet_b200_kv_release.restype = None
    L.welvet_b200_kv_fill.argtypes = [_vp, C.c_int32, C.c_int32, _vp, _vp, C.c_int32, _vp]
    L.welvet_b200_mha_prefill.argtypes = [_vp, _vp, C.c_int32, C.c_int32, _vp, _vp, _vp, C.c_int32, _vp]
    L.welvet_b200_mha_decode.argtypes = [_vp, _vp, C.c_int32, _vp, _vp, _vp, C.c_int32, _vp]
    L.welvet_b200_comm_unique_id.argtypes = [C.c_char_p]
    L.welvet_b200_comm_attach.argtypes = [_vp, C.c_char_p, C.c_int32, C.c_int32]
    L.welvet_b200_gemm.argtypes = [C.c_int32] * 4 + [_vp] * 6 + [C.c_int32, _vp]
    L.welvet_b200_split_tf32.argtypes = [_vp, _vp, _vp, C.c_int64, _vp]
    L.welvet_b200_attention.argtypes = [cfgp, C.c_int32, C.c_int32, _vp, _vp, _vp, _vp, C.c_int32, _vp]
    L.welvet_b200_codec_roundtrip.argtypes = [C.c_int32, _vp, _vp, C.c_int64, _vp]
    L.welvet_b200_codec_encode.argtypes = [C.c_int32, _vp, _vp, _vp, C.c_int64, _vp]
    L.welvet_b200_codec_decode.argtypes = [C.c_int32, _vp, _vp, _vp, C.c_int64, _vp]
    L.welvet_b200_fp8_rowscale_encode.argtypes = [_vp, C.c_int32, C.c_int32, _vp, _vp, _vp]
    L.welvet_b200_fp8_rowscale_decode.argtypes = [_vp, _vp, C.c_int32, C.c_int32, _vp, C.c_int32, _vp]
    L.welvet_b200_nf4_block_encode.argtypes = [_vp, C.c_int64, _vp, _vp, _vp]
    L.welvet_b200_nf4_block_decode.argtypes = [_vp, _vp, C.c_int64, _vp, C.c_int32, _vp]
    L.welvet_b200_fill_synthetic.argtypes = [_vp, C.c_int32, C.c_int64, C.c_uint64, C.c_uint64, C.c_int32,
                                             C.c_double, _vp]
    L.welvet_b200_launch_count.argtypes = [C.c_int32]
    L.welvet_b200_launch_count.restype = C.c_int64
    L.welvet_b200_profile_enable.argtypes = [C.c_int32]
    L.welvet_b200_profile_enable.restype = None
    L.welvet_b200_profile_read.argtypes = [C.POINTER(C.c_double), C.POINTER(C.c_int64), C.c_int32]
    L.welvet_b200_profile_read.restype = None
    L.welvet_b200_decode_attention_static.argtypes = [cfgp, C.c_int32, C.c_int32, _vp, C.c_int32, _vp, _vp, _vp,
                                                      C.c_int32, _vp, _vp, C.c_int32, _vp]
    L.welvet_b200_wait_probe.argtypes = [C.c_uint64, _vp]
    L.welvet_b200_mha_set_output_mode.argtypes = [_vp, C.c_int32]
    L.welvet_b200_attention_tf32.argtypes = [cfgp, C.c_int32, C.c_int32] + [_vp] * 9 + [_vp]
    for name in ("welvet_b200_wait_probe", "welvet_b200_mha_set_output_mode", "welvet_b200_attention_tf32",
"welvet_b200_mha_mount", "welvet_b200_mha_forward", "welvet_b200_mha_forward_rows",
                 "welvet_b200_mha_check",
                 "welvet_b200_kv_create", "welvet_b200_kv_fill", "welvet_b200_mha_prefill",
                 "welvet_b200_mha_decode", "welvet_b200_comm_unique_id", "welvet_b200_comm_attach",
                 "welvet_b200_gemm", "welvet_b200_split_tf32", "welvet_b200_attention",
                 "welvet_b200_codec_roundtrip", "welvet_b200_codec_encode", "welvet_b200_codec_decode",
                 "welvet_b200_fp8_rowscale_encode", "welvet_b200_fp8_rowscale_decode",
                 "welvet_b200_nf4_block_encode", "welvet_b200_nf4_block_decode",
                 "welvet_b200_fill_synthetic", "welvet_b200_device_check",
                 "welvet_b200_decode_attention_static"):
        getattr(L, name).restype = Status
    _LIB = L
    return L


def check(st: Status):
    if st.code:
        raise WelvetError(st.code, st.message.decode(errors="replace"))


# ------------------------------------------------------------------ pointers
def _ptr(a):
    """Device pointer of a torch tensor, host pointer of a numpy array, or None."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        if not a.flags["C_CONTIGUOUS"]:
            raise ValueError("numpy buffers must be C-contiguous")
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        if not a.is_contiguous():
            raise ValueError("tensors must be contiguous")
        return a.data_ptr()
    if isinstance(a, int):
        return a
    raise TypeError(type(a))


def _stream(s):
    if s is None:
        return None
    if hasattr(s, "cuda_stream"):
        return s.cuda_stream
    return int(s)


def _is_host(a) -> bool:
    return isinstance(a, np.ndarray) or (hasattr(a, "is_cuda") and not a.is_cuda)


def _on_device(*arrs) -> int:
    flags = {_is_host(a) for a in arrs if a is not None}
    if len(flags) > 1:
        raise ValueError("mix of host (numpy) and device (torch) buffers")
    return 0 if flags == {True} else 1


# ------------------------------------------------------------- welvet_c.h
def version() -> str:
    return lib().welvet_version().decode()


def runtime_identity() -> str:
    return lib().welvet_runtime_identity().decode()


def metal_init():
    check(lib().welvet_metal_init())


def metal_available() -> bool:
    return bool(lib().welvet_metal_available())


def mha_forward_f32(batch, seq, d_model, num_heads, num_kv_heads, head_dim, max_seq_len, mask, pos, dtype,
                    Q, K, V, O, x, backend=0):
    """welvet_mha_forward_f32 with numpy buffers. Returns (pre, post) as numpy."""
    hd = head_dim if head_dim > 0 else (d_model // num_heads if num_heads > 0 else 0)
    f = lambda a: np.ascontiguousarray(a, dtype=np.float32)
    Q, K, V, O, x = (f(a) for a in (Q, K, V, O, x))
    pre = np.zeros(max(1, batch * seq * num_heads * hd), np.float32)
    post = np.zeros(max(1, batch * seq * d_model), np.float32)
    st = lib().welvet_mha_forward_f32(batch, seq, d_model, num_heads, num_kv_heads, head_dim, max_seq_len,
                                      mask, pos, dtype, backend, _ptr(Q), _ptr(K), _ptr(V), _ptr(O), _ptr(x),
                                      _ptr(pre), _ptr(post))
    check(st)
    return pre, post


def mha_normalbp_f32(batch, seq, d_model, num_heads, num_kv_heads, head_dim, max_seq_len, mask, pos, dtype,
                     Q, K, V, O, x, grad_or_target, use_target, lr, backend=0, out=None):
    """welvet_mha_normalbp_f32 with numpy buffers: (pre, post, dX, dW, W_after, loss).
    `out` = (pre, post, dX, dW, W_after) lets a caller reuse its output arrays
    (contiguous float32 of M*q_dim, M*d_model, M*d_model, |W|, |W| elements)."""
    f = lambda a: np.ascontiguousarray(a, dtype=np.float32)  # noqa: E731
    Q, K, V, O, x, g = (f(a) for a in (Q, K, V, O, x, grad_or_target))
    M = batch * seq
    qd, kdim = Q.shape[0], K.shape[0]
    nw = Q.size + K.size + V.size + O.size
    sizes = (max(1, M * qd), max(1, M * d_model), max(1, M * d_model), nw, nw)
    if out is None:
        pre, post, dX, dW, Wa = (np.zeros(n, np.float32) for n in sizes)
    else:
        pre, post, dX, dW, Wa = out
        for a, n in zip(out, sizes):
            if a.dtype != np.float32 or not a.flags.c_contiguous or a.size != n:
                raise ValueError(f"mha_normalbp_f32: output buffers must be contiguous float32 of sizes {sizes}")
    loss = C.c_double(0.0)
    check(lib().welvet_mha_normalbp_f32(batch, seq, d_model, num_heads, num_kv_heads, head_dim, max_seq_len, mask,
                                        pos, dtype, backend, _ptr(Q), _ptr(K), _ptr(V), _ptr(O), _ptr(x), _ptr(g),
                                        int(use_target), float(lr), _ptr(pre), _ptr(post), _ptr(dX), _ptr(dW),
                                        _ptr(Wa), C.byref(loss)))
    return pre, post, dX, dW, Wa, loss.value


def swiglu_forward_f32(batch, seq, Gate, Up, Down, x, dtype=1, backend=0):
    """welvet_swiglu_forward_f32 with numpy buffers: (pre [B*S*inter], post [B*S*in])."""
    f = lambda a: np.ascontiguousarray(a, dtype=np.float32)  # noqa: E731
    Gate, Up, Down, x = (f(a) for a in (Gate, Up, Down, x))
    inter, d = Gate.shape
    pre = np.zeros(max(1, batch * seq * inter), np.float32)
    post = np.zeros(max(1, batch * seq * d), np.float32)
    check(lib().welvet_swiglu_forward_f32(batch, seq, d, inter, dtype, backend, _ptr(Gate), _ptr(Up), _ptr(Down),
                                          _ptr(x), _ptr(pre), _ptr(post)))
    return pre, post


def norm_forward_f32(layernorm, batch, seq, dim, eps, gamma, x, beta=None, dtype=1, backend=0):
    """welvet_rmsnorm_forward_f32 / welvet_layernorm_forward_f32: (pre, post)."""
    f = lambda a: np.ascontiguousarray(a, dtype=np.float32)  # noqa: E731
    gamma, x = f(gamma), f(x)
    n = max(1, batch * seq * dim)
    pre = np.zeros(n, np.float32)
    post = np.zeros(n, np.float32)
    if layernorm:
        beta = f(beta)
        st = lib().welvet_layernorm_forward_f32(batch, seq, dim, eps, dtype, backend, _ptr(gamma), _ptr(beta),
                                                _ptr(x), _ptr(pre), _ptr(post))
    else:
        st = lib().welvet_rmsnorm_forward_f32(batch, seq, dim, eps, dtype, backend, _ptr(gamma), _ptr(x),
                                              _ptr(pre), _ptr(post))
    check(st)
    return pre, post


def embedding_forward_f32(batch, vocab, emb, seq_len, in_rank, in_last, act, W, x, dtype=1, backend=0):
    """welvet_embedding_forward_f32: (pre, post), each [tokens * emb]."""
    W = np.ascontiguousarray(W, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    tokens = seq_len if in_rank == 1 else batch * seq_len
    pre = np.zeros(max(1, tokens * emb), np.float32)
    post = np.zeros(max(1, tokens * emb), np.float32)
    check(lib().welvet_embedding_forward_f32(batch, vocab, emb, seq_len, in_rank, in_last, act, dtype, backend,
                                             _ptr(W), _ptr(x), _ptr(pre), _ptr(post)))
    return pre, post


# -------------------------------------------------------------- extension
class SwigluLayer:
    """Resident SwiGLU feed-forward (welvet_b200_swiglu_*). precision 0: FP32
    tensors, 1: BF16 device tensors."""

    def __init__(self, Gate, Up, Down, dtype: int = 1, precision: int = 0, device: int = -1):
        self._h = _vp()
        on_dev = _on_device(Gate, Up, Down)
        if not on_dev:
            Gate, Up, Down = (np.ascontiguousarray(a, dtype=np.float32) for a in (Gate, Up, Down))
        self.inter, self.input_dim = Gate.shape
        self.precision = precision
        check(lib().welvet_b200_swiglu_mount(self.input_dim, self.inter, precision, device, dtype, _ptr(Gate),
                                             _ptr(Up), _ptr(Down), on_dev, C.byref(self._h)))

    def forward(self, tokens, x, pre, post, stream=None):
        """Device tensors (torch); pre may be None."""
        check(lib().welvet_b200_swiglu_forward(self._h, tokens, _ptr(x), _ptr(pre), _ptr(post), _stream(stream)))

    def forward_host(self, tokens, x, pre=None, post=None):
        x = np.ascontiguousarray(x, dtype=np.float32)
        if post is None:
            post = np.zeros(tokens * self.input_dim, np.float32)
        check(lib().welvet_b200_swiglu_forward_host(self._h, tokens, _ptr(x), _ptr(pre), _ptr(post)))
        return pre, post

    def close(self):
        if self._h:
            lib().welvet_b200_swiglu_release(self._h)
            self._h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def norm_forward(layernorm, rows, dim, eps, gamma, x, pre, post, beta=None, io_bf16=0, stream=None):
    """welvet_b200_norm_forward on device tensors (gamma/beta decoded FP32)."""
    check(lib().welvet_b200_norm_forward(1 if layernorm else 0, rows, dim, eps, _ptr(gamma), _ptr(beta), _ptr(x),
                                         _ptr(pre), _ptr(post), io_bf16, _stream(stream)))


def embedding_forward(tokens, vocab, emb, in_last, act, W, x, out, out_bf16=0, stream=None):
    """welvet_b200_embedding_forward on device tensors (W decoded FP32)."""
    check(lib().welvet_b200_embedding_forward(tokens, vocab, emb, in_last, act, _ptr(W), _ptr(x), _ptr(out),
                                              out_bf16, _stream(stream)))


class MhaLayer:
    """Resident MHA layer (welvet_b200_mha_*)."""

    def __init__(self, cfg: MhaConfig, Q, K, V, O, dtype: int = 1):
        self.cfg = cfg
        self._h = _vp()
        on_dev = _on_device(Q, K, V, O)
        if not on_dev:
            Q, K, V, O = (np.ascontiguousarray(a, dtype=np.float32) for a in (Q, K, V, O))
        self._keep = (Q, K, V, O)
        check(lib().welvet_b200_mha_mount(C.byref(cfg), dtype, _ptr(Q), _ptr(K), _ptr(V), _ptr(O), on_dev,
                                          C.byref(self._h)))
        self._keep = None
        hd, nk = cfg.resolved()
        hc = cfg.head_count if cfg.head_count > 0 else cfg.num_heads
        self.head_dim = hd
        self.q_dim_local = hc * hd
        self.kv_dim_local = max(1, hc // (cfg.num_heads // nk)) * hd

    def close(self):
        if self._h:
            lib().welvet_b200_mha_release(self._h)
            self._h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def forward(self, batch, seq, x, pre, post, stream=None):
        check(lib().welvet_b200_mha_forward(self._h, batch, seq, _ptr(x), _ptr(pre), _ptr(post),
                                            _on_device(x, pre, post), _stream(stream)))

    def forward_rows(self, batch_local, seq, x, post):
        """Row-sharded host I/O: this rank's batch_local sequences of x in, the same
        sequences of post (summed over ranks) out; host tensors / arrays."""
        check(lib().welvet_b200_mha_forward_rows(self._h, batch_local, seq, _ptr(x), _ptr(post)))

    def check_device(self):
        check(lib().welvet_b200_mha_check(self._h))

    def prefill(self, kv: "KvCache", batch, seq, x, pre, post, stream=None):
        check(lib().welvet_b200_mha_prefill(self._h, kv.handle, batch, seq, _ptr(x), _ptr(pre), _ptr(post),
                                            _on_device(x, pre, post), _stream(stream)))

    def decode(self, kv: "KvCache", batch, x, pre, post, stream=None):
        check(lib().welvet_b200_mha_decode(self._h, kv.handle, batch, _ptr(x), _ptr(pre), _ptr(post),
                                           _on_device(x, pre, post), _stream(stream)))

    def set_output_mode(self, mode: int):
        """0: all-reduce output (default); 1: reduce-scatter, rank r keeps the r-th
        row slice of each chunk summed; 2: the same rows through an exchange of the
        attention output before the output projection (BF16 layers; otherwise as 1)
        (welvet_b200_mha_set_output_mode)."""
        check(lib().welvet_b200_mha_set_output_mode(self._h, mode))

    def attach_comm(self, uid: bytes, nranks: int, rank: int):
        check(lib().welvet_b200_comm_attach(self._h, uid, nranks, rank))


class KvCache:
    def __init__(self, layer: MhaLayer, max_batch: int, max_ctx: int):
        self._h = _vp()
        self.layer = layer
        check(lib().welvet_b200_kv_create(layer.handle, max_batch, max_ctx, C.byref(self._h)))

    @property
    def handle(self):
        return self._h

    def fill(self, batch, ctx_len, k=None, v=None, stream=None):
        on = _on_device(k, v) if k is not None else 1
        check(lib().welvet_b200_kv_fill(self._h, batch, ctx_len, _ptr(k), _ptr(v), on, _stream(stream)))

    def close(self):
        if self._h:
            lib().welvet_b200_kv_release(self._h)
            self._h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def comm_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    check(lib().welvet_b200_comm_unique_id(buf))
    return buf.raw


# --------------------------------------------------------- kernel entries
def gemm(kind, M, N, K, a, b, out, a_lo=None, b_lo=None, b_scale=None, out_bf16=0, stream=None):
    check(lib().welvet_b200_gemm(kind, M, N, K, _ptr(a), _ptr(a_lo), _ptr(b), _ptr(b_lo), _ptr(b_scale),
                                 _ptr(out), out_bf16, _stream(stream)))


def split_tf32(x, hi, lo, stream=None):
    check(lib().welvet_b200_split_tf32(_ptr(x), _ptr(hi), _ptr(lo), x.numel(), _stream(stream)))


def attention(cfg: MhaConfig, batch, seq, q, k, v, out, impl=0, stream=None):
    check(lib().welvet_b200_attention(C.byref(cfg), batch, seq, _ptr(q), _ptr(k), _ptr(v), _ptr(out), impl,
                                      _stream(stream)))


def attention_tf32(cfg: MhaConfig, batch, seq, q, q_lo, k, k_lo, v, v_lo, out, out_hi=None, out_lo=None,
                   stream=None):
    """FP32 attention on the tensor cores from the TF32 split of q, k, v."""
    check(lib().welvet_b200_attention_tf32(C.byref(cfg), batch, seq, _ptr(q), _ptr(q_lo), _ptr(k), _ptr(k_lo),
                                           _ptr(v), _ptr(v_lo), _ptr(out), _ptr(out_hi), _ptr(out_lo),
                                           _stream(stream)))


def codec_roundtrip(dtype, w, out, stream=None):
    check(lib().welvet_b200_codec_roundtrip(dtype, _ptr(w), _ptr(out), w.numel(), _stream(stream)))


def codec_encode(dtype, w, codes, scale_out=None, stream=None):
    check(lib().welvet_b200_codec_encode(dtype, _ptr(w), _ptr(codes), _ptr(scale_out), w.numel(), _stream(stream)))


def codec_decode(dtype, codes, out, scale=None, stream=None):
    check(lib().welvet_b200_codec_decode(dtype, _ptr(codes), _ptr(scale), _ptr(out), out.numel(), _stream(stream)))


def fp8_rowscale_encode(w, codes, scales, stream=None):
    rows, cols = w.shape
    check(lib().welvet_b200_fp8_rowscale_encode(_ptr(w), rows, cols, _ptr(codes), _ptr(scales), _stream(stream)))


def fp8_rowscale_decode(codes, scales, out, out_bf16=0, stream=None):
    rows, cols = codes.shape
    check(lib().welvet_b200_fp8_rowscale_decode(_ptr(codes), _ptr(scales), rows, cols, _ptr(out), out_bf16,
                                                _stream(stream)))


def nf4_block_encode(w, packed, absmax, stream=None):
    check(lib().welvet_b200_nf4_block_encode(_ptr(w), w.numel(), _ptr(packed), _ptr(absmax), _stream(stream)))


def nf4_block_decode(packed, absmax, out, out_bf16=0, stream=None):
    check(lib().welvet_b200_nf4_block_decode(_ptr(packed), _ptr(absmax), out.numel(), _ptr(out), out_bf16,
                                             _stream(stream)))


def fill_synthetic(dst, seed, kind, a, offset=0, stream=None):
    import torch
    check(lib().welvet_b200_fill_synthetic(_ptr(dst), 1 if dst.dtype == torch.bfloat16 else 0, dst.numel(),
                                           seed, offset, kind, a, _stream(stream)))


def device_check():
    check(lib().welvet_b200_device_check())


def wait_probe(limit_ns: int, stream=None):
    """Launches the bounded-wait probe (a wait nothing satisfies, given up after
    limit_ns); the timeout is reported by the next device_check()."""
    check(lib().welvet_b200_wait_probe(limit_ns, _stream(stream)))


def launch_count(reset: bool = False) -> int:
    return int(lib().welvet_b200_launch_count(1 if reset else 0))


def profile_enable(on: bool = True):
    lib().welvet_b200_profile_enable(1 if on else 0)


def profile_read(reset: bool = True) -> dict:
    """{slot: (total_ms, launches)} of the live per-kernel event timing."""
    ms = (C.c_double * len(PROFILE_SLOTS))()
    cnt = (C.c_int64 * len(PROFILE_SLOTS))()
    lib().welvet_b200_profile_read(ms, cnt, 1 if reset else 0)
    return {name: (ms[i], cnt[i]) for i, name in enumerate(PROFILE_SLOTS)}


# ----------------------------------------------------------- synthetic data
_M1, _M2, _GOLD, _SEEDMUL = 0xBF58476D1CE4E5B9, 0x94D049BB133111EB, 0x9E3779B97F4A7C15, 0xD1B54A32D192ED03


def _mix64(z: np.ndarray) -> np.ndarray:
    z = z + np.uint64(_GOLD)
    z = (z ^ (z >> np.uint64(30))) * np.uint64(_M1)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(_M2)
    return z ^ (z >> np.uint64(31))


def _unif01(seed: int, idx: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = _mix64(np.uint64((seed * _SEEDMUL) & 0xFFFFFFFFFFFFFFFF) + idx.astype(np.uint64))
    return (z >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)


def synthetic(n: int, seed: int, kind: int, a: float, offset: int = 0) -> np.ndarray:
    """Host twin of welvet_b200_fill_synthetic (same counter stream): kind 0
    uniform(-a, a), kind 1 normal(0, a) by Box-Muller in double, as float32."""
    idx = np.arange(offset, offset + n, dtype=np.uint64)
    if kind == 0:
        v = a * (2.0 * _unif01(seed, idx) - 1.0)
    else:
        with np.errstate(over="ignore"):
            u1 = _unif01(seed, idx * np.uint64(2))
            u2 = _unif01(seed, idx * np.uint64(2) + np.uint64(1))
        v = a * np.sqrt(-2.0 * np.log(1.0 - u1)) * np.cos(6.283185307179586 * u2)
    return v.astype(np.float32)


def head_shard(num_heads: int, num_kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """(head_begin, head_count) of `rank` when `world` GPUs split one layer by heads:
    equal contiguous blocks of whole KV groups, as mha_mount requires. Each rank then
    holds the Wq/Wk/Wv rows and the Wo columns of its heads; the per-rank outputs of
    the O projection sum to the layer output (one all-reduce)."""
    nk = num_kv_heads if num_kv_heads > 0 else num_heads
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("head_shard: need 0 <= rank < world")
    if num_heads % nk or num_heads % world:
        raise ValueError(f"head_shard: {num_heads} heads do not split over {world} ranks")
    hc = num_heads // world
    if hc % (num_heads // nk):
        raise ValueError(f"head_shard: {hc} heads per rank do not cover whole KV groups of {num_heads // nk}")
    return rank * hc, hc


def xavier_weights(d_model: int, q_dim: int, kv_dim: int, seed: int = 0):
    """Wq [qd,d], Wk/Wv [kd,d], Wo [d,qd], Xavier-uniform a = sqrt(6/(fan_in+fan_out)),
    drawn in this order from one counter stream (seed 0 by default)."""
    shapes = [(q_dim, d_model), (kv_dim, d_model), (kv_dim, d_model), (d_model, q_dim)]
    out, off = [], 0
    for r, c in shapes:
        a = float(np.sqrt(6.0 / (r + c)))
        out.append(synthetic(r * c, seed, 0, a, off).reshape(r, c))
        off += r * c
    return out
