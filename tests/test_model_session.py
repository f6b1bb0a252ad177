"""WMN1 model sessions of MHA models (welvet_model_mount / forward / forward_pair /
export_weights, the reference's src/interop/model_session.cpp:319-576).

Descriptors are written here by the reference's grammar (model_wire.hpp,
child_wire.hpp:153-190, model_session.cpp read_store): magic, root, count, four
grid dimensions, children (MHA: 9 int32 + Q, K, V, O FP32; nested Stack: count +
children), Cameral controls (root, then each child's tree), the store count and
four stores per MHA child (dtype, rows, cols, scale, FP32 payload, native bytes,
bias), and for a Grid root six int32 per cell.

CPU: malformed descriptors and unsupported parts answer the reference's codes
before any device work; the training entry points answer code 2.
GPU: Stack (two MHA children, one inside a nested Stack) and Grid (a disabled
cell, a remote link) models against the FP64 oracle applied layer by layer on the
reference-decoded store weights, 1e-4; forward_pair; NWS1 export returns the
snapshots as mounted.
"""
import ctypes as C
import struct

import numpy as np
import pytest

import oracle_py as O
import welvet_b200 as W
from conftest import rel_err

F32_TOL = 1e-4


class Blob(C.Structure):
    _fields_ = [("data", C.POINTER(C.c_uint8)), ("size", C.c_size_t)]


def _lib():
    L = W.lib()
    L.welvet_model_abi_version.restype = C.c_int32
    L.welvet_model_mount.argtypes = [C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p)]
    L.welvet_model_mount.restype = W.Status
    for name in ("welvet_model_forward", "welvet_model_forward_pair"):
        getattr(L, name).argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.POINTER(Blob)]
        getattr(L, name).restype = W.Status
    L.welvet_model_export_weights.argtypes = [C.c_void_p, C.POINTER(Blob)]
    L.welvet_model_export_weights.restype = W.Status
    L.welvet_model_train_mse.argtypes = [C.c_void_p, C.c_int32, C.c_double, C.c_int32, C.c_void_p, C.c_size_t,
                                         C.POINTER(C.c_double)]
    L.welvet_model_train_mse.restype = W.Status
    L.welvet_model_sync.argtypes = [C.c_void_p, C.c_int32]
    L.welvet_model_sync.restype = W.Status
    L.welvet_model_release.argtypes = [C.c_void_p]
    L.welvet_model_release.restype = None
    L.welvet_metal_blob_free.argtypes = [C.POINTER(Blob)]
    L.welvet_metal_blob_free.restype = None
    return L


def _i32(*v):
    return struct.pack(f"<{len(v)}i", *v)


def _f32(a):
    return np.ascontiguousarray(a, np.float32).tobytes()


def _controls(sync=False):
    out = _i32(1, 0) + _i32(1) + struct.pack("<d", 0.01) + struct.pack("<3d", 0.0, 0.0, 0.0)
    if not sync:
        return out + _i32(0)
    return (out + _i32(1, 1) + struct.pack("<d", 0.5) + _i32(0) + _i32(1) + struct.pack("<d", 1.0) +
            _i32(1, 2, 0, 1) + _i32(1, 0, 0, 0, 0, 1, 0))


class Mha:
    def __init__(self, d, heads, kv, seq, msl, mask, pos, dtype, seed):
        self.d, self.heads, self.kv, self.seq, self.msl = d, heads, kv, seq, msl
        self.mask, self.pos, self.dtype = mask, pos, dtype
        hd = d // heads
        self.ws = W.xavier_weights(d, heads * hd, kv * hd, seed=seed)

    def child(self):
        return (_i32(7, self.seq, self.d, self.heads, self.kv, 0, self.msl, self.mask, self.pos, self.dtype) +
                b"".join(_f32(w) for w in self.ws))

    def stores(self):
        out = b""
        for w in self.ws:
            rows, cols = w.shape
            out += _i32(self.dtype, rows, cols) + struct.pack("<f", 0.0)
            out += _i32(w.size) + _f32(w)
            native = np.zeros(7, np.uint8)  # snapshot bytes: carried through export unchanged
            out += _i32(native.size) + native.tobytes() + _i32(0)
        return out

    def oracle(self, x, B, T):
        oc = O.MhaCfg(d_model=self.d, num_heads=self.heads, num_kv_heads=self.kv, max_seq_len=self.msl,
                      mask=self.mask, pos=self.pos)
        deq = [O.roundtrip(self.dtype, w).reshape(w.shape) for w in self.ws]
        return O.mha_forward(oc, B, T, *deq, x)


def _descriptor(root, cells, dims=(1, 1, 1, 1), grid_meta=b"", sync=False):
    """cells: list of Mha, None (kind None) or ('nested', [Mha...])."""
    body = b""
    mhas = []

    def child(c):
        nonlocal body
        if c is None:
            return _i32(0)
        if isinstance(c, tuple):
            return _i32(19, len(c[1])) + b"".join(child(x) for x in c[1])
        mhas.append(c)
        return c.child()

    def tree(c):
        if isinstance(c, tuple):
            return _controls() + b"".join(tree(x) for x in c[1])
        return _controls()

    body = struct.pack("<I", 0x314E4D57) + _i32(root, len(cells), *dims)
    body += b"".join(child(c) for c in cells)
    body += _controls(sync) + b"".join(tree(c) for c in cells)
    body += _i32(4 * len(mhas)) + b"".join(m.stores() for m in mhas)
    return body + grid_meta


def _tensor(x, shape):
    return _i32(len(shape), *shape) + _f32(x)


def _mount(desc):
    L = _lib()
    h = C.c_void_p()
    buf = C.create_string_buffer(desc, len(desc))
    st = L.welvet_model_mount(buf, len(desc), C.byref(h))
    return st, h


def _out_tensors(blob, count):
    raw = C.string_at(blob.data, blob.size)
    off, out = 0, []
    for _ in range(count):
        rank = struct.unpack_from("<i", raw, off)[0]
        shape = struct.unpack_from(f"<{rank}i", raw, off + 4)
        off += 4 + 4 * rank
        n = struct.unpack_from("<i", raw, off)[0]
        out.append(np.frombuffer(raw, np.float32, n, off + 4).reshape(shape))
        off += 4 + 4 * n
    assert off == blob.size
    return out


# ----------------------------------------------------------------------- CPU
def test_abi_version_and_training_entries():
    L = _lib()
    assert L.welvet_model_abi_version() == 1
    loss = C.c_double(1.0)
    st = L.welvet_model_train_mse(None, 0, 0.1, 1, None, 0, C.byref(loss))
    assert st.code == 2 and loss.value == 0.0
    assert L.welvet_model_sync(None, 0).code == 2


def test_malformed_descriptors():
    m = Mha(64, 4, 4, 8, 64, 1, 0, 1, 0)
    good = _descriptor(0, [m])
    st, _ = _mount(b"XXXX" + good[4:])
    assert st.code == 1 and b"descriptor version" in st.message
    st, _ = _mount(good[:len(good) // 2])
    assert st.code == 1
    st, _ = _mount(good + b"\0\0\0\0")
    assert st.code == 1 and b"trailing" in st.message
    bad_store = bytearray(good)
    # the first store's rows: after magic, root/count/dims (6 int32), the child, controls
    off = 4 + 24 + len(m.child()) + len(_controls()) * 2 + 4 + 4
    struct.pack_into("<i", bad_store, off, 3)
    st, _ = _mount(bytes(bad_store))
    assert st.code == 1 and b"store metadata" in st.message
    st, _ = _mount(struct.pack("<I", 0x314E4D57) + _i32(1, 1, 1, 1, 1, 1) + _i32(0) + b"\0" * 64)
    assert st.code == 2  # Parallel root
    st, _ = _mount(struct.pack("<I", 0x314E4D57) + _i32(0, 1, 1, 1, 1, 1) + _i32(1, 4, 4, 0, 1) + b"\0" * 64)
    assert st.code == 2 and b"kind 1" in st.message  # a Dense child


# ----------------------------------------------------------------------- GPU
@pytest.mark.gpu
def test_stack_model_against_oracle(torch_cuda):
    L = _lib()
    B, T, d = 2, 12, 64
    m1 = Mha(d, 4, 2, T, 64, 1, 0, 9, seed=0)   # Int8 storage, GQA, RoPE
    m2 = Mha(d, 4, 4, T, 64, 2, 2, 1, seed=1)   # Float32, bidirectional, ALiBi (inside a nested Stack)
    desc = _descriptor(0, [m1, None, ("nested", [m2])], sync=True)
    st, h = _mount(desc)
    assert st.code == 0, st.message
    x = W.synthetic(B * T * d, 1, 1, 1.0).reshape(B * T, d)
    inp = _tensor(x, (B, T, d))
    blob = Blob()
    st = L.welvet_model_forward(h, C.create_string_buffer(inp, len(inp)), len(inp), C.byref(blob))
    assert st.code == 0, st.message
    (post,) = _out_tensors(blob, 1)
    L.welvet_metal_blob_free(C.byref(blob))
    _, p1 = m1.oracle(x, B, T)
    pre2, p2 = m2.oracle(p1, B, T)
    assert post.shape == (B, T, d)
    assert rel_err(post.reshape(-1, d), p2) < F32_TOL
    st = L.welvet_model_forward_pair(h, C.create_string_buffer(inp, len(inp)), len(inp), C.byref(blob))
    assert st.code == 0, st.message
    pre, post2 = _out_tensors(blob, 2)
    L.welvet_metal_blob_free(C.byref(blob))
    assert rel_err(pre.reshape(B * T, -1), pre2) < F32_TOL and rel_err(post2.reshape(-1, d), p2) < F32_TOL
    # NWS1 export: the snapshots as mounted
    st = L.welvet_model_export_weights(h, C.byref(blob))
    assert st.code == 0, st.message
    raw = C.string_at(blob.data, blob.size)
    L.welvet_metal_blob_free(C.byref(blob))
    assert raw[:4] == b"NWS1" and struct.unpack_from("<i", raw, 4)[0] == 8
    assert raw[8:-4] == m1.stores() + m2.stores() and raw[-4:] == _i32(0)
    L.welvet_model_release(h)


@pytest.mark.gpu
def test_grid_model_against_oracle(torch_cuda):
    """1x1x1x3 grid: cell 0 -> cell 1 (disabled) -> cell 2, whose remote link
    takes cell 0's output."""
    L = _lib()
    B, T, d = 1, 16, 64
    ms = [Mha(d, 4, 4, T, 32, 1, 0, 14, seed=s) for s in range(3)]  # Int4 storage
    meta = _i32(1, 0, 0, 0, 0, 0) + _i32(0, 0, 0, 0, 0, 0) + _i32(1, 1, 0, 0, 0, 0)
    desc = _descriptor(2, ms, dims=(1, 1, 1, 3), grid_meta=meta)
    st, h = _mount(desc)
    assert st.code == 0, st.message
    x = W.synthetic(B * T * d, 1, 1, 1.0).reshape(B * T, d)
    inp = _tensor(x, (B, T, d))
    blob = Blob()
    st = L.welvet_model_forward(h, C.create_string_buffer(inp, len(inp)), len(inp), C.byref(blob))
    assert st.code == 0, st.message
    (post,) = _out_tensors(blob, 1)
    L.welvet_metal_blob_free(C.byref(blob))
    _, p0 = ms[0].oracle(x, B, T)
    _, p2 = ms[2].oracle(p0, B, T)
    assert rel_err(post.reshape(-1, d), p2) < F32_TOL
    L.welvet_model_release(h)
