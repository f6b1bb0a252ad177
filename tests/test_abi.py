"""CPU tests of the drop-in boundary: the library loads, exports every symbol
declared in include/*.h, reports the reference's version string, and applies the
reference's argument / config checks (which run before any device work)."""
import os
import re

import numpy as np
import pytest

import welvet_b200 as W
from conftest import ROOT


def declared_symbols():
    names = []
    for h in ("welvet_c.h", "welvet_b200.h"):
        with open(os.path.join(ROOT, "include", h)) as f:
            src = f.read()
        names += re.findall(r"WELVET_API\s+[\w\s\*]+?\b(welvet_\w+)\s*\(", src)
    return sorted(set(names))


def test_headers_declare_the_reference_mha_entry_points():
    names = declared_symbols()
    for n in ("welvet_version", "welvet_runtime_identity", "welvet_metal_init", "welvet_metal_available",
              "welvet_mha_forward_f32", "welvet_mha_normalbp_f32", "welvet_swiglu_forward_f32",
              "welvet_rmsnorm_forward_f32",
              "welvet_layernorm_forward_f32", "welvet_embedding_forward_f32"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = W.lib()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing
    assert set(declared_symbols()) == set(W.C_ABI_SYMBOLS + W.EXT_SYMBOLS)


def test_version_matches_reference_abi():
    assert W.version() == "0.71"  # reference src/interop/c_abi.cpp:79-82
    assert W.runtime_identity().startswith("cuda:")


@pytest.mark.parametrize("args,code", [
    (dict(batch=0), 1), (dict(seq=0), 1), (dict(d_model=0), 1), (dict(num_heads=0), 1),
])
def test_mha_forward_rejects_bad_arguments(args, code):
    base = dict(batch=1, seq=4, d_model=8, num_heads=2, num_kv_heads=0, head_dim=0, max_seq_len=0, mask=1, pos=0,
                dtype=1)
    base.update(args)
    z = np.zeros(64, np.float32)
    with pytest.raises(W.WelvetError) as e:
        W.mha_forward_f32(**base, Q=z, K=z, V=z, O=z, x=z)
    assert e.value.code == code and "invalid argument" in e.value.message


def test_mha_forward_rejects_null_pointers():
    lib = W.lib()
    st = lib.welvet_mha_forward_f32(1, 4, 8, 2, 0, 0, 0, 1, 0, 1, 0, None, None, None, None, None, None, None)
    assert st.code == 1


@pytest.mark.parametrize("kw,msg", [
    (dict(d_model=10, num_heads=4), "HeadDim unset"),
    (dict(d_model=64, num_heads=4, num_kv_heads=3), "not divisible"),
    (dict(d_model=64, num_heads=4, softmax=2), "unknown Softmax"),
    (dict(d_model=64, num_heads=4, precision=0, weight_format=1), "weight_format"),
    (dict(d_model=64, num_heads=4, head_begin=3, head_count=2), "head shard"),
])
def test_config_validation_matches_reference(kw, msg):
    """validate() of src/layers/mha/mha.cpp:63-94 (plus the B200 execution checks)."""
    cfg = W.MhaConfig.make(kw.pop("d_model"), kw.pop("num_heads"), kw.pop("num_kv_heads", 0), **kw)
    z = np.zeros(64 * 64, np.float32)
    with pytest.raises(W.WelvetError) as e:
        W.MhaLayer(cfg, z, z, z, z)
    assert e.value.code == 1 and msg in e.value.message


def test_unsupported_dtype_is_reported_not_silently_changed():
    z = np.zeros(64 * 64, np.float32)
    with pytest.raises(W.WelvetError) as e:
        W.mha_forward_f32(1, 4, 64, 4, 0, 0, 0, 1, 0, 40, z, z, z, z, np.zeros(4 * 64, np.float32))
    assert e.value.code == 2


def test_synthetic_stream_is_deterministic():
    a = W.synthetic(1000, 7, 0, 1.0)
    b = np.concatenate([W.synthetic(500, 7, 0, 1.0), W.synthetic(500, 7, 0, 1.0, offset=500)])
    np.testing.assert_array_equal(a, b)
    n = W.synthetic(20000, 1, 1, 1.0)
    assert abs(n.mean()) < 0.05 and abs(n.std() - 1) < 0.05


# ---------------------------------------------------------- block entries
def test_block_entries_reject_bad_arguments_like_the_reference():
    """Argument checks of src/interop/c_abi.cpp:326-361, 437-469, 543-577, 792-832
    (code 1, '<layer>: invalid argument'); no device work is reached."""
    z = np.zeros(64, np.float32)
    lib = W.lib()
    cases = [
        (lib.welvet_swiglu_forward_f32(0, 1, 4, 4, 1, 0, *[W._ptr(z)] * 6), "swiglu"),
        (lib.welvet_swiglu_forward_f32(1, 1, 4, 0, 1, 0, *[W._ptr(z)] * 6), "swiglu"),
        (lib.welvet_rmsnorm_forward_f32(1, 1, 0, 0.0, 1, 0, *[W._ptr(z)] * 4), "rmsnorm"),
        (lib.welvet_layernorm_forward_f32(1, 1, 4, 0.0, 1, 0, W._ptr(z), None, W._ptr(z), W._ptr(z), W._ptr(z)),
         "layernorm"),
        (lib.welvet_embedding_forward_f32(1, 0, 4, 2, 2, 1, -1, 1, 0, *[W._ptr(z)] * 4), "embedding"),
    ]
    for st, name in cases:
        assert st.code == 1 and st.message.decode() == f"{name}: invalid argument"
    st = lib.welvet_embedding_forward_f32(1, 4, 4, 2, 4, 1, -1, 1, 0, *[W._ptr(z)] * 4)
    assert st.code == 1 and st.message.decode() == "embedding: bad in_rank"


def test_block_entries_report_unknown_dtypes_with_the_reference_codes():
    # reference: norms/embedding -> 3 "... gap? pack_native unknown" (WeightStore::make),
    # SwiGLU -> 2 "swiglu Gate: dense ... FormatNone forward unsupported ..." (dense mount)
    z = np.zeros(64, np.float32)
    lib = W.lib()
    st = lib.welvet_rmsnorm_forward_f32(1, 2, 8, 0.0, 34, 0, *[W._ptr(z)] * 4)
    assert st.code == 3 and st.message.decode().startswith("rmsnorm gamma:")
    st = lib.welvet_layernorm_forward_f32(1, 2, 8, 0.0, 40, 0, *[W._ptr(z)] * 5)
    assert st.code == 3 and st.message.decode().startswith("layernorm gamma:")
    st = lib.welvet_embedding_forward_f32(1, 4, 8, 2, 2, 1, -1, 34, 0, *[W._ptr(z)] * 4)
    assert st.code == 3 and st.message.decode().startswith("embedding weights:")
    st = lib.welvet_swiglu_forward_f32(2, 1, 8, 4, 34, 0, *[W._ptr(z)] * 6)
    assert st.code == 2 and st.message.decode().startswith("swiglu Gate:")
    # embedding rank 3 needs in_last 1 or emb
    st = lib.welvet_embedding_forward_f32(1, 4, 8, 2, 3, 3, -1, 1, 0, *[W._ptr(z)] * 4)
    assert st.code == 1 and "want 1 or emb" in st.message.decode()


def test_normalbp_rejects_bad_arguments_and_dtypes_like_the_reference():
    """c_abi.cpp:249-268: null / non-positive arguments -> 1 "mha nbp: invalid
    argument"; dtype outside 0-33 -> 1 "mha nbp: bad dtype"; SGD of non-FP32 storage
    is the documented gap (status 2). No device work is reached."""
    z = np.zeros(4096, np.float32)
    lib = W.lib()
    loss = W.C.c_double(0.0)
    args = lambda b, dt, lr: (b, 4, 16, 2, 0, 0, 0, 1, 0, dt, 0, *[W._ptr(z)] * 6, 1, lr, *[W._ptr(z)] * 5,  # noqa
                              W.C.byref(loss))
    st = lib.welvet_mha_normalbp_f32(*args(0, 1, 0.0))
    assert st.code == 1 and st.message.decode() == "mha nbp: invalid argument"
    st = lib.welvet_mha_normalbp_f32(*args(1, 34, 0.0))
    assert st.code == 1 and st.message.decode() == "mha nbp: bad dtype 34"
    st = lib.welvet_mha_normalbp_f32(*args(1, 9, 0.01))
    assert st.code == 2 and "Float32 only" in st.message.decode()
