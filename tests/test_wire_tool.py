"""The wire tool (welvet.metal_b200/lib/welvet_dense_fwd) and the C++ layer /
volume API behind it.

CPU: the tool's argument and wire handling (version, usage, malformed and
unsupported wires give the reference tool's exit codes and messages), and a C++
program against include/welvet/*.hpp checking the API's host-side logic (validate
defaults and messages, hop order, coordinates, remote links, volume_dense answers).

GPU: the reference's golden MHA cases piped through WVM1 (-> welvet_mha_forward_f32)
and through a 1x1x1x1 WMV1 volume (mha::new_configured + architecture::bind_mha +
runtime::forward::volume_dense), within 1e-4 of the reference's own outputs;
--bench wires; chained (1x1x1x2) and remote-link (1x1x1x3) volumes against the FP64
oracle applied cell by cell.
"""
import os
import struct
import subprocess

import numpy as np
import pytest

import oracle_py as O
import welvet_b200 as W
from conftest import ROOT, golden_cases, load_golden, rel_err

TOOL = os.path.join(ROOT, "welvet.metal_b200", "lib", "welvet_dense_fwd")
F32_TOL = 1e-4


def _run(wire: bytes, *args, timeout=300):
    return subprocess.run([TOOL, *args], input=wire, capture_output=True, timeout=timeout)


def _i32(*v):
    return struct.pack(f"<{len(v)}i", *v)


def _f32(a):
    return np.ascontiguousarray(a, np.float32).tobytes()


# ----------------------------------------------------------------------- CPU
def test_tool_version_and_usage():
    r = subprocess.run([TOOL, "--version"], capture_output=True, text=True)
    assert r.returncode == 0 and r.stdout.strip() == W.lib().welvet_version().decode()
    r = subprocess.run([TOOL, "--help"], capture_output=True, text=True)
    assert r.returncode == 0 and "WVM1" in r.stderr and "WMV1" in r.stderr
    r = subprocess.run([TOOL, "--nope"], capture_output=True, text=True)
    assert r.returncode == 2 and "unknown arg" in r.stderr


def test_tool_rejects_malformed_wires():
    assert _run(b"").returncode == 2                                   # no magic
    r = _run(b"WVD3" + _i32(1, 2, 3, 4))
    assert r.returncode == 2 and b"unsupported wire WVD3" in r.stderr  # other families: not this path
    r = _run(b"WVM1" + _i32(1, 2, 3))
    assert r.returncode == 2 and b"short WVM1 header" in r.stderr
    r = _run(b"WVM1" + _i32(1, 4, 10, 3, 0, 0, 0, 1, 0, 1, 0))
    assert r.returncode == 2 and b"bad mha dims" in r.stderr           # 10 % 3 != 0
    r = _run(b"WVM1" + _i32(1, 4, 8, 2, 0, 0, 0, 1, 0, 1, 0) + _f32(np.zeros(10)))
    assert r.returncode == 2 and b"short WVM1 weights" in r.stderr
    r = _run(b"WMV1" + _i32(1, 1, 1))
    assert r.returncode == 2 and b"short WMV1 header" in r.stderr
    r = _run(b"WMV1" + _i32(1, 1, 1, 1, 0, 0, 0))
    assert r.returncode == 2 and b"bad batch" in r.stderr
    r = _run(b"WMV1" + _i32(1, 1, 1, 1, 1, 0, 0) + _i32(0))           # the only cell is disabled
    assert r.returncode == 1


def test_cxx_api_host_logic(tmp_path):
    exe = tmp_path / "cxx_api_check"
    lib = os.path.join(ROOT, "welvet.metal_b200", "lib")
    subprocess.run(["g++", "-std=c++17", "-O1", f"-I{os.path.join(ROOT, 'include')}",
                    os.path.join(ROOT, "tests", "cxx_api_check.cpp"), "-o", str(exe), f"-L{lib}", "-lwelvet_b200",
                    f"-Wl,-rpath,{lib}"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stdout + r.stderr


# ----------------------------------------------------------------------- GPU
def _wire_cases():
    """Golden cases the WVM1 wire can express (no softmax kind, window or prefix fields)."""
    return sorted(n for n, c in golden_cases().items()
                  if not any(c["cfg"].get(k, 0) for k in ("softmax", "window", "prefix_len")))


def _weights(c):
    return W.xavier_weights(c.d_model, c.q_dim, c.kv_dim, seed=0)


def _wvm1(case, x):
    kw = case["cfg"]
    c = O.MhaCfg(**kw).resolved()
    hdr = _i32(case["batch"], case["seq"], c.d_model, c.num_heads, kw.get("num_kv_heads", 0), 0,
               kw.get("max_seq_len", 0), kw.get("mask", 1), kw.get("pos", 0), case["dtype"], 0)
    return b"WVM1" + hdr + b"".join(_f32(w) for w in _weights(c)) + _f32(x)


def _cell(case, seq, Ws):
    kw = case["cfg"]
    c = O.MhaCfg(**kw).resolved()
    return (_i32(1, seq, c.d_model, c.num_heads, kw.get("num_kv_heads", 0), 0, kw.get("max_seq_len", 0),
                 kw.get("mask", 1), kw.get("pos", 0), case["dtype"]) + b"".join(_f32(w) for w in Ws))


def _parse_wvmo(out: bytes):
    assert out[:4] == b"WVMO"
    n_pre = struct.unpack_from("<i", out, 4)[0]
    pre = np.frombuffer(out, np.float32, n_pre, 8)
    n_post = struct.unpack_from("<i", out, 8 + 4 * n_pre)[0]
    post = np.frombuffer(out, np.float32, n_post, 12 + 4 * n_pre)
    return pre, post


def _parse_wvfo(out: bytes):
    assert out[:4] == b"WVFO"
    n = struct.unpack_from("<i", out, 4)[0]
    return np.frombuffer(out, np.float32, n, 8)


@pytest.mark.gpu
@pytest.mark.parametrize("name", _wire_cases())
def test_wvm1_golden(torch_cuda, name):
    case = golden_cases()[name]
    g = load_golden(name)
    r = _run(_wvm1(case, g["x"]))
    assert r.returncode == 0, r.stderr.decode()
    pre, post = _parse_wvmo(r.stdout)
    assert rel_err(pre, g["pre"].reshape(-1)) < F32_TOL
    assert rel_err(post, g["post"].reshape(-1)) < F32_TOL


@pytest.mark.gpu
@pytest.mark.parametrize("name", _wire_cases())
def test_wmv1_single_cell_golden(torch_cuda, name):
    case = golden_cases()[name]
    g = load_golden(name)
    c = O.MhaCfg(**case["cfg"]).resolved()
    wire = b"WMV1" + _i32(1, 1, 1, 1, case["batch"], 0, 0) + _cell(case, case["seq"], _weights(c)) + _f32(g["x"])
    r = _run(wire)
    assert r.returncode == 0, r.stderr.decode()
    assert rel_err(_parse_wvfo(r.stdout), g["post"].reshape(-1)) < F32_TOL


@pytest.mark.gpu
def test_bench_wires(torch_cuda):
    name = "cfg1_tiny_f32"
    case = golden_cases()[name]
    g = load_golden(name)
    r = _run(_wvm1(case, g["x"]), "--bench=2")
    assert r.returncode == 0, r.stderr.decode()
    assert r.stdout[:4] == b"WVB1"
    ns, iters = struct.unpack_from("<qi", r.stdout, 4)
    assert ns > 0 and iters == 2
    _, post = _parse_wvmo(r.stdout[16:])
    assert rel_err(post, g["post"].reshape(-1)) < F32_TOL
    c = O.MhaCfg(**case["cfg"]).resolved()
    wire = b"WMV1" + _i32(1, 1, 1, 1, case["batch"], 0, 0) + _cell(case, case["seq"], _weights(c)) + _f32(g["x"])
    r = _run(wire, "--bench=3")
    assert r.returncode == 0, r.stderr.decode()
    assert r.stdout[:4] == b"WVB2"
    mount_ns, exec_ns, iters = struct.unpack_from("<qqi", r.stdout, 4)
    assert mount_ns > 0 and exec_ns > 0 and iters == 3
    assert rel_err(_parse_wvfo(r.stdout[24:]), g["post"].reshape(-1)) < F32_TOL


def _oracle_cell(case, Ws, x, B, T):
    kw = dict(case["cfg"])
    oc = O.MhaCfg(**kw)
    _, post = O.mha_forward(oc, B, T, *[O.roundtrip(case["dtype"], w).reshape(w.shape) for w in Ws], x)
    return post


@pytest.mark.gpu
def test_wmv1_chained_and_remote_link_volumes(torch_cuda):
    """1x1x1x2: cell 1 takes cell 0's post. 1x1x1x3 with a remote link from l=2 to
    l=0: cell 2 takes cell 0's post instead of cell 1's."""
    case = {"cfg": {"d_model": 64, "num_heads": 4, "num_kv_heads": 2, "max_seq_len": 64}, "dtype": 9}  # int8
    B, T, d = 2, 12, 64
    c = O.MhaCfg(**case["cfg"]).resolved()
    Ws = [W.xavier_weights(d, c.q_dim, c.kv_dim, seed=s) for s in range(3)]
    x = W.synthetic(B * T * d, 1, 1, 1.0).reshape(B * T, d)
    p0 = _oracle_cell(case, Ws[0], x, B, T)
    p1 = _oracle_cell(case, Ws[1], p0, B, T)
    wire = b"WMV1" + _i32(1, 1, 1, 2, B, 0, 0) + _cell(case, T, Ws[0]) + _cell(case, T, Ws[1]) + _f32(x)
    r = _run(wire)
    assert r.returncode == 0, r.stderr.decode()
    assert rel_err(_parse_wvfo(r.stdout), p1.reshape(-1)) < F32_TOL
    p2 = _oracle_cell(case, Ws[2], p0, B, T)
    wire = (b"WMV1" + _i32(1, 1, 1, 3, B, 0, 1) + _i32(0, 0, 0, 2, 0, 0, 0, 0) + _cell(case, T, Ws[0]) +
            _cell(case, T, Ws[1]) + _cell(case, T, Ws[2]) + _f32(x))
    r = _run(wire)
    assert r.returncode == 0, r.stderr.decode()
    assert rel_err(_parse_wvfo(r.stdout), p2.reshape(-1)) < F32_TOL
