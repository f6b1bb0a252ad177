"""Failure handling without a GPU fault: every failure ends in a status code,
never a hang (the reference's contract, include/welvet/status.hpp:8-30).

* Device side: the bounded-wait probe (welvet_b200_wait_probe) waits on an
  mbarrier that nothing arrives at, through the same bounded wait the pipeline
  kernels use, with a 50 ms limit. The kernel records the timeout in the error
  word and returns; device_check reports code 4, and the device keeps working.
* NCCL init: a layer attaches a 2-rank communicator whose second rank never
  joins; the attach gives up after WELVET_B200_COMM_TIMEOUT_MS, aborts the
  communicator and returns code 4 (one GPU).
* NCCL collective: two ranks on two GPUs run one forward together, then rank 1
  leaves between steps (no kernel or collective of it in flight); rank 0's next
  forward waits in the all-reduce, its bounded stream wait runs out, the
  communicator is aborted and the call returns code 4. NVLS is off. Skipped
  with fewer than two GPUs.

The NCCL cases run as child processes (rendezvous on 127.0.0.1) under a
timeout, so a regression cannot hold the test session.
"""
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

import welvet_b200 as W

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_wait_probe_rejects_bad_limit():
    """Host-side argument check (no GPU needed)."""
    st = W.lib().welvet_b200_wait_probe(0, None)
    assert st.code == 1
    st = W.lib().welvet_b200_wait_probe(20 * 10**9, None)
    assert st.code == 1


@pytest.mark.gpu
def test_wait_timeout_is_status_4_and_device_stays_usable(torch_cuda):
    torch = torch_cuda
    W.device_check()
    W.wait_probe(50_000_000)  # 50 ms
    with pytest.raises(W.WelvetError) as e:
        W.device_check()
    assert e.value.code == 4 and "wait timeout" in e.value.message
    W.device_check()  # the word was cleared
    # the context is intact: a tensor-core GEMM after the timeout is still right
    M, N, K = 256, 256, 128
    a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    b = torch.randn(N, K, device="cuda").to(torch.bfloat16)
    out = torch.empty(M, N, device="cuda")
    W.check(W.lib().welvet_b200_gemm(0, M, N, K, a.data_ptr(), None, b.data_ptr(), None, None, out.data_ptr(), 0,
                                     None))
    torch.cuda.synchronize()
    ref = a.float() @ b.float().t()
    assert (out - ref).abs().max().item() <= 1e-3 * ref.abs().max().item()
    W.device_check()


_CHILD_PRELUDE = f"""
import os, sys
sys.path[:0] = [{os.path.join(ROOT, 'welvet.metal_b200')!r}]
import numpy as np
import welvet_b200 as W
"""


def _run_child(code: str, env: dict, timeout: int = 180) -> subprocess.CompletedProcess:
    full_env = dict(os.environ)
    full_env.update(env)
    return subprocess.run([sys.executable, "-c", _CHILD_PRELUDE + textwrap.dedent(code)], env=full_env,
                          capture_output=True, text=True, timeout=timeout)


def _layer_src(device: int) -> str:
    return f"""
import torch
torch.cuda.set_device({device})
d, H = 256, 4
Ws = W.xavier_weights(d, d, d, seed=0)
cfg = W.MhaConfig.make(d, H, H, precision=1, seq_mode=1, head_begin=0, head_count=H, device={device})
"""


@pytest.mark.gpu
def test_comm_init_times_out_when_a_rank_never_joins(torch_cuda):
    code = _layer_src(0) + """
cfg.head_count = 2  # this rank's half of the heads
layer = W.MhaLayer(cfg, *Ws, dtype=1)
uid = W.comm_unique_id()
try:
    layer.attach_comm(uid, 2, 0)   # rank 1 never starts
    print("RESULT attached")
except W.WelvetError as e:
    print("RESULT", e.code, e.message)
layer.close()
"""
    r = _run_child(code, {"WELVET_B200_COMM_TIMEOUT_MS": "3000", "NCCL_NVLS_ENABLE": "0"})
    out = [ln for ln in r.stdout.splitlines() if ln.startswith("RESULT")]
    assert r.returncode == 0 and out, r.stdout + r.stderr
    assert out[0].startswith("RESULT 4") and "timed out" in out[0], out[0]


@pytest.mark.gpu
def test_collective_times_out_when_a_peer_leaves(torch_cuda):
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import tempfile
    tmp = tempfile.mkdtemp()
    uid_path = os.path.join(tmp, "uid")
    code = """
import time
rank = int(os.environ["TEST_RANK"])
""" + _layer_src(0).replace("torch.cuda.set_device(0)", "torch.cuda.set_device(rank)").replace(
        "device=0", "device=rank") + f"""
cfg.head_begin, cfg.head_count = 2 * rank, 2
layer = W.MhaLayer(cfg, *Ws, dtype=1)
uid_path = {uid_path!r}
if rank == 0:
    uid = W.comm_unique_id()
    with open(uid_path + ".tmp", "wb") as f:
        f.write(uid)
    os.replace(uid_path + ".tmp", uid_path)
else:
    while not os.path.exists(uid_path):
        time.sleep(0.05)
    uid = open(uid_path, "rb").read()
layer.attach_comm(uid, 2, rank)
B, T = 2, 64
x = W.synthetic(B * T * d, 1, 1, 1.0).reshape(B * T, d)
xb = torch.from_numpy(x).to(torch.bfloat16)
post = torch.empty(B * T, d, dtype=torch.bfloat16)
layer.forward(B, T, xb, None, post)       # step 1: both ranks
if rank == 1:
    os._exit(0)                           # leaves between steps
t0 = time.time()
try:
    layer.forward(B, T, xb, None, post)   # step 2: the peer is gone
    print("RESULT finished")
except W.WelvetError as e:
    print("RESULT", e.code, round(time.time() - t0, 1), e.message)
"""
    env = {"WELVET_B200_COMM_TIMEOUT_MS": "5000", "NCCL_NVLS_ENABLE": "0"}
    procs = []
    for rank in range(2):
        e = dict(os.environ)
        e.update(env)
        e["TEST_RANK"] = str(rank)
        procs.append(subprocess.Popen([sys.executable, "-c", _CHILD_PRELUDE + textwrap.dedent(code)], env=e,
                                      stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True))
    outs = []
    for p in procs:
        try:
            o, er = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            p.kill()
            o, er = p.communicate()
        outs.append((p.returncode, o, er))
    rc0, o0, e0 = outs[0]
    res = [ln for ln in o0.splitlines() if ln.startswith("RESULT")]
    assert res, o0 + e0
    assert res[0].startswith("RESULT 4"), res[0]
    assert outs[1][0] == 0, outs[1][2]
