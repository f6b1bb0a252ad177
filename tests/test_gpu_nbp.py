"""GPU parity of the MHA NormalBP leaf (welvet_mha_normalbp_f32) through the C ABI:
against golden vectors made by the reference itself (tests/golden/nbp_*.npz) and
against the FP64 oracle on larger shapes. FP32 outputs within 1e-4 (max-norm
relative); the loss within 1e-6 relative."""
import numpy as np
import pytest

import oracle_py as O
import welvet_b200 as W
from conftest import rel_err
from test_nbp_oracle import load_nbp, nbp_cases

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4


def run_case(kw, B, T, dtype, Ws, x, tgt, use_target, lr):
    cfg = O.MhaCfg(**kw)
    return W.mha_normalbp_f32(B, T, cfg.d_model, cfg.num_heads, kw.get("num_kv_heads", 0), 0,
                              kw.get("max_seq_len", 0), kw.get("mask", 1), kw.get("pos", 0), dtype, *Ws, x, tgt,
                              use_target, lr)


@pytest.mark.parametrize("name", sorted(nbp_cases()))
def test_normalbp_matches_reference_golden(torch_cuda, name):
    case = nbp_cases()[name]
    g = load_nbp(name)
    cfg = O.MhaCfg(**case["cfg"])
    c = cfg.resolved()
    Ws = W.xavier_weights(c.d_model, c.q_dim, c.kv_dim, seed=0)
    pre, post, dX, dW, Wa, loss = run_case(case["cfg"], case["batch"], case["seq"], case["dtype"], Ws, g["x"],
                                           g["target"], case["use_target"], case["lr"])
    for got, key in ((pre, "pre"), (post, "post"), (dX, "dX"), (dW, "dW"), (Wa, "W_after")):
        assert rel_err(got, g[key]) < F32_TOL, key
    ref_loss = float(g["loss"])
    assert abs(loss - ref_loss) <= 1e-6 * max(abs(ref_loss), 1e-30)


@pytest.mark.parametrize("kw,B,T,use_target,lr", [
    (dict(d_model=128, num_heads=4), 2, 48, 1, 0.01),
    (dict(d_model=128, num_heads=4, num_kv_heads=2, pos=3), 3, 20, 0, 0.0),
    (dict(d_model=64, num_heads=2, max_seq_len=32, mask=3), 3, 24, 1, 0.05),
    # head_dim 128 (two 64-dimension chunks, several GEMM tiles), the stream wrapping the ring
    (dict(d_model=256, num_heads=2, max_seq_len=96), 2, 80, 1, 0.01),
    # odd head_dim with RoPE: the last element of each head is not rotated
    (dict(d_model=42, num_heads=2), 2, 9, 1, 0.0),
    # 300 queries (the key/value reduction split over query rows), 600 keys in batch 1
    # (the q-gradient GEMM split over keys), the stream wrapping a 400-slot ring
    (dict(d_model=128, num_heads=2, max_seq_len=400), 2, 300, 1, 0.01),
])
def test_normalbp_against_oracle(torch_cuda, kw, B, T, use_target, lr):
    cfg = O.MhaCfg(**kw)
    c = cfg.resolved()
    Ws = W.xavier_weights(c.d_model, c.q_dim, c.kv_dim, seed=3)
    x = W.synthetic(B * T * c.d_model, 4, 1, 1.0)
    tgt = W.synthetic(B * T * c.d_model, 5, 1, 1.0)
    pre, post, dX, dW, Wa, loss = run_case(kw, B, T, 1, Ws, x, tgt, use_target, lr)
    code, rpre, rpost, rdX, rdW, rWa, rloss = O.mha_normalbp(cfg, B, T, *Ws, x, tgt, use_target, lr)
    assert code == 0
    for got, ref, key in ((pre, rpre, "pre"), (post, rpost, "post"), (dX, rdX, "dX"), (dW, rdW, "dW"),
                          (Wa, rWa, "W_after")):
        assert rel_err(got, ref) < F32_TOL, key
    assert abs(loss - rloss) <= 1e-6 * max(abs(rloss), 1e-30)


def test_normalbp_repeated_calls_of_one_configuration(torch_cuda):
    """Calls of one configuration reuse the device workspace and the mounted forward
    layer, loading each call's weights into it: weights that change between calls,
    a call of another shape in between, and caller-owned output arrays reused."""
    kw, B, T = dict(d_model=64, num_heads=4), 2, 16
    cfg = O.MhaCfg(**kw)
    c = cfg.resolved()
    x = W.synthetic(B * T * c.d_model, 7, 1, 1.0)
    tgt = W.synthetic(B * T * c.d_model, 8, 1, 1.0)
    M, nw = B * T, 4 * c.d_model * c.d_model
    outs = tuple(np.zeros(n, np.float32) for n in (M * c.q_dim, M * c.d_model, M * c.d_model, nw, nw))
    other = dict(d_model=32, num_heads=2)
    for seed in (11, 12, None, 11):
        if seed is None:
            oc = O.MhaCfg(**other).resolved()
            Wo = W.xavier_weights(oc.d_model, oc.q_dim, oc.kv_dim, seed=5)
            run_case(other, 3, 8, 1, Wo, W.synthetic(24 * oc.d_model, 9, 1, 1.0),
                     W.synthetic(24 * oc.d_model, 10, 1, 1.0), 1, 0.01)
            continue
        Ws = W.xavier_weights(c.d_model, c.q_dim, c.kv_dim, seed=seed)
        got = W.mha_normalbp_f32(B, T, c.d_model, c.num_heads, 0, 0, 0, 1, 0, 1, *Ws, x, tgt, 1, 0.01, out=outs)
        code, *ref = O.mha_normalbp(cfg, B, T, *Ws, x, tgt, 1, 0.01)
        assert code == 0
        for g, r in zip(got[:5], ref[:5]):
            assert rel_err(g, r) < F32_TOL, seed
        assert got[0] is outs[0]
