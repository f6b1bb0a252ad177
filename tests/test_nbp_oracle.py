"""CPU tests of the checker for the MHA NormalBP leaf (welvet_mha_normalbp_f32:
forward, MSE, backward, SGD): the FP64 oracle (oracle_mha_normalbp) against golden
vectors made by the reference's own code (tests/golden/nbp_*.npz, from oracle/_ref)
and, where oracle/_ref exists, against the reference run live."""
import json
import os

import numpy as np
import pytest

import oracle_py as O
from conftest import GOLDEN
from golden.make_golden import wsum
from welvet_b200 import synthetic, xavier_weights


def nbp_cases():
    with open(os.path.join(GOLDEN, "nbp_cases.json")) as f:
        return json.load(f)


def load_nbp(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


def ulps(a, b):
    a = (np.ascontiguousarray(a, np.float32).ravel() + np.float32(0)).view(np.int32).astype(np.int64)
    b = (np.ascontiguousarray(b, np.float32).ravel() + np.float32(0)).view(np.int32).astype(np.int64)
    return np.abs(a - b)


def oracle_case(case, g):
    cfg = O.MhaCfg(**case["cfg"])
    c = cfg.resolved()
    Ws = xavier_weights(c.d_model, c.q_dim, c.kv_dim, seed=0)
    assert wsum(Ws) == case["wsum"], "weight stream drifted from the fixture"
    dec = [O.roundtrip(case["dtype"], w).reshape(w.shape) for w in Ws]
    return O.mha_normalbp(cfg, case["batch"], case["seq"], *dec, g["x"], g["target"], case["use_target"],
                          case["lr"], sgd_f32=case["dtype"] == 1)


@pytest.mark.parametrize("name", sorted(nbp_cases()))
def test_nbp_oracle_matches_reference_golden(name):
    case = nbp_cases()[name]
    g = load_nbp(name)
    code, pre, post, dX, dW, Wa, loss = oracle_case(case, g)
    assert code == 0
    # IEEE double against the reference's float2 soft-double: equal after FP32
    # rounding except within ~2^-48 of a rounding boundary.
    for got, key in ((pre, "pre"), (post, "post"), (dX, "dX"), (dW, "dW"), (Wa, "W_after")):
        u = ulps(got, g[key])
        assert u.max() <= 1, key
        assert np.mean(u == 0) > 0.99, key
    assert abs(loss - float(g["loss"])) <= 1e-12 * max(abs(float(g["loss"])), 1e-30)


def test_nbp_stream_quirk_keys_of_earlier_batches_are_zero():
    # In the reference's backward the key/value ring is cleared per batch, so a later
    # batch's recomputed softmax sees earlier positions as zero keys: its gradients
    # differ from those of a per-batch independent backward. The golden two-batch
    # case therefore does not equal twice the one-batch case.
    case = nbp_cases()["nbp_stream2_sgd"]
    g = load_nbp("nbp_stream2_sgd")
    assert np.abs(g["dX"]).max() > 0 and case["batch"] == 2


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built (reference sources absent)")
@pytest.mark.parametrize("seed", [5, 6])
def test_nbp_oracle_matches_reference_live(seed):
    rng = np.random.default_rng(seed)
    H = int(rng.choice([1, 2, 4]))
    kw = dict(d_model=8 * H, num_heads=H, mask=int(rng.choice([1, 2, 3])), pos=int(rng.choice([0, 1, 2, 3])),
              max_seq_len=int(rng.choice([0, 6])))
    B, T = int(rng.integers(1, 4)), int(rng.integers(2, 7))
    cfg = O.MhaCfg(**kw)
    c = cfg.resolved()
    Ws = xavier_weights(c.d_model, c.q_dim, c.kv_dim, seed=seed)
    x = synthetic(B * T * c.d_model, seed, 1, 1.0)
    tgt = synthetic(B * T * c.d_model, seed + 1, 1, 1.0)
    lr = float(rng.choice([0.0, 0.05]))
    code, msg, pre, post, dX, dW, Wa, loss = O.ref_mha_normalbp(cfg, B, T, *Ws, x, tgt, 1, lr)
    assert code == 0, msg
    oc, p2, q2, dX2, dW2, Wa2, l2 = O.mha_normalbp(cfg, B, T, *Ws, x, tgt, 1, lr)
    assert oc == 0
    for got, ref in ((p2, pre), (q2, post), (dX2, dX), (dW2, dW), (Wa2, Wa)):
        assert ulps(got, ref).max() <= 1
