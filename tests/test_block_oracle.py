"""CPU tests of the checker for the transformer-block forwards around the MHA
(RMSNorm, LayerNorm, SwiGLU, Embedding): the FP64 oracle (oracle/block_oracle.cpp)
against golden vectors made by the reference's own code (tests/golden/block_*.npz,
from oracle/_ref) and, where oracle/_ref exists, against the reference run live."""
import json
import os

import numpy as np
import pytest

import oracle_py as O
from conftest import GOLDEN, rel_err


def block_cases():
    with open(os.path.join(GOLDEN, "block_cases.json")) as f:
        return json.load(f)


def load_block(name):
    return dict(np.load(os.path.join(GOLDEN, f"block_{name}.npz")))


def oracle_block(case, g):
    """The oracle's (pre, post) for a golden block case, weights decoded as `dtype`."""
    dt, kind = case["dtype"], case["kind"]
    dec = lambda w: O.roundtrip(dt, w).reshape(np.shape(w))  # noqa: E731
    if kind in ("rmsnorm", "layernorm"):
        return O.norm_forward(kind == "layernorm", g["x"].reshape(-1, case["dim"]), dec(g["gamma"]),
                              dec(g["beta"]), case["eps"])
    if kind == "swiglu":
        return O.swiglu_forward(g["x"].reshape(-1, case["input_dim"]), dec(g["Gate"]), dec(g["Up"]),
                                dec(g["Down"]))
    return O.embedding_forward(g["x"], dec(g["W"]), case["in_last"], case["act"])


def ulps(a, b):
    """Distance in FP32 units in the last place; +0 and -0 count as equal (the
    soft-double product of a zero weight is +0 where IEEE gives -0)."""
    a = (np.ascontiguousarray(a, np.float32).ravel() + np.float32(0)).view(np.int32).astype(np.int64)
    b = (np.ascontiguousarray(b, np.float32).ravel() + np.float32(0)).view(np.int32).astype(np.int64)
    return np.abs(a - b)


@pytest.mark.parametrize("name", sorted(block_cases()))
def test_block_oracle_matches_reference_golden(name):
    case = block_cases()[name]
    g = load_block(name)
    pre, post = oracle_block(case, g)
    # IEEE double against the reference's float2 soft-double: equal after FP32
    # rounding except within ~2^-48 of a rounding boundary (at most 1 ulp).
    for got, ref in ((pre, g["pre"]), (post, g["post"])):
        u = ulps(got, ref)
        assert u.max() <= 1
        assert np.mean(u == 0) > 0.99


def test_layernorm_large_mean_is_not_cancelled():
    # mean 100, std 1: E[x^2] - mean^2 loses ~13 bits in FP32; the oracle (double)
    # matches the reference's soft-double to the last bit.
    case = block_cases()["ln_offset_mean"]
    g = load_block("ln_offset_mean")
    pre, _ = oracle_block(case, g)
    assert np.abs(pre.ravel()).max() < 5 and ulps(pre, g["pre"]).max() <= 1


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built (reference sources absent)")
@pytest.mark.parametrize("seed", [3, 4])
def test_block_oracle_matches_reference_live(seed):
    rng = np.random.default_rng(seed)
    dt = int(rng.choice([1, 3, 9, 16, 26, 31]))
    # norms
    B, T, D = 2, 3, int(rng.integers(1, 300))
    x = (rng.standard_normal(B * T * D) * 3 + rng.uniform(-5, 5)).astype(np.float32)
    gam = rng.standard_normal(D).astype(np.float32)
    bet = rng.standard_normal(D).astype(np.float32)
    for ln in (False, True):
        code, msg, pre, post = O.ref_norm_forward(ln, B, T, D, 1e-4, gam, x, beta=bet, dtype=dt)
        assert code == 0, msg
        p2, q2 = O.norm_forward(ln, x.reshape(-1, D), O.roundtrip(dt, gam), O.roundtrip(dt, bet), 1e-4)
        assert ulps(p2, pre).max() <= 1 and ulps(q2, post).max() <= 1
    # SwiGLU
    d, h = int(rng.integers(1, 40)), int(rng.integers(1, 60))
    Ws = [rng.standard_normal(s).astype(np.float32) * 0.3 for s in ((h, d), (h, d), (d, h))]
    xs = rng.standard_normal(B * T * d).astype(np.float32)
    code, msg, pre, post = O.ref_swiglu_forward(B, T, *Ws, xs, dtype=dt)
    assert code == 0, msg
    p2, q2 = O.swiglu_forward(xs.reshape(-1, d), *[O.roundtrip(dt, w).reshape(w.shape) for w in Ws])
    assert ulps(p2, pre).max() <= 1 and ulps(q2, post).max() <= 1
    # Embedding, every activation
    V, E = int(rng.integers(1, 30)), int(rng.integers(1, 20))
    W = rng.standard_normal((V, E)).astype(np.float32) * 2
    ids = (rng.uniform(-3 * V, 3 * V, B * T)).astype(np.float32)
    for act in (-1, 0, 1, 2, 3, 4, 5, 6):
        code, msg, pre, post = O.ref_embedding_forward(B, V, E, T, 2, 1, act, W, ids, dtype=dt)
        assert code == 0, msg
        p2, _ = O.embedding_forward(ids, O.roundtrip(dt, W).reshape(W.shape), 1, act)
        if act == 2:
            # GELU's 1 + tanh(u) cancels for u << 0: the soft-double tanh is exact to
            # ~2^-48 absolute, so tiny outputs differ in many ulps; the tolerance metric
            # (relative to the largest output) sees ~1e-14.
            assert rel_err(p2.ravel(), pre) < 1e-6
        else:
            assert ulps(p2, pre).max() <= 1, act
