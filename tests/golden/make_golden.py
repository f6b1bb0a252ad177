"""Generates tests/golden/*.npz from the REFERENCE ITSELF: oracle/_ref/libwelvet_ref.so
is the reference's own src/layers/mha/mha.cpp, src/layers/dense/dense.cpp,
src/weights/*.cpp, src/core/float_codecs.cpp and its soft-double shaders
(shaders/welvet_dense.metal, ops_common.metal, ops_mha.metal) compiled for the CPU
(recipe: oracle/Makefile `ref` target). Run here, where the reference sources exist:

    make -C oracle ref && python tests/golden/make_golden.py

Weights are regenerated at test time from the counter-based Xavier stream
(welvet_b200.xavier_weights, seed 0 — integer arithmetic, platform independent);
inputs x are stored, since the normal stream goes through libm.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "welvet.metal_b200"))

import oracle_py as O  # noqa: E402
from welvet_b200 import synthetic, xavier_weights  # noqa: E402

# name: (config kwargs, batch, seq, dtype)
MHA_CASES = {
    "cfg1_tiny_f32": (dict(d_model=64, num_heads=4), 1, 16, 1),
    "gqa_stream": (dict(d_model=64, num_heads=4, num_kv_heads=2), 2, 8, 1),
    "ring_wrap": (dict(d_model=64, num_heads=4, max_seq_len=16), 3, 8, 1),
    "bidir_alibi": (dict(d_model=64, num_heads=4, mask=2, pos=2), 2, 8, 1),
    "window_ropealibi_sigmoid": (dict(d_model=64, num_heads=4, mask=3, pos=3, window=3, softmax=1), 2, 8, 1),
    "prefix_nopos_fp8": (dict(d_model=64, num_heads=4, mask=4, prefix_len=5, pos=1), 1, 16, 4),
    "nf4": (dict(d_model=64, num_heads=4), 1, 16, 26),
    "bf16": (dict(d_model=64, num_heads=4), 1, 16, 3),
    "f16": (dict(d_model=64, num_heads=4), 2, 8, 2),
    "e5m2": (dict(d_model=64, num_heads=4), 1, 12, 5),
    "f64": (dict(d_model=64, num_heads=4), 1, 12, 0),
    "hd64_two_seq": (dict(d_model=128, num_heads=2, max_seq_len=64), 2, 32, 1),
    "hd128": (dict(d_model=256, num_heads=2, max_seq_len=64), 1, 24, 1),
    "hd64_gqa_window": (dict(d_model=256, num_heads=4, num_kv_heads=2, mask=3, window=7, max_seq_len=64), 1, 40, 1),
    # integer / sub-byte FormatNone dtypes (native_codec.cpp:189-870)
    "int64": (dict(d_model=64, num_heads=4), 1, 8, 6),
    "int32": (dict(d_model=64, num_heads=4), 1, 8, 7),
    "int8_gqa": (dict(d_model=64, num_heads=4, num_kv_heads=2), 2, 8, 9),
    "uint8": (dict(d_model=64, num_heads=4), 1, 8, 13),
    "uint64": (dict(d_model=64, num_heads=4), 1, 8, 10),
    "int4": (dict(d_model=64, num_heads=4), 1, 8, 14),
    "uint4": (dict(d_model=64, num_heads=4), 1, 8, 15),
    "fp4": (dict(d_model=64, num_heads=4), 1, 8, 16),
    "uint2_causal_window": (dict(d_model=64, num_heads=4, mask=3, window=4), 1, 12, 18),
    "ternary": (dict(d_model=64, num_heads=4), 1, 8, 19),
    "binary": (dict(d_model=64, num_heads=4), 1, 8, 20),
    "fp6_bidir": (dict(d_model=64, num_heads=4, mask=2), 1, 8, 27),
    "uint5": (dict(d_model=64, num_heads=4), 1, 8, 31),
    "int3": (dict(d_model=64, num_heads=4), 1, 8, 32),
}

# Transformer-block forwards (reference C entries welvet_{rmsnorm,layernorm,swiglu,
# embedding}_forward_f32). name: (kind, params); inputs are stored with the outputs.
BLOCK_CASES = {
    "rms_d64_f32": ("rmsnorm", dict(batch=2, seq=8, dim=64, eps=0.0, dtype=1)),
    "rms_d4096_bf16": ("rmsnorm", dict(batch=1, seq=4, dim=4096, eps=1e-5, dtype=3)),
    "rms_seq1_int8": ("rmsnorm", dict(batch=3, seq=1, dim=96, eps=0.0, dtype=9)),
    "ln_d64_f32": ("layernorm", dict(batch=2, seq=8, dim=64, eps=0.0, dtype=1)),
    "ln_d1000_nf4": ("layernorm", dict(batch=1, seq=5, dim=1000, eps=1e-3, dtype=26)),
    "ln_offset_mean": ("layernorm", dict(batch=1, seq=4, dim=256, eps=0.0, dtype=1, mean=100.0)),
    "swiglu_f32": ("swiglu", dict(batch=2, seq=8, input_dim=64, intermediate_dim=176, dtype=1)),
    "swiglu_seq1_fp8": ("swiglu", dict(batch=4, seq=1, input_dim=32, intermediate_dim=96, dtype=4)),
    "swiglu_int4": ("swiglu", dict(batch=1, seq=6, input_dim=48, intermediate_dim=128, dtype=14)),
    "emb_rank2_linear": ("embedding", dict(batch=2, vocab=50, emb=32, seq_len=6, in_rank=2, in_last=1, act=-1,
                                           dtype=1)),
    "emb_rank1_silu_int8": ("embedding", dict(batch=1, vocab=17, emb=24, seq_len=9, in_rank=1, in_last=1, act=1,
                                              dtype=9)),
    "emb_rank3_gelu": ("embedding", dict(batch=2, vocab=40, emb=16, seq_len=3, in_rank=3, in_last=16, act=2,
                                         dtype=1)),
    "emb_rank2_leaky_bf16": ("embedding", dict(batch=3, vocab=1000, emb=64, seq_len=5, in_rank=2, in_last=1, act=5,
                                               dtype=3)),
}


# MHA NormalBP leaf (reference welvet_mha_normalbp_f32): name: (config kwargs, batch,
# seq, dtype, use_target, lr). Weights from the Xavier stream (seed 0); x, the target
# / gradient and every output are stored.
NBP_CASES = {
    "nbp_tiny_sgd": (dict(d_model=16, num_heads=2), 1, 8, 1, 1, 0.01),
    "nbp_stream2_sgd": (dict(d_model=16, num_heads=2), 2, 6, 1, 1, 0.01),
    "nbp_gqa_gradout": (dict(d_model=32, num_heads=4, num_kv_heads=2), 2, 5, 1, 0, 0.0),
    "nbp_alibi_sgd": (dict(d_model=16, num_heads=2, pos=2), 2, 4, 1, 1, 0.02),
    "nbp_ropealibi_bidir": (dict(d_model=16, num_heads=2, pos=3, mask=2), 2, 4, 1, 1, 0.0),
    "nbp_ring_wrap_sgd": (dict(d_model=16, num_heads=2, max_seq_len=8), 3, 6, 1, 1, 0.01),
    "nbp_window_bf16": (dict(d_model=24, num_heads=2, mask=3), 2, 7, 3, 1, 0.0),
    "nbp_prefix_nopos_int8": (dict(d_model=16, num_heads=2, mask=4, pos=1), 2, 5, 9, 0, 0.0),
}


def block_inputs(kind, p, seed):
    """Deterministic inputs of a block case (counter-based stream, platform independent
    up to libm in the normal transform; stored in the fixture)."""
    if kind in ("rmsnorm", "layernorm"):
        n = p["batch"] * p["seq"] * p["dim"]
        x = synthetic(n, seed, 1, 1.0) + np.float32(p.get("mean", 0.0))
        g = synthetic(p["dim"], seed + 1, 1, 0.1) + np.float32(1.0)
        b = synthetic(p["dim"], seed + 2, 1, 0.1)
        return dict(x=x.astype(np.float32), gamma=g.astype(np.float32), beta=b)
    if kind == "swiglu":
        d, h = p["input_dim"], p["intermediate_dim"]
        a = (6.0 / (d + h)) ** 0.5
        return dict(x=synthetic(p["batch"] * p["seq"] * d, seed, 1, 1.0),
                    Gate=synthetic(h * d, seed + 1, 0, a).reshape(h, d),
                    Up=synthetic(h * d, seed + 2, 0, a).reshape(h, d),
                    Down=synthetic(d * h, seed + 3, 0, a).reshape(d, h))
    tokens = p["batch"] * p["seq_len"] if p["in_rank"] > 1 else p["seq_len"]
    ids = np.floor(synthetic(tokens * p["in_last"], seed, 0, 3.0 * p["vocab"])).astype(np.float32)
    ids[::5] += np.float32(0.75)  # fractional ids truncate toward zero
    return dict(x=ids, W=synthetic(p["vocab"] * p["emb"], seed + 1, 1, 1.0).reshape(p["vocab"], p["emb"]))


def block_run(kind, p, inp):
    if kind in ("rmsnorm", "layernorm"):
        return O.ref_norm_forward(kind == "layernorm", p["batch"], p["seq"], p["dim"], p["eps"], inp["gamma"],
                                  inp["x"], beta=inp["beta"], dtype=p["dtype"])
    if kind == "swiglu":
        return O.ref_swiglu_forward(p["batch"], p["seq"], inp["Gate"], inp["Up"], inp["Down"], inp["x"],
                                    dtype=p["dtype"])
    return O.ref_embedding_forward(p["batch"], p["vocab"], p["emb"], p["seq_len"], p["in_rank"], p["in_last"],
                                   p["act"], inp["W"], inp["x"], dtype=p["dtype"])


# Extra matrices for the all-dtype round trips: positive absmax (Int32's
# out-of-range conversion), all zeros (absmax 0 and span 0), a constant.
def codec_matrices(w):
    wp = synthetic(8 * 64, 5, 0, 0.3).reshape(8, 64)
    wp[3, 7] = 1.5
    wp[5, 9] = -0.75
    return {"w": w, "wpos": wp, "wzero": np.zeros((4, 16), np.float32),
            "wconst": np.full((4, 16), 0.7, np.float32)}


def _save(path, **arrays):
    """Writes the npz only when its arrays changed, so a rerun leaves git clean."""
    if os.path.exists(path):
        old = dict(np.load(path))
        if old.keys() == arrays.keys() and all(
                old[k].dtype == np.asarray(v).dtype and old[k].shape == np.shape(v)
                and old[k].tobytes() == np.asarray(v).tobytes() for k, v in arrays.items()):
            return
    np.savez_compressed(path, **arrays)


def weights_for(cfg: O.MhaCfg):
    c = cfg.resolved()
    return xavier_weights(c.d_model, c.q_dim, c.kv_dim, seed=0)


def wsum(ws) -> str:
    h = hashlib.sha256()
    for w in ws:
        h.update(np.ascontiguousarray(w, np.float32).tobytes())
    return h.hexdigest()


def main():
    if not O.ref_available():
        raise SystemExit("oracle/_ref/libwelvet_ref.so missing: run `make -C oracle ref` first")
    out = {}
    for name, (kw, B, T, dtype) in MHA_CASES.items():
        cfg = O.MhaCfg(**kw)
        Wq, Wk, Wv, Wo = weights_for(cfg)
        x = synthetic(B * T * cfg.d_model, 1, 1, 1.0).reshape(B * T, cfg.d_model)
        code, msg, pre, post = O.ref_mha_forward(cfg, B, T, Wq, Wk, Wv, Wo, x, dtype)
        if code:
            raise SystemExit(f"{name}: reference returned {code} {msg}")
        out[name] = dict(cfg=kw, batch=B, seq=T, dtype=dtype, wsum=wsum((Wq, Wk, Wv, Wo)))
        _save(os.path.join(HERE, f"mha_{name}.npz"), x=x, pre=pre, post=post)
    with open(os.path.join(HERE, "mha_cases.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)

    nbp = {}
    for name, (kw, B, T, dt, ut, lr) in NBP_CASES.items():
        cfg = O.MhaCfg(**kw)
        Wq, Wk, Wv, Wo = weights_for(cfg)
        x = synthetic(B * T * cfg.d_model, 1, 1, 1.0)
        tgt = synthetic(B * T * cfg.d_model, 2, 1, 1.0)
        code, msg, pre, post, dX, dW, Wa, loss = O.ref_mha_normalbp(cfg, B, T, Wq, Wk, Wv, Wo, x, tgt, ut, lr,
                                                                    dtype=dt)
        if code:
            raise SystemExit(f"{name}: reference returned {code} {msg}")
        nbp[name] = dict(cfg=kw, batch=B, seq=T, dtype=dt, use_target=ut, lr=lr, wsum=wsum((Wq, Wk, Wv, Wo)))
        _save(os.path.join(HERE, f"{name}.npz"), x=x, target=tgt, pre=pre, post=post, dX=dX, dW=dW, W_after=Wa,
              loss=np.float64(loss))
    with open(os.path.join(HERE, "nbp_cases.json"), "w") as f:
        json.dump(nbp, f, indent=1, sort_keys=True)

    blocks = {}
    for i, (name, (kind, p)) in enumerate(BLOCK_CASES.items()):
        inp = block_inputs(kind, p, 100 + 10 * i)
        code, msg, pre, post = block_run(kind, p, inp)
        if code:
            raise SystemExit(f"{name}: reference returned {code} {msg}")
        blocks[name] = dict(kind=kind, **p)
        _save(os.path.join(HERE, f"block_{name}.npz"), pre=pre, post=post, **inp)
    with open(os.path.join(HERE, "block_cases.json"), "w") as f:
        json.dump(blocks, f, indent=1, sort_keys=True)

    # Codec known answers straight from the reference converters.
    lib = O.ref_lib()
    codes = np.arange(256, dtype=np.uint8)
    e4m3_dec = np.array([lib.ref_fp8e4m3_decode(int(b)) for b in codes], np.float32)
    e5m2_dec = np.array([lib.ref_fp8e5m2_decode(int(b)) for b in codes], np.float32)
    probes = np.array([0.0, -0.0, 1.0, -1.0, 1.0625, 1.0624, 448.0, 449.0, 500.0, -500.0, 0.01, 0.001953125,
                       0.0019, 0.015625, 0.0146, 0.5, 3.14159, -2.71828, 240.0, 1e-8, float("nan"),
                       float("inf"), -float("inf"), 57344.0, 60000.0, 1.5e-5, 6.1e-5, 65504.0, 70000.0,
                       1.00390625, 1.0078125, 0.33333334], np.float32)
    rng = np.random.default_rng(7)
    probes = np.concatenate([probes, (rng.standard_normal(2000) * np.exp(rng.uniform(-12, 8, 2000))).astype(np.float32)])
    e4m3_enc = np.array([lib.ref_fp8e4m3_encode(float(f)) for f in probes], np.uint8)
    e5m2_enc = np.array([lib.ref_fp8e5m2_encode(float(f)) for f in probes], np.uint8)
    bf16_enc = np.array([lib.ref_bf16_encode(float(f)) for f in probes], np.uint16)
    f16_enc = np.array([lib.ref_f16_encode(float(f)) for f in probes], np.uint16)
    # FormatNone matrix round trips (WeightStore::make + export_f32) of a 32x64 matrix.
    w = synthetic(32 * 64, 3, 1, 0.05).reshape(32, 64)
    w[0, :8] = [0.5, -0.25, 0.1, -1.0, 0.0, 2.0, -3.0, 1e-6]
    rt = {}
    for dt in (0, 1, 2, 3, 4, 5, 26):
        code, msg, native, scale, dec = O.ref_weight_roundtrip(dt, w)
        if code:
            raise SystemExit(f"roundtrip dtype {dt}: {code} {msg}")
        rt[f"native_{dt}"] = native
        rt[f"scale_{dt}"] = np.float32(scale)
        rt[f"dec_{dt}"] = dec
    # decode(encode(w)) of every FormatNone dtype 0-33 on each matrix.
    mats = codec_matrices(w)
    for mname, m in mats.items():
        for dt in range(34):
            code, msg, _, _, dec = O.ref_weight_roundtrip(dt, m)
            if code:
                raise SystemExit(f"roundtrip dtype {dt} on {mname}: {code} {msg}")
            rt[f"rt_{mname}_{dt}"] = dec
    mats.pop("w")
    _save(os.path.join(HERE, "codecs.npz"), e4m3_dec=e4m3_dec, e5m2_dec=e5m2_dec, probes=probes,
          e4m3_enc=e4m3_enc, e5m2_enc=e5m2_enc, bf16_enc=bf16_enc, f16_enc=f16_enc, w=w, **mats, **rt)
    print(f"wrote {len(MHA_CASES)} MHA cases, {len(BLOCK_CASES)} block cases and codecs.npz to {HERE}")


if __name__ == "__main__":
    main()
