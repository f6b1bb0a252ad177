"""GPU parity tests of the individual sm_100a kernels, called through the C ABI
(libwelvet_b200.so) on device buffers: the tcgen05 GEMMs against a float64 torch
product of the same operands, the codec kernels bit-exactly against the
reference's own converters (tests/golden/codecs.npz) and the oracle, and the
attention kernels against the FP64 oracle."""
import numpy as np
import pytest

import oracle_py as O
import welvet_b200 as W
from conftest import GOLDEN, rel_err

pytestmark = pytest.mark.gpu


def _dev(torch, a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.to(dtype) if dtype is not None else t


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 512, 256), (1000, 768, 1024), (77, 1000, 512),
                                   (4096, 3072, 2048)])
def test_gemm_bf16_tcgen05(torch_cuda, M, N, K):
    torch = torch_cuda
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.empty(M, N, device="cuda", dtype=torch.float32)
    W.gemm(0, M, N, K, a, b, out, out_bf16=0)
    torch.cuda.synchronize()
    W.device_check()
    ref = a.double() @ b.double().T
    # FP32 accumulation of exact bf16 products: ~1e-6 relative
    assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) < 1e-5


def test_gemm_bf16_output_bf16(torch_cuda):
    torch = torch_cuda
    M, N, K = 512, 512, 512
    a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    b = torch.randn(N, K, device="cuda").to(torch.bfloat16)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    W.gemm(0, M, N, K, a, b, out, out_bf16=1)
    torch.cuda.synchronize()
    ref = (a.double() @ b.double().T)
    assert rel_err(out.float().cpu().numpy(), ref.cpu().numpy()) < 8e-3


@pytest.mark.parametrize("M,N,K", [(128, 128, 32), (333, 384, 1024), (2048, 1024, 1024)])
def test_gemm_tf32x3_is_fp32_accurate(torch_cuda, M, N, K):
    torch = torch_cuda
    torch.manual_seed(M * 7919 + N * 31 + K)  # inputs independent of the tests run before
    a = torch.randn(M, K, device="cuda", dtype=torch.float32)
    b = torch.randn(N, K, device="cuda", dtype=torch.float32)
    ah, al, bh, bl = (torch.empty_like(t) for t in (a, a, b, b))
    W.split_tf32(a, ah, al)
    W.split_tf32(b, bh, bl)
    torch.cuda.synchronize()
    assert torch.equal(ah + al, a) and torch.equal(bh + bl, b)
    out = torch.empty(M, N, device="cuda", dtype=torch.float32)
    W.gemm(1, M, N, K, ah, bh, out, a_lo=al, b_lo=bl)
    torch.cuda.synchronize()
    W.device_check()
    ref = a.double() @ b.double().T
    # The FP32 path's budget is 1e-4. 3xTF32 drops only lo*lo (2^-22 relative), but the
    # tensor-core accumulator does not round each addition to nearest: measured
    # 8e-6 to 1.02e-5 at K=1024 on B200 over different random draws, growing
    # ~linearly with K. The bound keeps a 2x margin and stays 5x inside the 1e-4
    # budget of the FP32 path.
    assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) < 2e-5 * max(1.0, K / 1024)


def test_gemm_fp8_rowscale_weights(torch_cuda):
    torch = torch_cuda
    M, N, K = 700, 512, 1024
    w = W.synthetic(N * K, 11, 1, 0.02).reshape(N, K)
    codes, scales, dec = O.fp8_rowscale(w)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    out = torch.empty(M, N, device="cuda", dtype=torch.float32)
    W.gemm(2, M, N, K, x, _dev(torch, codes), out, b_scale=_dev(torch, scales))
    torch.cuda.synchronize()
    W.device_check()
    ref = x.double() @ _dev(torch, dec).double().T
    assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) < 1e-5


def test_gemm_nf4_block_weights(torch_cuda):
    torch = torch_cuda
    M, N, K = 513, 768, 512
    w = W.synthetic(N * K, 12, 1, 0.02).reshape(N, K)
    packed, amax, dec = O.nf4_block(w, 64)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    out = torch.empty(M, N, device="cuda", dtype=torch.float32)
    W.gemm(3, M, N, K, x, _dev(torch, packed.reshape(N, K // 2)), out, b_scale=_dev(torch, amax))
    torch.cuda.synchronize()
    W.device_check()
    ref = x.double() @ _dev(torch, dec).double().T
    # weights are dequantised to bf16 in shared memory (2^-9 relative per weight)
    assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) < 4e-3


# ------------------------------------------------------------------- codecs
def test_codec_roundtrip_bitexact_against_reference(torch_cuda):
    torch = torch_cuda
    g = dict(np.load(f"{GOLDEN}/codecs.npz"))
    w = _dev(torch, g["w"].ravel())
    for dt in (0, 1, 2, 3, 4, 5, 26):
        out = torch.empty_like(w)
        W.codec_roundtrip(dt, w, out)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), g[f"dec_{dt}"].ravel().view(np.uint32),
                                      err_msg=f"dtype {dt}")


@pytest.mark.parametrize("dtype", range(34))
def test_codec_roundtrip_all_dtypes_bitexact(torch_cuda, dtype):
    """Device decode(encode(w)) of every FormatNone dtype against the reference's
    own round trips (golden) and, on a 3M-element tensor that spans many blocks of
    the statistics reduction, against the oracle port."""
    torch = torch_cuda
    g = dict(np.load(f"{GOLDEN}/codecs.npz"))
    for m in ("w", "wpos", "wzero", "wconst"):
        w = _dev(torch, g[m].ravel())
        out = torch.empty_like(w)
        W.codec_roundtrip(dtype, w, out)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), g[f"rt_{m}_{dtype}"].ravel().view(np.uint32),
                                      err_msg=f"{m} dtype {dtype}")
    big = W.synthetic(3 << 20, 11, 1, 0.05)
    big[123457] = 0.9      # positive absmax, far from block 0
    big[2999999] = -0.4    # minimum in the last block
    w = _dev(torch, big)
    out = torch.empty_like(w)
    W.codec_roundtrip(dtype, w, out)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), O.roundtrip(dtype, big).view(np.uint32))


def _nearest_value_edges():
    """Values at and one ulp either side of every midpoint of the NF4 levels and
    of the FP4 grid (where the reference's first-minimum scan breaks ties), plus
    the extremes where the FP4 scan's rounded errors tie or reach FLT_MAX."""
    nf4 = np.array([O.oracle_lib().oracle_nf4_level(c) for c in range(16)], np.float32)
    fp4 = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6], np.float32)
    vals = [0.0, -0.0, 1.0, -1.0]
    for grid in (fp4, -fp4, nf4):
        g = np.sort(grid)
        mids = ((g[:-1] + g[1:]) / np.float32(2)).astype(np.float32)
        for m in mids:
            vals += [m, np.nextafter(m, np.float32(np.inf)), np.nextafter(m, np.float32(-np.inf))]
    big = np.float32(3.4028235e38)
    vals += [6.0, 6.5, 7.0, 1e7, 16777216.0, 16777220.0, 3e38, big, -big, np.nextafter(big, np.float32(0)),
             1e-30, -1e-30, -6.5, -1e9]
    return np.array(vals, np.float32)


@pytest.mark.parametrize("dtype", [16, 26])
def test_codec_nearest_value_ties(torch_cuda, dtype):
    torch = torch_cuda
    v = _nearest_value_edges()
    if dtype == 26:
        v = np.clip(v, -1, 1).astype(np.float32)  # absmax 1: r = w exactly
    else:
        v = np.concatenate([v, np.array([np.inf, -np.inf, np.nan], np.float32)])
    v = np.tile(v, 5)  # vector body and tail
    for off in (0, 1):  # 16-byte aligned and element-aligned (scalar) paths
        w = torch.zeros(v.size + 1, dtype=torch.float32, device="cuda")
        w[off:off + v.size] = torch.from_numpy(v).cuda()
        out = torch.zeros_like(w)
        W.codec_roundtrip(dtype, w[off:off + v.size], out[off:off + v.size])
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out[off:off + v.size].cpu().numpy().view(np.uint32),
                                      O.roundtrip(dtype, v).view(np.uint32), err_msg=f"offset {off}")
    if dtype == 26:
        w = _dev(torch, v)
        packed = torch.empty((v.size + 1) // 2, dtype=torch.uint8, device="cuda")
        amax = torch.empty((v.size + 63) // 64, dtype=torch.float32, device="cuda")
        W.nf4_block_encode(w, packed, amax)
        torch.cuda.synchronize()
        p_o, a_o, _ = O.nf4_block(v, 64)
        np.testing.assert_array_equal(packed.cpu().numpy(), p_o)


def test_codec_encode_bytes_match_reference(torch_cuda):
    torch = torch_cuda
    g = dict(np.load(f"{GOLDEN}/codecs.npz"))
    w = _dev(torch, g["w"].ravel())
    n = w.numel()
    for dt, nbytes in ((0, 8 * n), (2, 2 * n), (3, 2 * n), (4, n), (5, n), (26, n // 2)):
        codes = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
        scale = torch.zeros(1, dtype=torch.float32, device="cuda")
        W.codec_encode(dt, w, codes, scale)
        dec = torch.empty_like(w)
        W.codec_decode(dt, codes, dec, scale)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(codes.cpu().numpy(), g[f"native_{dt}"], err_msg=f"dtype {dt}")
        np.testing.assert_array_equal(dec.cpu().numpy().view(np.uint32), g[f"dec_{dt}"].ravel().view(np.uint32))
        if dt == 26:
            assert scale.item() == g["scale_26"]


def test_codec_probe_values(torch_cuda):
    torch = torch_cuda
    g = dict(np.load(f"{GOLDEN}/codecs.npz"))
    p = _dev(torch, g["probes"])
    for dt, key, view in ((4, "e4m3_enc", np.uint8), (5, "e5m2_enc", np.uint8), (3, "bf16_enc", np.uint16),
                          (2, "f16_enc", np.uint16)):
        codes = torch.zeros(p.numel() * np.dtype(view).itemsize, dtype=torch.uint8, device="cuda")
        W.codec_encode(dt, p, codes)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(codes.cpu().numpy().view(view), g[key], err_msg=key)
    all_codes = torch.arange(256, dtype=torch.int32, device="cuda").to(torch.uint8)
    for dt, key in ((4, "e4m3_dec"), (5, "e5m2_dec")):
        out = torch.empty(256, dtype=torch.float32, device="cuda")
        W.codec_decode(dt, all_codes, out)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), g[key].view(np.uint32))


@pytest.mark.parametrize("rows,cols", [(96, 320), (7, 100), (64, 4096)])
def test_extension_formats_bitexact_against_oracle(torch_cuda, rows, cols):
    """(96, 320), (64, 4096): the vectorised decodes; (7, 100): the scalar ones."""
    torch = torch_cuda
    w = W.synthetic(rows * cols, 13, 1, 0.02).reshape(rows, cols)
    w[3, :] = 0.0  # all-zero row -> scale 1
    codes_o, scales_o, dec_o = O.fp8_rowscale(w)
    wd = _dev(torch, w)
    codes = torch.empty(rows, cols, dtype=torch.uint8, device="cuda")
    scales = torch.empty(rows, dtype=torch.float32, device="cuda")
    W.fp8_rowscale_encode(wd, codes, scales)
    dec = torch.empty(rows, cols, dtype=torch.float32, device="cuda")
    W.fp8_rowscale_decode(codes, scales, dec)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(codes.cpu().numpy(), codes_o)
    np.testing.assert_array_equal(scales.cpu().numpy(), scales_o)
    np.testing.assert_array_equal(dec.cpu().numpy(), dec_o)
    packed_o, amax_o, ndec_o = O.nf4_block(w, 64)
    packed = torch.empty((w.size + 1) // 2, dtype=torch.uint8, device="cuda")
    amax = torch.empty((w.size + 63) // 64, dtype=torch.float32, device="cuda")
    W.nf4_block_encode(wd, packed, amax)
    ndec = torch.empty(w.size, dtype=torch.float32, device="cuda")
    W.nf4_block_decode(packed, amax, ndec)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(packed.cpu().numpy(), packed_o)
    np.testing.assert_array_equal(amax.cpu().numpy(), amax_o)
    np.testing.assert_array_equal(ndec.cpu().numpy().reshape(rows, cols), ndec_o)
    # BF16 outputs: each FP32 value rounded to nearest even
    from conftest import bf16_round
    db = torch.empty(rows, cols, dtype=torch.bfloat16, device="cuda")
    W.fp8_rowscale_decode(codes, scales, db, out_bf16=1)
    nb = torch.empty(w.size, dtype=torch.bfloat16, device="cuda")
    W.nf4_block_decode(packed, amax, nb, out_bf16=1)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(db.float().cpu().numpy().view(np.uint32), bf16_round(dec_o).view(np.uint32))
    np.testing.assert_array_equal(nb.float().cpu().numpy().reshape(rows, cols).view(np.uint32),
                                  bf16_round(ndec_o).view(np.uint32))


# ---------------------------------------------------------------- attention
ATTN_CASES = [
    # (cfg kwargs, batch, seq)
    (dict(d_model=64, num_heads=4, seq_mode=1), 2, 40),
    (dict(d_model=256, num_heads=4, num_kv_heads=2, seq_mode=1), 2, 130),
    (dict(d_model=256, num_heads=2, seq_mode=1), 1, 257),                  # hd 128
    (dict(d_model=64, num_heads=4, seq_mode=0, max_seq_len=64), 3, 16),   # stream
    (dict(d_model=64, num_heads=4, seq_mode=0, max_seq_len=20), 3, 16),   # stream, ring wrap
    (dict(d_model=64, num_heads=4, seq_mode=1, mask=2, pos=2), 2, 33),
    (dict(d_model=64, num_heads=4, seq_mode=1, mask=3, window=5, softmax=1), 1, 50),
    (dict(d_model=64, num_heads=4, seq_mode=1, mask=3, window=6, window_causal=0), 1, 50),
    (dict(d_model=64, num_heads=4, seq_mode=0, mask=4, prefix_len=9, max_seq_len=64), 2, 20),
    (dict(d_model=48, num_heads=4, seq_mode=1), 2, 19),                   # hd 12
    (dict(d_model=1024, num_heads=8, seq_mode=1), 2, 1100),               # hd 128, 9 key blocks
    (dict(d_model=512, num_heads=8, num_kv_heads=2, seq_mode=1), 1, 777),  # hd 64, GQA
    (dict(d_model=256, num_heads=2, seq_mode=1, mask=2), 1, 300),         # bidirectional, hd 128
    (dict(d_model=256, num_heads=4, seq_mode=1, mask=3, window=200, pos=2), 1, 700),
]


@pytest.mark.parametrize("kw,B,T", ATTN_CASES)
# impl 2: the persistent tensor-core kernel (CTAs loop over query tiles); impl 4:
# the same pipeline with one CTA per query tile.
@pytest.mark.parametrize("precision,impl", [(0, 1), (1, 1), (1, 2), (1, 4)])
def test_attention_against_oracle(torch_cuda, kw, B, T, precision, impl):
    torch = torch_cuda
    kw = dict(kw)
    cfg = W.MhaConfig.make(kw.pop("d_model"), kw.pop("num_heads"), kw.pop("num_kv_heads", 0), precision=precision,
                           **kw)
    hd, nk = cfg.resolved()
    qd, kd = cfg.num_heads * hd, nk * hd
    M = B * T
    q = W.synthetic(M * qd, 21, 1, 1.0).reshape(M, qd)
    k = W.synthetic(M * kd, 22, 1, 1.0).reshape(M, kd)
    v = W.synthetic(M * kd, 23, 1, 1.0).reshape(M, kd)
    if precision == 1:  # the oracle sees the same bf16-rounded inputs
        q, k, v = (torch.from_numpy(a).to(torch.bfloat16).float().numpy() for a in (q, k, v))
    oc = O.MhaCfg(d_model=cfg.d_model, num_heads=cfg.num_heads, num_kv_heads=nk, head_dim=hd,
                  max_seq_len=cfg.max_seq_len, mask=cfg.mask, pos=1 if cfg.pos == 0 else cfg.pos,
                  softmax=cfg.softmax, window=cfg.window, prefix_len=cfg.prefix_len,
                  window_causal=cfg.window_causal, per_sequence=cfg.seq_mode)
    # the kernel receives rotated q/k; compare with RoPE off on both sides
    cfg.pos = oc.pos
    ref = O.attention(oc, B, T, q, k, v)
    dt = torch.float32 if precision == 0 else torch.bfloat16
    out = torch.zeros(M, qd, device="cuda", dtype=dt)
    try:
        W.attention(cfg, B, T, _dev(torch, q, dt), _dev(torch, k, dt), _dev(torch, v, dt), out, impl=impl)
    except W.WelvetError as e:
        if impl in (2, 4) and e.code == 2:
            pytest.skip("tensor-core kernel does not cover this head_dim / mode")
        raise
    torch.cuda.synchronize()
    W.device_check()
    tol = 1e-4 if precision == 0 else 2e-2
    assert rel_err(out.float().cpu().numpy(), ref) < tol


# FP32 attention on the tensor cores (3xTF32, head_dim 64) from the TF32 split of
# q, k, v: every case above that the kernel takes, plus long causal sequences
# (many 64-key blocks, lazy rescale and the two partial softmaxes merged), GQA,
# ALiBi with sigmoid scores, against the FP64 oracle within the FP32 budget 1e-4.
TF32_CASES = ATTN_CASES + [
    (dict(d_model=1024, num_heads=16, seq_mode=1), 1, 2048),               # the cfg2 head shape
    (dict(d_model=512, num_heads=8, num_kv_heads=2, seq_mode=1, pos=2, softmax=1), 2, 333),
    (dict(d_model=256, num_heads=4, seq_mode=1, mask=4, prefix_len=100), 1, 260),
]


@pytest.mark.parametrize("kw,B,T", TF32_CASES)
def test_attention_tf32_against_oracle(torch_cuda, kw, B, T):
    torch = torch_cuda
    kw = dict(kw)
    cfg = W.MhaConfig.make(kw.pop("d_model"), kw.pop("num_heads"), kw.pop("num_kv_heads", 0), precision=0, **kw)
    hd, nk = cfg.resolved()
    qd, kd = cfg.num_heads * hd, nk * hd
    M = B * T
    q = W.synthetic(M * qd, 21, 1, 1.0).reshape(M, qd)
    k = W.synthetic(M * kd, 22, 1, 1.0).reshape(M, kd)
    v = W.synthetic(M * kd, 23, 1, 1.0).reshape(M, kd)
    oc = O.MhaCfg(d_model=cfg.d_model, num_heads=cfg.num_heads, num_kv_heads=nk, head_dim=hd,
                  max_seq_len=cfg.max_seq_len, mask=cfg.mask, pos=1 if cfg.pos == 0 else cfg.pos,
                  softmax=cfg.softmax, window=cfg.window, prefix_len=cfg.prefix_len,
                  window_causal=cfg.window_causal, per_sequence=cfg.seq_mode)
    cfg.pos = oc.pos
    parts = []
    for a in (q, k, v):
        t = _dev(torch, a)
        hi, lo = torch.empty_like(t), torch.empty_like(t)
        W.split_tf32(t, hi, lo)
        parts += [hi, lo]
    out = torch.zeros(M, qd, device="cuda")
    oh, ol = torch.zeros_like(out), torch.zeros_like(out)
    try:
        W.attention_tf32(cfg, B, T, *parts, out, oh, ol)
    except W.WelvetError as e:
        if e.code == 2 and (hd != 64 or (cfg.seq_mode == 0 and B * T > cfg.max_seq_len)):
            pytest.skip("3xTF32 kernel: head_dim 64 without the stream ring wrap")
        raise
    torch.cuda.synchronize()
    W.device_check()
    ref = O.attention(oc, B, T, q, k, v)
    assert rel_err(out.cpu().numpy(), ref) < 1e-4
    assert torch.equal(oh + ol, out)
    assert not torch.any(oh.view(torch.int32) & 0x1FFF)


# CTA-pair tensor-core attention (impl 3: clusters of two CTAs, M = 256 UMMAs;
# head_dim 128, sequences of whole 256-query tile pairs): the masks, position
# biases and score functions of the reference, GQA, stream semantics, against the
# oracle on the same bf16-rounded inputs.
PAIR_CASES = [
    (dict(d_model=256, num_heads=2, seq_mode=1), 2, 512),                  # causal, 4 key blocks
    (dict(d_model=1024, num_heads=8, num_kv_heads=2, seq_mode=1), 1, 1280),  # GQA, 10 key blocks
    (dict(d_model=256, num_heads=2, seq_mode=1, mask=2), 1, 512),          # bidirectional
    (dict(d_model=256, num_heads=2, seq_mode=1, mask=3, window=200, pos=2), 1, 768),  # window + ALiBi
    (dict(d_model=256, num_heads=2, seq_mode=1, mask=3, window=130, window_causal=0, softmax=1), 1, 512),
    (dict(d_model=256, num_heads=2, seq_mode=0, max_seq_len=1024, mask=4, prefix_len=300), 2, 256),  # stream
    (dict(d_model=256, num_heads=2, seq_mode=1), 3, 256),                  # one pair per sequence
]


@pytest.mark.parametrize("kw,B,T", PAIR_CASES)
def test_attention_cta_pairs_against_oracle(torch_cuda, kw, B, T):
    torch = torch_cuda
    kw = dict(kw)
    cfg = W.MhaConfig.make(kw.pop("d_model"), kw.pop("num_heads"), kw.pop("num_kv_heads", 0), precision=1, **kw)
    hd, nk = cfg.resolved()
    assert hd == 128 and T % 256 == 0
    qd, kd = cfg.num_heads * hd, nk * hd
    M = B * T
    q, k, v = (torch.from_numpy(W.synthetic(M * n, s, 1, 1.0).reshape(M, n)).to(torch.bfloat16)
               for n, s in ((qd, 31), (kd, 32), (kd, 33)))
    oc = O.MhaCfg(d_model=cfg.d_model, num_heads=cfg.num_heads, num_kv_heads=nk, head_dim=hd,
                  max_seq_len=cfg.max_seq_len, mask=cfg.mask, pos=1 if cfg.pos == 0 else cfg.pos,
                  softmax=cfg.softmax, window=cfg.window, prefix_len=cfg.prefix_len,
                  window_causal=cfg.window_causal, per_sequence=cfg.seq_mode)
    cfg.pos = oc.pos
    ref = O.attention(oc, B, T, q.float().numpy(), k.float().numpy(), v.float().numpy())
    out = torch.zeros(M, qd, device="cuda", dtype=torch.bfloat16)
    W.attention(cfg, B, T, q.cuda(), k.cuda(), v.cuda(), out, impl=3)
    torch.cuda.synchronize()
    W.device_check()
    got = out.float().cpu().numpy()
    assert rel_err(got, ref) < 2e-2
    # both CTAs of every pair: rows of the even and the odd query tiles
    assert rel_err(got[:128], ref[:128]) < 2e-2 and rel_err(got[128:256], ref[128:256]) < 2e-2


# FormatNone codes dequantised inside the GEMM mainloop (kinds 4 Int8, 5 Int4, 6 FP4):
# every code value, two's-complement Int4 nibbles and the E2M1 levels of the
# reference's kFp4 table (float_codecs.cpp:184), low nibble first, with a per-row
# epilogue scale, against an FP64 product of the decoded weights.
FP4_LEVELS = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6], np.float32)


@pytest.mark.parametrize("kind", [4, 5, 6])
def test_gemm_formatnone_code_weights(torch_cuda, kind):
    torch = torch_cuda
    M, N, K = 700, 512, 1024
    rng = np.random.default_rng(kind)
    scale = (rng.random(N).astype(np.float32) + 0.5) * np.float32(0.01)
    if kind == 4:
        q = rng.integers(-128, 128, size=(N, K)).astype(np.int8)
        codes, dec = q.view(np.uint8), q.astype(np.float32) * scale[:, None]
    else:
        nib = rng.integers(0, 16, size=(N, K)).astype(np.uint8)
        codes = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
        lv = np.where(nib < 8, nib, nib.astype(np.int16) - 16).astype(np.float32) if kind == 5 else FP4_LEVELS[nib]
        if kind == 6:
            scale[:] = 1.0
        dec = lv * scale[:, None]
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    out = torch.empty(M, N, device="cuda", dtype=torch.float32)
    W.gemm(kind, M, N, K, x, _dev(torch, np.ascontiguousarray(codes)), out, b_scale=_dev(torch, scale))
    torch.cuda.synchronize()
    W.device_check()
    ref = x.double() @ _dev(torch, dec.astype(np.float32)).double().T
    # codes are exact in BF16 and the scale is applied once in FP32
    assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("dtype", [9, 14, 16])
def test_formatnone_code_encoder_bitexact_against_reference(torch_cuda, dtype):
    """The device encoder of the resident Int8 / Int4 / FP4 codes gives the
    reference's own pack_native bytes and scale (oracle/_ref, the reference's
    WeightStore compiled for the CPU), on a tensor with ties, zeros and extremes."""
    torch = torch_cuda
    if not O.ref_available():
        pytest.skip("oracle/_ref (the reference compiled for the CPU) not built")
    rows, cols = 64, 1000
    w = W.synthetic(rows * cols, 15, 1, 0.7 if dtype == 16 else 0.02).reshape(rows, cols)
    w[0, :8] = [0.0, -0.0, 1e-9, -1e-9, 0.25, -0.75, 7.0, -9.0]  # zeros, FP4 midpoints and clamps
    code, msg, native, scale, _ = O.ref_weight_roundtrip(dtype, w)
    assert code == 0, msg
    n = w.size
    codes = torch.empty(n if dtype == 9 else (n + 1) // 2, device="cuda", dtype=torch.uint8)
    sc = torch.empty(1, device="cuda", dtype=torch.float32)
    W.codec_encode(dtype, _dev(torch, w.reshape(-1)), codes, sc)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(codes.cpu().numpy(), native[:codes.numel()])
    if dtype != 16:
        assert sc.item() == np.float32(scale)
