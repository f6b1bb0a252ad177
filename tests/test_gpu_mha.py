"""GPU parity tests of the whole MHA forward through the C ABI:
  * welvet_mha_forward_f32 (the drop-in entry of include/welvet_c.h) against the
    golden outputs of the reference's own code (tests/golden) — FP32, 1e-4;
  * the resident extension layer (FP32 3xTF32 and BF16 / FP8 / NF4 weights) against
    the FP64 oracle on the same (dequantised) weights — 1e-4 / 2e-2;
  * KV-cache prefill + split-KV decode against the oracle's decode."""
import numpy as np
import pytest

import oracle_py as O
import welvet_b200 as W
from conftest import bf16_round, golden_cases, load_golden, rel_err

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4   # FP32 outputs vs the FP64-accumulated reference
LOW_TOL = 2e-2   # BF16 / FP8 / NF4 paths vs the oracle on the same dequantised weights


@pytest.mark.parametrize("name", sorted(golden_cases()))
def test_c_abi_forward_matches_reference_golden(torch_cuda, name):
    case = golden_cases()[name]
    kw = case["cfg"]
    cfg = O.MhaCfg(**kw)
    c = cfg.resolved()
    Wq, Wk, Wv, Wo = W.xavier_weights(c.d_model, c.q_dim, c.kv_dim, seed=0)
    g = load_golden(name)
    if kw.get("softmax", 0) or kw.get("window", 0) or kw.get("prefix_len", 0):
        # not settable through welvet_mha_forward_f32: use the extension layer with
        # the reference's stream semantics
        lc = W.MhaConfig.make(c.d_model, c.num_heads, kw.get("num_kv_heads", 0), seq_mode=0,
                              **{k: v for k, v in kw.items() if k not in ("d_model", "num_heads", "num_kv_heads")})
        layer = W.MhaLayer(lc, Wq, Wk, Wv, Wo, dtype=case["dtype"])
        M = case["batch"] * case["seq"]
        pre = np.zeros((M, c.q_dim), np.float32)
        post = np.zeros((M, c.d_model), np.float32)
        layer.forward(case["batch"], case["seq"], g["x"], pre, post)
        layer.close()
    else:
        pre, post = W.mha_forward_f32(case["batch"], case["seq"], c.d_model, c.num_heads,
                                      kw.get("num_kv_heads", 0), 0, kw.get("max_seq_len", 0), kw.get("mask", 1),
                                      kw.get("pos", 0), case["dtype"], Wq, Wk, Wv, Wo, g["x"])
    assert rel_err(pre.reshape(g["pre"].shape), g["pre"]) < F32_TOL
    assert rel_err(post.reshape(g["post"].shape), g["post"]) < F32_TOL


def _layer_case(torch, kw, B, T, dtype=1, precision=0, weight_format=0):
    kw = dict(kw)
    d, H, NK = kw.pop("d_model"), kw.pop("num_heads"), kw.pop("num_kv_heads", 0)
    cfg = W.MhaConfig.make(d, H, NK, precision=precision, weight_format=weight_format, **kw)
    hd, nk = cfg.resolved()
    if weight_format == 0:
        Wq, Wk, Wv, Wo = W.xavier_weights(d, H * hd, nk * hd, seed=0)
    else:
        shapes = [(H * hd, d), (nk * hd, d), (nk * hd, d), (d, H * hd)]
        off, ws = 0, []
        for r, cc in shapes:
            ws.append(W.synthetic(r * cc, 0, 1, 0.02, off).reshape(r, cc))
            off += r * cc
        Wq, Wk, Wv, Wo = ws
    x = W.synthetic(B * T * d, 1, 1, 1.0).reshape(B * T, d)
    return cfg, (Wq, Wk, Wv, Wo), x, hd, nk


def _oracle_weights(Ws, dtype, weight_format):
    out = []
    for w in Ws:
        if weight_format == 1:
            out.append(O.fp8_rowscale(w)[2])
        elif weight_format == 2:
            out.append(O.nf4_block(w, 64)[2])
        else:
            out.append(O.roundtrip(dtype, w).reshape(w.shape))
    return out


RESIDENT_CASES = [
    (dict(d_model=256, num_heads=4, seq_mode=1), 2, 256),                   # hd 64 (cfg 2 shape class)
    (dict(d_model=256, num_heads=2, seq_mode=1), 2, 200),                   # hd 128
    (dict(d_model=512, num_heads=8, num_kv_heads=2, seq_mode=1), 3, 130),   # GQA
    (dict(d_model=256, num_heads=4, seq_mode=0, max_seq_len=512), 3, 100),  # stream semantics
]


@pytest.mark.parametrize("kw,B,T", RESIDENT_CASES)
def test_resident_fp32_layer(torch_cuda, kw, B, T):
    cfg, Ws, x, hd, nk = _layer_case(torch_cuda, kw, B, T)
    layer = W.MhaLayer(cfg, *Ws, dtype=1)
    M = B * T
    pre = np.zeros((M, cfg.num_heads * hd), np.float32)
    post = np.zeros((M, cfg.d_model), np.float32)
    layer.forward(B, T, x, pre, post)
    oc = O.MhaCfg(d_model=cfg.d_model, num_heads=cfg.num_heads, num_kv_heads=nk, max_seq_len=cfg.max_seq_len,
                  per_sequence=cfg.seq_mode)
    rpre, rpost = O.mha_forward(oc, B, T, *Ws, x)
    assert rel_err(pre, rpre) < F32_TOL
    assert rel_err(post, rpost) < F32_TOL


@pytest.mark.parametrize("weight_format", [0, 1, 2])
@pytest.mark.parametrize("kw,B,T", RESIDENT_CASES[:3])
def test_resident_bf16_layer(torch_cuda, kw, B, T, weight_format):
    torch = torch_cuda
    cfg, Ws, x, hd, nk = _layer_case(torch, kw, B, T, precision=1, weight_format=weight_format)
    layer = W.MhaLayer(cfg, *Ws, dtype=1)
    M = B * T
    xb = torch.from_numpy(x).cuda().to(torch.bfloat16)
    pre = torch.zeros(M, cfg.num_heads * hd, device="cuda", dtype=torch.bfloat16)
    post = torch.zeros(M, cfg.d_model, device="cuda", dtype=torch.bfloat16)
    layer.forward(B, T, xb, pre, post)
    torch.cuda.synchronize()
    layer.check_device()
    oc = O.MhaCfg(d_model=cfg.d_model, num_heads=cfg.num_heads, num_kv_heads=nk, per_sequence=1)
    rpre, rpost = O.mha_forward(oc, B, T, *_oracle_weights(Ws, 1, weight_format), xb.float().cpu().numpy())
    assert rel_err(pre.float().cpu().numpy(), rpre) < LOW_TOL
    assert rel_err(post.float().cpu().numpy(), rpost) < LOW_TOL


def test_bf16_weights_dtype3_truncation(torch_cuda):
    """dtype 3 (BF16 storage) truncates like float32_to_bfloat16 (float_codecs.cpp:53)."""
    cfg, Ws, x, hd, nk = _layer_case(torch_cuda, dict(d_model=128, num_heads=2, seq_mode=1), 1, 64)
    layer = W.MhaLayer(cfg, *Ws, dtype=3)
    pre = np.zeros((64, 128), np.float32)
    post = np.zeros((64, 128), np.float32)
    layer.forward(1, 64, x, pre, post)
    oc = O.MhaCfg(d_model=128, num_heads=2, per_sequence=1)
    rpre, rpost = O.mha_forward(oc, 1, 64, *_oracle_weights(Ws, 3, 0), x)
    assert rel_err(post, rpost) < F32_TOL


@pytest.mark.parametrize("precision", [1, 0])
def test_prefill_then_decode_against_oracle(torch_cuda, precision):
    torch = torch_cuda
    d, H, NK, B, L = 512, 8, 2, 4, 100
    cfg = W.MhaConfig.make(d, H, NK, precision=precision)
    hd, nk = cfg.resolved()
    Ws = W.xavier_weights(d, H * hd, nk * hd, seed=0)
    layer = W.MhaLayer(cfg, *Ws, dtype=1)
    kv = W.KvCache(layer, B, 256)
    dt = torch.bfloat16 if precision else torch.float32
    x = torch.from_numpy(W.synthetic(B * (L + 3) * d, 1, 1, 1.0).reshape(B, L + 3, d)).cuda().to(dt)
    xp = x[:, :L].contiguous().reshape(B * L, d)
    post = torch.zeros(B * L, d, device="cuda", dtype=dt)
    layer.prefill(kv, B, L, xp, None, post)
    oc = O.MhaCfg(d_model=d, num_heads=H, num_kv_heads=NK, per_sequence=1)
    Wd = _oracle_weights(Ws, 1, 0)
    tol = LOW_TOL if precision else F32_TOL
    for step in range(3):
        xn = x[:, L + step].contiguous()
        dpost = torch.zeros(B, d, device="cuda", dtype=dt)
        dpre = torch.zeros(B, H * hd, device="cuda", dtype=dt)
        layer.decode(kv, B, xn, dpre, dpost)
        torch.cuda.synchronize()
        layer.check_device()
        # oracle: full per-sequence forward over L+step+1 tokens, last row
        n = L + step + 1
        xf = x[:, :n].float().cpu().numpy().reshape(B * n, d)
        rpre, rpost = O.mha_forward(oc, B, n, *Wd, xf)
        last = rpost.reshape(B, n, d)[:, -1]
        assert rel_err(dpost.float().cpu().numpy(), last) < tol, f"step {step}"


def test_decode_gqa_against_oracle_decode(torch_cuda):
    """Decode with a cache filled directly (GQA decode shape class: 32/8 heads x 64)."""
    torch = torch_cuda
    d, H, NK, B, L = 512, 8, 2, 6, 333
    cfg = W.MhaConfig.make(d, H, NK, precision=1)
    hd, nk = cfg.resolved()
    Ws = W.xavier_weights(d, H * hd, nk * hd, seed=0)
    layer = W.MhaLayer(cfg, *Ws, dtype=1)
    kv = W.KvCache(layer, B, 512)
    kc = (W.synthetic(B * L * nk * hd, 2, 1, 0.5).reshape(B, L, nk * hd))
    vc = (W.synthetic(B * L * nk * hd, 2, 1, 0.5, offset=B * L * nk * hd).reshape(B, L, nk * hd))
    kcb = torch.from_numpy(kc).cuda().to(torch.bfloat16)
    vcb = torch.from_numpy(vc).cuda().to(torch.bfloat16)
    kv.fill(B, L, kcb, vcb)
    x = torch.from_numpy(W.synthetic(B * d, 1, 1, 1.0).reshape(B, d)).cuda().to(torch.bfloat16)
    post = torch.zeros(B, d, device="cuda", dtype=torch.bfloat16)
    pre = torch.zeros(B, H * hd, device="cuda", dtype=torch.bfloat16)
    layer.decode(kv, B, x, pre, post)
    torch.cuda.synchronize()
    layer.check_device()
    oc = O.MhaCfg(d_model=d, num_heads=H, num_kv_heads=NK, per_sequence=1)
    rpre, rpost, _, _ = O.mha_decode(oc, [L] * B, kcb.float().cpu().numpy(), vcb.float().cpu().numpy(),
                                     *Ws, x.float().cpu().numpy())
    assert rel_err(pre.float().cpu().numpy(), rpre) < LOW_TOL
    assert rel_err(post.float().cpu().numpy(), rpost) < LOW_TOL


def test_head_shards_sum_to_full_layer(torch_cuda):
    """Two head shards on one GPU: the sum of their row-sharded O projections
    equals the unsharded layer (what the NCCL all-reduce computes across GPUs)."""
    torch = torch_cuda
    d, H, B, T = 256, 4, 2, 64
    Ws = W.xavier_weights(d, d, d, seed=0)
    x = torch.from_numpy(W.synthetic(B * T * d, 1, 1, 1.0).reshape(B * T, d)).cuda()
    full = W.MhaLayer(W.MhaConfig.make(d, H, 0), *Ws)
    post = torch.zeros(B * T, d, device="cuda")
    full.forward(B, T, x, None, post)
    acc = torch.zeros_like(post)
    for s in range(2):
        part = W.MhaLayer(W.MhaConfig.make(d, H, 0, head_begin=2 * s, head_count=2), *Ws)
        p = torch.zeros_like(post)
        part.forward(B, T, x, None, p)
        acc += p
    torch.cuda.synchronize()
    assert rel_err(acc.cpu().numpy(), post.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("precision", [0, 1])
def test_chunked_forward_with_communicator(torch_cuda, precision):
    """With a communicator attached (one rank here) the layer runs the batch in chunks
    whose all-reduce overlaps the next chunk's compute. Every row is computed by the
    same kernels over the same K loop, so the output equals the unchunked layer bit
    for bit; the host-buffer path stages pre and post of every chunk."""
    torch = torch_cuda
    d, H, NK, B, T = 256, 4, 2, 6, 96
    Ws = W.xavier_weights(d, d, NK * d // H, seed=0)
    dt = torch.float32 if precision == 0 else torch.bfloat16
    x = torch.from_numpy(W.synthetic(B * T * d, 1, 1, 1.0).reshape(B * T, d)).cuda().to(dt)
    cfg = W.MhaConfig.make(d, H, NK, precision=precision)
    plain = W.MhaLayer(cfg, *Ws)
    chunked = W.MhaLayer(cfg, *Ws)
    chunked.attach_comm(W.comm_unique_id(), 1, 0)
    outs = []
    for layer in (plain, chunked):
        pre = torch.zeros(B * T, d, device="cuda", dtype=dt)
        post = torch.zeros(B * T, d, device="cuda", dtype=dt)
        layer.forward(B, T, x, pre, post)
        torch.cuda.synchronize()
        outs.append((pre.float().cpu().numpy(), post.float().cpu().numpy()))
    assert np.array_equal(outs[0][0], outs[1][0])
    assert np.array_equal(outs[0][1], outs[1][1])
    xh = x.cpu()
    pre_h = torch.zeros(B * T, d, dtype=dt)
    post_h = torch.zeros(B * T, d, dtype=dt)
    for layer in (chunked, plain):  # host buffers: copies of chunk i+1 / i-1 overlap chunk i
        pre_h.zero_()
        post_h.zero_()
        layer.forward(B, T, xh, pre_h, post_h)
        assert np.array_equal(pre_h.float().numpy(), outs[0][0])
        assert np.array_equal(post_h.float().numpy(), outs[0][1])
    chunked.check_device()
    chunked.close()
    plain.close()


@pytest.mark.parametrize("H,NK,pos,softmax", [
    (8, 2, 2, 0),   # GQA 4, head_dim 64, ALiBi
    (8, 2, 0, 1),   # sigmoid scores, RoPE
    (4, 4, 3, 0),   # MHA, head_dim 128, RoPE + ALiBi
    (2, 1, 0, 0),   # GQA 2, head_dim 256
])
def test_decode_variants_against_oracle(torch_cuda, H, NK, pos, softmax):
    """The paged decode kernel (TMA page rings + m16n8k16 MMAs) on the position
    encodings and score functions of the reference, through the layer's decode."""
    torch = torch_cuda
    d, B, L = 512, 3, 150
    cfg = W.MhaConfig.make(d, H, NK, precision=1, pos=pos, softmax=softmax)
    hd, nk = cfg.resolved()
    Ws = W.xavier_weights(d, H * hd, nk * hd, seed=0)
    layer = W.MhaLayer(cfg, *Ws, dtype=1)
    kv = W.KvCache(layer, B, 256)
    n = B * L * nk * hd
    kcb = torch.from_numpy(W.synthetic(n, 2, 1, 0.5).reshape(B, L, nk * hd)).cuda().to(torch.bfloat16)
    vcb = torch.from_numpy(W.synthetic(n, 2, 1, 0.5, offset=n).reshape(B, L, nk * hd)).cuda().to(torch.bfloat16)
    kv.fill(B, L, kcb, vcb)
    x = torch.from_numpy(W.synthetic(B * d, 1, 1, 1.0).reshape(B, d)).cuda().to(torch.bfloat16)
    post = torch.zeros(B, d, device="cuda", dtype=torch.bfloat16)
    pre = torch.zeros(B, H * hd, device="cuda", dtype=torch.bfloat16)
    layer.decode(kv, B, x, pre, post)
    torch.cuda.synchronize()
    layer.check_device()
    oc = O.MhaCfg(d_model=d, num_heads=H, num_kv_heads=NK, pos=pos, softmax=softmax, per_sequence=1)
    rpre, rpost, _, _ = O.mha_decode(oc, [L] * B, kcb.float().cpu().numpy(), vcb.float().cpu().numpy(),
                                     *Ws, x.float().cpu().numpy())
    assert rel_err(pre.float().cpu().numpy(), rpre) < LOW_TOL
    assert rel_err(post.float().cpu().numpy(), rpost) < LOW_TOL


@pytest.mark.parametrize("precision", [0, 1])
def test_forward_rows_one_rank_equals_host_forward(torch_cuda, precision):
    """welvet_b200_mha_forward_rows with a communicator of one rank is the host-buffer
    forward of the caller's sequences: same chunks, same kernels, equal bit for bit."""
    torch = torch_cuda
    d, H, NK, B, T = 256, 4, 2, 6, 96
    Ws = W.xavier_weights(d, d, NK * d // H, seed=0)
    dt = torch.float32 if precision == 0 else torch.bfloat16
    x = torch.from_numpy(W.synthetic(B * T * d, 1, 1, 1.0).reshape(B * T, d)).to(dt).pin_memory()
    cfg = W.MhaConfig.make(d, H, NK, precision=precision)
    plain = W.MhaLayer(cfg, *Ws)
    rows = W.MhaLayer(cfg, *Ws)
    rows.attach_comm(W.comm_unique_id(), 1, 0)
    want = torch.zeros(B * T, d, dtype=dt).pin_memory()
    got = torch.zeros(B * T, d, dtype=dt).pin_memory()
    plain.forward(B, T, x, None, want)
    rows.forward_rows(B, T, x, got)
    assert torch.equal(want, got)


@pytest.mark.parametrize("dtype", [9, 14, 16])  # Int8, Int4, FP4 codes resident (weight_format 3)
def test_resident_formatnone_code_layer(torch_cuda, dtype):
    """The reference's FormatNone codes kept resident and dequantised inside the
    GEMM mainloop, against the oracle on the reference-decoded weights of the same
    dtype (decode(encode(w)), per tensor) and the same bf16 inputs; GQA head shard."""
    torch = torch_cuda
    d, H, NK, B, T = 512, 8, 2, 2, 160
    cfg = W.MhaConfig.make(d, H, NK, precision=1, weight_format=3, seq_mode=1)
    hd, nk = cfg.resolved()
    Ws = W.xavier_weights(d, H * hd, nk * hd, seed=0)
    if dtype == 16:
        Ws = [w * np.float32(8.0) for w in Ws]  # FP4 has no scale: use its range
    layer = W.MhaLayer(cfg, *Ws, dtype=dtype)
    # (FP4 weights are 8x larger: the input is 8x smaller so that the logits, and
    # with them the softmax's sensitivity to the BF16 rounding of q and k, stay as
    # for the other dtypes)
    x = W.synthetic(B * T * d, 1, 1, 0.125 if dtype == 16 else 1.0).reshape(B * T, d)
    xb = torch.from_numpy(x).cuda().to(torch.bfloat16)
    pre = torch.zeros(B * T, H * hd, device="cuda", dtype=torch.bfloat16)
    post = torch.zeros(B * T, d, device="cuda", dtype=torch.bfloat16)
    layer.forward(B, T, xb, pre, post)
    torch.cuda.synchronize()
    layer.check_device()
    oc = O.MhaCfg(d_model=d, num_heads=H, num_kv_heads=nk, per_sequence=1)
    deq = [O.roundtrip(dtype, w).reshape(w.shape) for w in Ws]
    rpre, rpost = O.mha_forward(oc, B, T, *deq, xb.float().cpu().numpy())
    assert rel_err(pre.float().cpu().numpy(), rpre) < LOW_TOL
    assert rel_err(post.float().cpu().numpy(), rpost) < LOW_TOL
    layer.close()


@pytest.mark.parametrize("weight_format,dtype", [(0, 1), (1, 1), (2, 1), (3, 9), (3, 14)])
def test_decode_split_k_weight_formats(torch_cuda, weight_format, dtype):
    """Decode projections at few rows split their K range over the SMs (FP32 partials
    summed in split order, then scale, RoPE and the BF16 store); every resident weight
    format, against the oracle's decode on the decoded weights."""
    torch = torch_cuda
    d, H, NK, B, L = 1024, 16, 4, 5, 70
    cfg = W.MhaConfig.make(d, H, NK, precision=1, weight_format=weight_format)
    hd, nk = cfg.resolved()
    Ws = W.xavier_weights(d, H * hd, nk * hd, seed=3)
    layer = W.MhaLayer(cfg, *Ws, dtype=dtype)
    kv = W.KvCache(layer, B, 128)
    kc = W.synthetic(B * L * nk * hd, 2, 1, 0.5).reshape(B, L, nk * hd)
    vc = W.synthetic(B * L * nk * hd, 2, 1, 0.5, offset=B * L * nk * hd).reshape(B, L, nk * hd)
    kcb = torch.from_numpy(kc).cuda().to(torch.bfloat16)
    vcb = torch.from_numpy(vc).cuda().to(torch.bfloat16)
    kv.fill(B, L, kcb, vcb)
    x = torch.from_numpy(W.synthetic(B * d, 1, 1, 1.0).reshape(B, d)).cuda().to(torch.bfloat16)
    post = torch.zeros(B, d, device="cuda", dtype=torch.bfloat16)
    pre = torch.zeros(B, H * hd, device="cuda", dtype=torch.bfloat16)
    layer.decode(kv, B, x, pre, post)
    torch.cuda.synchronize()
    layer.check_device()
    oc = O.MhaCfg(d_model=d, num_heads=H, num_kv_heads=NK, per_sequence=1)
    rpre, rpost, _, _ = O.mha_decode(oc, [L] * B, kcb.float().cpu().numpy(), vcb.float().cpu().numpy(),
                                     *_oracle_weights(Ws, dtype, weight_format), x.float().cpu().numpy())
    assert rel_err(pre.float().cpu().numpy(), rpre) < LOW_TOL
    assert rel_err(post.float().cpu().numpy(), rpost) < LOW_TOL
    layer.close()


@pytest.mark.parametrize("d,H,NK,B", [(2048, 16, 4, 20), (1536, 12, 12, 33), (512, 8, 2, 64)])
def test_decode_gemv_shapes(torch_cuda, d, H, NK, B):
    """BF16 decode projections through the weight-streaming GEMV (K a multiple of
    512): head_dim 128 and 64 RoPE pairs inside the 128-column tiles, batch rows
    padded to the MMA's N (32, 48, 64), K split over clusters of 4, 3... 1 CTAs, the
    K/V rows appended to the cache pages in the epilogue; against the oracle's
    decode, two steps (the second reads the first step's appended rows)."""
    torch = torch_cuda
    L = 40
    cfg = W.MhaConfig.make(d, H, NK, precision=1)
    hd, nk = cfg.resolved()
    Ws = W.xavier_weights(d, H * hd, nk * hd, seed=5)
    layer = W.MhaLayer(cfg, *Ws, dtype=1)
    kv = W.KvCache(layer, B, 64)
    n = B * L * nk * hd
    kc = torch.from_numpy(W.synthetic(n, 2, 1, 0.5).reshape(B, L, nk * hd)).cuda().to(torch.bfloat16)
    vc = torch.from_numpy(W.synthetic(n, 2, 1, 0.5, offset=n).reshape(B, L, nk * hd)).cuda().to(torch.bfloat16)
    kv.fill(B, L, kc, vc)
    oc = O.MhaCfg(d_model=d, num_heads=H, num_kv_heads=NK, per_sequence=1)
    kcn, vcn = kc.float().cpu().numpy(), vc.float().cpu().numpy()
    Wb = _oracle_weights(Ws, 1, 0)
    for step in range(2):
        x = torch.from_numpy(W.synthetic(B * d, 40 + step, 1, 1.0).reshape(B, d)).cuda().to(torch.bfloat16)
        post = torch.zeros(B, d, device="cuda", dtype=torch.bfloat16)
        pre = torch.zeros(B, H * hd, device="cuda", dtype=torch.bfloat16)
        layer.decode(kv, B, x, pre, post)
        torch.cuda.synchronize()
        layer.check_device()
        rpre, rpost, kn, vn = O.mha_decode(oc, [L + step] * B, kcn, vcn, *Wb, x.float().cpu().numpy())
        assert rel_err(pre.float().cpu().numpy(), rpre) < LOW_TOL, step
        assert rel_err(post.float().cpu().numpy(), rpost) < LOW_TOL, step
        kcn = np.concatenate([kcn, bf16_round(kn)[:, None, :]], axis=1)
        vcn = np.concatenate([vcn, bf16_round(vn)[:, None, :]], axis=1)
    layer.close()
