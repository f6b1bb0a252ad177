"""Parity at the benchmark configurations' own shapes (not shape classes): the
kernels run at the full stated size and rows of their output are compared with
the FP64 oracle on the same (dequantised) weights and inputs. Causal attention
makes rows [0, n) of a sequence depend on its tokens [0, n) only, so a row slice of
the full-size run is checked against an oracle run of that prefix.

  cfg2: FP32 prefill B=8 T=2048 d=1024 16x64 (3xTF32 projections, FP32
        attention) -- sequences 0 and 7, every row, 1e-4.
  cfg3: BF16 decode, 64 sequences over a 4096-token paged KV cache, GQA 32/8 x 64
        -- one decode step, sequences 0, 31 and 63, 2e-2.
  cfg4: prefill B=4 T=4096 d=4096 32x128 with FP8 row-scale and NF4 block-64
        weights -- sequence 0 tokens 0..1023 and sequence 3 tokens 0..511, 2e-2.
  cfg5 head shape at T=8192: the tensor-core flash kernel over one 8192-token
        sequence (64 key blocks: lazy rescale and the merge of the two
        warpgroups' partial softmaxes), every row of two heads, 2e-2.
"""
import numpy as np
import pytest

import oracle_py as O
import welvet_b200 as W
from conftest import bf16_round, rel_err

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4
LOW_TOL = 2e-2


def _weights(torch, d, H, NK, hd, quantised):
    """Device FP32 weights from the bench's counter stream (Xavier-uniform, or
    N(0, 0.02) for the quantised configurations) and their host copies."""
    shapes = [(H * hd, d), (NK * hd, d), (NK * hd, d), (d, H * hd)]
    ws, off = [], 0
    for r, c in shapes:
        t = torch.empty(r, c, device="cuda", dtype=torch.float32)
        W.fill_synthetic(t, 0, 1 if quantised else 0, 0.02 if quantised else (6.0 / (r + c)) ** 0.5, offset=off)
        off += r * c
        ws.append(t)
    torch.cuda.synchronize()
    return ws, [t.cpu().numpy() for t in ws]


def test_cfg2_fp32_full_shape(torch_cuda):
    torch = torch_cuda
    B, T, d, H = 8, 2048, 1024, 16
    hd = d // H
    ws, host = _weights(torch, d, H, H, hd, False)
    layer = W.MhaLayer(W.MhaConfig.make(d, H, H, precision=0, seq_mode=1), *ws, dtype=1)
    x = torch.empty(B * T, d, device="cuda")
    W.fill_synthetic(x, 1, 1, 1.0)
    pre = torch.empty(B * T, d, device="cuda")
    post = torch.empty(B * T, d, device="cuda")
    layer.forward(B, T, x, pre, post)
    torch.cuda.synchronize()
    layer.check_device()
    oc = O.MhaCfg(d_model=d, num_heads=H, max_seq_len=T, per_sequence=1)
    for b in (0, B - 1):
        rows = slice(b * T, (b + 1) * T)
        rpre, rpost = O.mha_forward(oc, 1, T, *host, x[rows].cpu().numpy())
        assert rel_err(pre[rows].cpu().numpy(), rpre) < F32_TOL, b
        assert rel_err(post[rows].cpu().numpy(), rpost) < F32_TOL, b
    layer.close()


def test_cfg3_decode_full_shape(torch_cuda):
    torch = torch_cuda
    B, L, d, H, NK = 64, 4096, 2048, 32, 8
    hd = d // H
    kd = NK * hd
    ws, host = _weights(torch, d, H, NK, hd, False)
    layer = W.MhaLayer(W.MhaConfig.make(d, H, NK, precision=1, seq_mode=1), *ws, dtype=1)
    kv = W.KvCache(layer, B, L + 16)
    kc = torch.empty(B, L, kd, device="cuda", dtype=torch.bfloat16)
    vc = torch.empty(B, L, kd, device="cuda", dtype=torch.bfloat16)
    W.fill_synthetic(kc, 2, 1, 0.5, offset=0)
    W.fill_synthetic(vc, 2, 1, 0.5, offset=kc.numel())
    kv.fill(B, L, kc, vc)
    x = torch.empty(B, d, device="cuda", dtype=torch.bfloat16)
    W.fill_synthetic(x, 1, 1, 1.0)
    pre = torch.empty(B, H * hd, device="cuda", dtype=torch.bfloat16)
    post = torch.empty(B, d, device="cuda", dtype=torch.bfloat16)
    layer.decode(kv, B, x, pre, post)
    torch.cuda.synchronize()
    layer.check_device()
    sel = [0, 31, 63]
    oc = O.MhaCfg(d_model=d, num_heads=H, num_kv_heads=NK, max_seq_len=L + 1, per_sequence=1)
    rpre, rpost, _, _ = O.mha_decode(oc, [L] * len(sel), kc[sel].float().cpu().numpy(),
                                     vc[sel].float().cpu().numpy(), *[bf16_round(w) for w in host],
                                     x[sel].float().cpu().numpy())
    assert rel_err(pre[sel].float().cpu().numpy(), rpre) < LOW_TOL
    assert rel_err(post[sel].float().cpu().numpy(), rpost) < LOW_TOL
    kv.close()
    layer.close()


@pytest.mark.parametrize("weight_format", [1, 2])
def test_cfg4_quantised_full_shape(torch_cuda, weight_format):
    torch = torch_cuda
    B, T, d, H = 4, 4096, 4096, 32
    hd = d // H
    ws, host = _weights(torch, d, H, H, hd, True)
    layer = W.MhaLayer(W.MhaConfig.make(d, H, H, precision=1, weight_format=weight_format, seq_mode=1), *ws,
                       dtype=1)
    del ws
    x = torch.empty(B * T, d, device="cuda", dtype=torch.bfloat16)
    W.fill_synthetic(x, 1, 1, 1.0)
    pre = torch.empty(B * T, d, device="cuda", dtype=torch.bfloat16)
    post = torch.empty(B * T, d, device="cuda", dtype=torch.bfloat16)
    layer.forward(B, T, x, pre, post)
    torch.cuda.synchronize()
    layer.check_device()
    deq = [O.fp8_rowscale(w)[2] if weight_format == 1 else O.nf4_block(w, 64)[2] for w in host]
    for b, n in ((0, 1024), (3, 512)):
        rows = slice(b * T, b * T + n)
        oc = O.MhaCfg(d_model=d, num_heads=H, max_seq_len=n, per_sequence=1)
        rpre, rpost = O.mha_forward(oc, 1, n, *deq, x[rows].float().cpu().numpy())
        assert rel_err(pre[rows].float().cpu().numpy(), rpre) < LOW_TOL, b
        assert rel_err(post[rows].float().cpu().numpy(), rpost) < LOW_TOL, b
    layer.close()


@pytest.mark.parametrize("impl", [2, 3, 4])  # persistent; CTA pairs (M = 256 UMMAs); one CTA per tile
def test_cfg5_heads_tensor_core_attention_at_8192(torch_cuda, impl):
    torch = torch_cuda
    T, H, hd = 8192, 2, 128
    cfg = W.MhaConfig.make(H * hd, H, H, precision=1, pos=1, seq_mode=1, max_seq_len=T)
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(T, H * hd, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(T, H * hd, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(T, H * hd, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.empty_like(q)
    W.attention(cfg, 1, T, q, k, v, out, impl=impl)
    torch.cuda.synchronize()
    W.device_check()
    oc = O.MhaCfg(d_model=H * hd, num_heads=H, max_seq_len=T, pos=1, per_sequence=1)
    want = O.attention(oc, 1, T, q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy())
    got = out.float().cpu().numpy()
    assert rel_err(got, want) < LOW_TOL
    # the last 128 rows see all 64 key blocks: check them on their own scale too
    assert rel_err(got[-128:], want[-128:]) < LOW_TOL
