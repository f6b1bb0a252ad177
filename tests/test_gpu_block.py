"""GPU parity of the transformer-block forwards around the MHA (RMSNorm, LayerNorm,
SwiGLU, Embedding), all through the C ABI: the reference entries against golden
vectors made by the reference itself, and the extension's resident / device entries
against the FP64 oracle on the same decoded weights."""
import numpy as np
import pytest

import oracle_py as O
import welvet_b200 as W
from conftest import rel_err
from test_block_oracle import block_cases, load_block

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4   # FP32 outputs vs the reference / FP64 oracle
LOW_TOL = 2e-2   # BF16 operands vs the oracle on the same bf16-rounded inputs


def _dev(torch, a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


@pytest.mark.parametrize("name", sorted(block_cases()))
def test_block_c_abi_matches_reference_golden(torch_cuda, name):
    c = block_cases()[name]
    g = load_block(name)
    kind, dt = c["kind"], c["dtype"]
    if kind in ("rmsnorm", "layernorm"):
        pre, post = W.norm_forward_f32(kind == "layernorm", c["batch"], c["seq"], c["dim"], c["eps"], g["gamma"],
                                       g["x"], beta=g["beta"], dtype=dt)
    elif kind == "swiglu":
        pre, post = W.swiglu_forward_f32(c["batch"], c["seq"], g["Gate"], g["Up"], g["Down"], g["x"], dtype=dt)
    else:
        pre, post = W.embedding_forward_f32(c["batch"], c["vocab"], c["emb"], c["seq_len"], c["in_rank"],
                                            c["in_last"], c["act"], g["W"], g["x"], dtype=dt)
    assert rel_err(pre, g["pre"]) < F32_TOL
    assert rel_err(post, g["post"]) < F32_TOL


@pytest.mark.parametrize("layernorm", [False, True])
@pytest.mark.parametrize("rows,dim,mean", [(64, 4096, 0.0), (37, 1000, 30.0), (300, 64, 0.0), (5, 1, 2.0),
                                           (3, 8192, -4.0), (2, 1030, 0.0)])
def test_norm_device_entry_against_oracle(torch_cuda, layernorm, rows, dim, mean):
    torch = torch_cuda
    rng = np.random.default_rng(rows * 7 + dim)
    x = (rng.standard_normal((rows, dim)) * 2 + mean).astype(np.float32)
    gam = (rng.standard_normal(dim) * 0.2 + 1).astype(np.float32)
    bet = (rng.standard_normal(dim) * 0.1).astype(np.float32)
    rpre, rpost = O.norm_forward(layernorm, x, gam, bet, 1e-5)
    xd, gd, bd = _dev(torch, x), _dev(torch, gam), _dev(torch, bet)
    pre, post = torch.empty_like(xd), torch.empty_like(xd)
    W.norm_forward(layernorm, rows, dim, 1e-5, gd, xd, pre, post, beta=bd)
    torch.cuda.synchronize()
    W.device_check()
    assert rel_err(pre.cpu().numpy(), rpre) < 1e-6   # FP64 statistics: ~1 ulp
    assert rel_err(post.cpu().numpy(), rpost) < 1e-6
    # BF16 activations in and out, pre omitted
    xb = xd.to(torch.bfloat16)
    postb = torch.empty_like(xb)
    W.norm_forward(layernorm, rows, dim, 1e-5, gd, xb, None, postb, beta=bd, io_bf16=1)
    torch.cuda.synchronize()
    _, rpost_b = O.norm_forward(layernorm, xb.float().cpu().numpy(), gam, bet, 1e-5)
    assert rel_err(postb.float().cpu().numpy(), rpost_b) < LOW_TOL


@pytest.mark.parametrize("d,inter,tokens,dtype", [(512, 1376, 256, 1), (30, 50, 7, 9), (128, 256, 1, 26),
                                                  (1024, 2816, 640, 3)])
def test_swiglu_resident_fp32_against_oracle(torch_cuda, d, inter, tokens, dtype):
    """FP32 layer (3xTF32 tensor-core GEMMs, SiLU*up fused in the Gate|Up epilogue),
    including the zero padding of input_dim to 4 and intermediate_dim to 32."""
    torch = torch_cuda
    a = (6.0 / (d + inter)) ** 0.5
    Gt = W.synthetic(inter * d, 21, 0, a).reshape(inter, d)
    Up = W.synthetic(inter * d, 22, 0, a).reshape(inter, d)
    Dn = W.synthetic(d * inter, 23, 0, a).reshape(d, inter)
    x = W.synthetic(tokens * d, 24, 1, 1.0).reshape(tokens, d)
    dec = [O.roundtrip(dtype, w).reshape(w.shape) for w in (Gt, Up, Dn)]
    rpre, rpost = O.swiglu_forward(x, *dec)
    layer = W.SwigluLayer(Gt, Up, Dn, dtype=dtype, precision=0)
    xd = _dev(torch, x)
    pre = torch.empty(tokens, inter, device="cuda")
    post = torch.empty(tokens, d, device="cuda")
    layer.forward(tokens, xd, pre, post)
    torch.cuda.synchronize()
    W.device_check()
    assert rel_err(pre.cpu().numpy(), rpre) < F32_TOL
    assert rel_err(post.cpu().numpy(), rpost) < F32_TOL
    # host-buffer path of the same layer
    hpre = np.zeros(tokens * inter, np.float32)
    _, hpost = layer.forward_host(tokens, x, hpre)
    assert rel_err(hpre, rpre.ravel()) < F32_TOL and rel_err(hpost, rpost.ravel()) < F32_TOL
    layer.close()


def test_swiglu_resident_bf16_against_oracle(torch_cuda):
    torch = torch_cuda
    d, inter, tokens = 1024, 2816, 512
    a = (6.0 / (d + inter)) ** 0.5
    Ws = [W.synthetic(inter * d, 31 + i, 0, a).reshape(inter, d) for i in range(2)]
    Ws.append(W.synthetic(d * inter, 33, 0, a).reshape(d, inter))
    x = W.synthetic(tokens * d, 34, 1, 1.0).reshape(tokens, d)
    layer = W.SwigluLayer(*Ws, dtype=1, precision=1)
    xb = _dev(torch, x, torch.bfloat16)
    pre = torch.empty(tokens, inter, device="cuda", dtype=torch.bfloat16)
    post = torch.empty(tokens, d, device="cuda", dtype=torch.bfloat16)
    layer.forward(tokens, xb, pre, post)
    torch.cuda.synchronize()
    W.device_check()
    bf = lambda w: torch.from_numpy(w).to(torch.bfloat16).float().numpy()  # noqa: E731
    rpre, rpost = O.swiglu_forward(xb.float().cpu().numpy(), *[bf(w) for w in Ws])
    assert rel_err(pre.float().cpu().numpy(), rpre) < LOW_TOL
    assert rel_err(post.float().cpu().numpy(), rpost) < LOW_TOL
    layer.close()


@pytest.mark.parametrize("act", [-1, 0, 1, 2, 3, 4, 5, 6])
def test_embedding_device_entry_against_oracle(torch_cuda, act):
    torch = torch_cuda
    vocab, emb, tokens = 5000, 256, 3000
    Wt = W.synthetic(vocab * emb, 41, 1, 1.5).reshape(vocab, emb)
    ids = np.floor(W.synthetic(tokens, 42, 0, 4.0 * vocab)).astype(np.float32)
    ids[::7] += np.float32(0.5)
    ids[:4] = [-0.0, -1.5, 3e9, -3e9]   # beyond int32: saturated, still inside the table
    rpre, _ = O.embedding_forward(ids[4:], Wt, 1, act)
    out = torch.empty(tokens, emb, device="cuda")
    W.embedding_forward(tokens, vocab, emb, 1, act, _dev(torch, Wt), _dev(torch, ids), out)
    torch.cuda.synchronize()
    W.device_check()
    got = out.cpu().numpy()
    assert rel_err(got[4:], rpre) < 1e-6
    assert np.isfinite(got[:4]).all()
    outb = torch.empty(tokens, emb, device="cuda", dtype=torch.bfloat16)
    W.embedding_forward(tokens, vocab, emb, 1, act, _dev(torch, Wt), _dev(torch, ids), outb, out_bf16=1)
    torch.cuda.synchronize()
    assert rel_err(outb.float().cpu().numpy()[4:], rpre) < LOW_TOL


def test_embedding_unaligned_rows_and_rank3(torch_cuda):
    # emb 13 takes the scalar path; rank 3 reads the id from the first of in_last values
    vocab, emb, B, T = 77, 13, 2, 5
    Wt = W.synthetic(vocab * emb, 51, 1, 1.0).reshape(vocab, emb)
    x = W.synthetic(B * T * emb, 52, 0, 300.0)
    pre, post = W.embedding_forward_f32(B, vocab, emb, T, 3, emb, 4, Wt, x, dtype=1)
    rpre, _ = O.embedding_forward(x, Wt, emb, 4)
    assert rel_err(pre, rpre.ravel()) < 1e-6 and np.array_equal(pre, post)
