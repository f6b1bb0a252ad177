"""welvet_b200_decode_attention_static: split-KV decode attention whose split
partials live in a fixed per-device array, so the call allocates nothing. It is
for callers that must not let a library allocate device memory while they decode:
a serving loop whose HBM is reserved up front by its own pool, or a framework whose
caching allocator accounts for all device memory.

The GPU tests call it through the C ABI on a paged KV cache built here (pages in
shuffled order) and compare each sequence's output with the FP64 oracle's
attention (oracle/, the reference's op_attention restated) over the same q/k/v
values: decoding the query at position L-1 over keys [0, L) is row L-1 of a
causal per-sequence attention. BF16 (tensor-core decode kernel) and FP32
(CUDA-core decode kernel) buffers, softmax and sigmoid scores, ALiBi, GQA and
ragged lengths. Two consecutive calls must both match (the array is reused and
need not start at zero). The file name sorts last so the calls also run after
every other GPU test in one session; each test builds its own inputs, so it
passes alone too.
"""
import ctypes as C

import numpy as np
import pytest

import oracle_py as O
import welvet_b200 as W
from conftest import rel_err

STATIC_FLOATS = 1 << 20  # WELVET_B200_DECODE_STATIC_FLOATS
TOL = 2e-2               # BF16 tolerance of the attention parity tests
TOL_F32 = 1e-4           # FP32 tolerance against the FP64 oracle


def _call(cfg, batch, max_ctx, q, ldq, k_pool, v_pool, bt, max_pages, ctx, out, ldo):
    return W.lib().welvet_b200_decode_attention_static(C.byref(cfg), batch, max_ctx, q, ldq, k_pool, v_pool, bt,
                                                       max_pages, ctx, out, ldo, None)


def test_rejects_without_launch():
    """Argument and size checks return before any device work (runs without a GPU)."""
    cfg = W.MhaConfig.make(128 * 128, 128, 16, precision=1, pos=1)
    dummy = 16  # never dereferenced: every call below is rejected on the host
    st = _call(cfg, 64, 1024, dummy, 128 * 128, dummy, dummy, dummy, 64, dummy, dummy, 128 * 128)
    assert st.code == 1 and b"static scratch" in st.message  # 64*128*130 floats > 2^20
    st = _call(cfg, 0, 1024, dummy, 128 * 128, dummy, dummy, dummy, 64, dummy, dummy, 128 * 128)
    assert st.code == 1
    st = _call(cfg, 2, 1024, dummy, 128 * 128, dummy, dummy, dummy, 63, dummy, dummy, 128 * 128)
    assert st.code == 1  # 63 pages of 16 tokens cannot hold 1024 keys
    win = W.MhaConfig.make(128 * 128, 128, 16, precision=1, pos=1, mask=3, window=64)
    st = _call(win, 2, 1024, dummy, 128 * 128, dummy, dummy, dummy, 64, dummy, dummy, 128 * 128)
    assert st.code == 2


def _paged(torch, kv, B, T, NK, hd, bt):
    """Token-major kv [B*T, NK*hd] -> page pool [pages, NK, 16, hd] through block table bt [B, pps]."""
    pool = torch.zeros(bt.numel(), NK, 16, hd, device="cuda", dtype=kv.dtype)
    t = torch.arange(T, device="cuda")
    for b in range(B):
        pool[bt[b, t // 16].long(), :, t % 16, :] = kv[b * T:(b + 1) * T].view(T, NK, hd)
    return pool


def _setup(torch, B, T, H, NK, hd, pos, seed, precision=1, softmax=0):
    cfg = W.MhaConfig.make(H * hd, H, NK, head_dim=hd, precision=precision, pos=pos, mask=1, max_seq_len=T,
                           softmax=softmax)
    dt = torch.bfloat16 if precision == 1 else torch.float32
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B * T, H * hd, device="cuda", generator=g).to(dt)
    k = torch.randn(B * T, NK * hd, device="cuda", generator=g).to(dt)
    v = torch.randn(B * T, NK * hd, device="cuda", generator=g).to(dt)
    pps = (T + 15) // 16
    bt = torch.randperm(B * pps, device="cuda", generator=g).view(B, pps).to(torch.int32).contiguous()
    return cfg, q, k, v, bt, _paged(torch, k, B, T, NK, hd, bt), _paged(torch, v, B, T, NK, hd, bt)


def _oracle_rows(q, k, v, B, T, H, NK, hd, pos, softmax, lens):
    """Row L-1 of each sequence's causal attention, by the FP64 oracle over the
    same (bf16-valued or FP32) q/k/v; only the first L rows of a sequence are fed."""
    out = []
    for b, L in enumerate(lens):
        cfg = O.MhaCfg(d_model=H * hd, num_heads=H, num_kv_heads=NK, head_dim=hd, max_seq_len=L, mask=1,
                       pos=pos, softmax=softmax, per_sequence=1)
        sl = slice(b * T, b * T + L)
        rows = O.attention(cfg, 1, L, q[sl].float().cpu().numpy(), k[sl].float().cpu().numpy(),
                           v[sl].float().cpu().numpy())
        out.append(rows[L - 1])
    return np.stack(out)


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,H,NK,hd,pos,lens,precision,softmax", [
    (3, 300, 8, 2, 128, 1, None, 1, 0),                   # GQA 4, no positional bias
    (4, 517, 16, 16, 64, 2, [517, 480, 33, 1], 1, 0),     # MHA, ALiBi, ragged lengths incl. a single key
    (2, 1024, 32, 4, 128, 1, [1024, 700], 1, 0),          # GQA 8
    (3, 400, 8, 4, 64, 2, [400, 129, 17], 0, 0),          # FP32 buffers: CUDA-core decode kernel, ALiBi
    (2, 333, 8, 2, 128, 1, [333, 64], 1, 1),              # sigmoid scores (BF16)
    (2, 200, 4, 4, 128, 1, [200, 31], 0, 1),              # sigmoid scores (FP32)
])
def test_matches_oracle_attention(torch_cuda, B, T, H, NK, hd, pos, lens, precision, softmax):
    torch = torch_cuda
    cfg, q, k, v, bt, kp, vp = _setup(torch, B, T, H, NK, hd, pos, seed=7, precision=precision, softmax=softmax)
    lens = lens or [T] * B
    want = _oracle_rows(q, k, v, B, T, H, NK, hd, pos, softmax, lens)
    rows = torch.tensor([b * T + L - 1 for b, L in enumerate(lens)], device="cuda")
    q_dec = q[rows].contiguous()
    ctx = torch.tensor(lens, device="cuda", dtype=torch.int32)
    tol = TOL if precision == 1 else TOL_F32
    for call in range(2):
        out = torch.full((B, H * hd), float("nan"), device="cuda", dtype=q.dtype)
        st = _call(cfg, B, T, q_dec.data_ptr(), H * hd, kp.data_ptr(), vp.data_ptr(), bt.data_ptr(), bt.shape[1],
                   ctx.data_ptr(), out.data_ptr(), H * hd)
        assert st.code == 0, st.message
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_err(got, want) < tol, f"call {call}: {rel_err(got, want)}"
    W.device_check()


@pytest.mark.gpu
def test_fewer_splits_when_default_does_not_fit(torch_cuda):
    """FP32 buffers (CUDA-core decode kernel), B=64 sequences, 64 heads of 128 over 8
    KV heads, 600 cached keys: the kernel's default of 2 splits needs 2*64*64*130 floats
    > 2^20, so the call runs with one split; checked against a float64 PyTorch
    softmax(q k^T) v of the same inputs."""
    torch = torch_cuda
    B, T, H, NK, hd = 64, 600, 64, 8, 128
    assert 2 * B * H * (hd + 2) > STATIC_FLOATS >= B * H * (hd + 2)
    cfg, q, k, v, bt, kp, vp = _setup(torch, B, T, H, NK, hd, pos=1, seed=11, precision=0)
    lens = [T - (b * 37) % 500 for b in range(B)]
    rows = torch.tensor([b * T + L - 1 for b, L in enumerate(lens)], device="cuda")
    q_dec = q[rows].contiguous()
    ctx = torch.tensor(lens, device="cuda", dtype=torch.int32)
    want = []
    for b, L in enumerate(lens):
        qb = q_dec[b].double().view(H, hd)
        kb = k[b * T:b * T + L].double().view(L, NK, hd).repeat_interleave(H // NK, dim=1)
        vb = v[b * T:b * T + L].double().view(L, NK, hd).repeat_interleave(H // NK, dim=1)
        s = torch.einsum("hd,lhd->hl", qb, kb) / hd ** 0.5
        want.append(torch.einsum("hl,lhd->hd", torch.softmax(s, dim=1), vb).reshape(-1).cpu().numpy())
    want = np.stack(want)
    for call in range(2):
        out = torch.full((B, H * hd), float("nan"), device="cuda", dtype=torch.float32)
        st = _call(cfg, B, T, q_dec.data_ptr(), H * hd, kp.data_ptr(), vp.data_ptr(), bt.data_ptr(), bt.shape[1],
                   ctx.data_ptr(), out.data_ptr(), H * hd)
        assert st.code == 0, st.message
        torch.cuda.synchronize()
        assert rel_err(out.cpu().numpy(), want) < TOL_F32, f"call {call}"
    W.device_check()
