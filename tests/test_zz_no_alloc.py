"""welvet_b200_decode_attention_static: split-KV decode attention whose split
partials live in a fixed per-device array, so the call allocates nothing.

The GPU tests call it through the C ABI on a paged KV cache built here (pages in
shuffled order) and compare each sequence's output with the row of the same query
position in the existing prefill attention entry point (welvet_b200_attention over
the same q/k/v, causal): decoding the query at position L-1 over keys [0, L)
is that row. Two consecutive calls must both match (the array is reused and need
not start at zero). The file name sorts last so the calls also run after every
other GPU test in one session; each test builds its own inputs, so it passes alone too.
"""
import ctypes as C

import numpy as np
import pytest

import welvet_b200 as W
from conftest import rel_err

STATIC_FLOATS = 1 << 20  # WELVET_B200_DECODE_STATIC_FLOATS
TOL = 2e-2               # BF16 tolerance of the attention parity tests


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


def _setup(torch, B, T, H, NK, hd, pos, seed):
    cfg = W.MhaConfig.make(H * hd, H, NK, head_dim=hd, precision=1, pos=pos, mask=1, max_seq_len=T)
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B * T, H * hd, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B * T, NK * hd, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B * T, NK * hd, device="cuda", generator=g).to(torch.bfloat16)
    pps = (T + 15) // 16
    bt = torch.randperm(B * pps, device="cuda", generator=g).view(B, pps).to(torch.int32).contiguous()
    return cfg, q, k, v, bt, _paged(torch, k, B, T, NK, hd, bt), _paged(torch, v, B, T, NK, hd, bt)


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,H,NK,hd,pos,lens", [
    (3, 300, 8, 2, 128, 1, None),          # GQA 4, no positional bias
    (4, 517, 16, 16, 64, 2, [517, 480, 33, 1]),  # MHA, ALiBi, ragged lengths incl. a single key
    (2, 1024, 32, 4, 128, 1, [1024, 700]),  # GQA 8
])
def test_matches_prefill_attention(torch_cuda, B, T, H, NK, hd, pos, lens):
    torch = torch_cuda
    cfg, q, k, v, bt, kp, vp = _setup(torch, B, T, H, NK, hd, pos, seed=7)
    ref = torch.zeros_like(q)
    W.attention(cfg, B, T, q, k, v, ref)  # existing entry point, causal prefill
    lens = lens or [T] * B
    rows = torch.tensor([b * T + L - 1 for b, L in enumerate(lens)], device="cuda")
    q_dec = q[rows].contiguous()
    want = ref[rows].float().cpu().numpy()
    ctx = torch.tensor(lens, device="cuda", dtype=torch.int32)
    for call in range(2):
        out = torch.full((B, H * hd), float("nan"), device="cuda", dtype=torch.bfloat16)
        st = _call(cfg, B, T, q_dec.data_ptr(), H * hd, kp.data_ptr(), vp.data_ptr(), bt.data_ptr(), bt.shape[1],
                   ctx.data_ptr(), out.data_ptr(), H * hd)
        assert st.code == 0, st.message
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_err(got, want) < TOL, f"call {call}"
    W.device_check()


@pytest.mark.gpu
def test_fewer_splits_when_default_does_not_fit(torch_cuda):
    """B=2, 64 heads of 256 over 8 KV heads at 9600 keys: the default 37 splits need
    2*64*258*37 floats > 2^20, so the call runs with 31 splits; checked against a
    float32 PyTorch softmax(q k^T) v of the same bf16 inputs."""
    torch = torch_cuda
    B, T, H, NK, hd = 2, 9600, 64, 8, 256
    assert B * H * (hd + 2) * 37 > STATIC_FLOATS
    cfg, q, k, v, bt, kp, vp = _setup(torch, B, T, H, NK, hd, pos=1, seed=11)
    lens = [T, 5000]
    rows = torch.tensor([b * T + L - 1 for b, L in enumerate(lens)], device="cuda")
    q_dec = q[rows].contiguous()
    ctx = torch.tensor(lens, device="cuda", dtype=torch.int32)
    want = []
    for b, L in enumerate(lens):
        qb = q_dec[b].float().view(H, hd)
        kb = k[b * T:b * T + L].float().view(L, NK, hd).repeat_interleave(H // NK, dim=1)
        vb = v[b * T:b * T + L].float().view(L, NK, hd).repeat_interleave(H // NK, dim=1)
        s = torch.einsum("hd,lhd->hl", qb, kb) / hd ** 0.5
        want.append(torch.einsum("hl,lhd->hd", torch.softmax(s, dim=1), vb).reshape(-1).cpu().numpy())
    want = np.stack(want)
    for call in range(2):
        out = torch.full((B, H * hd), float("nan"), device="cuda", dtype=torch.bfloat16)
        st = _call(cfg, B, T, q_dec.data_ptr(), H * hd, kp.data_ptr(), vp.data_ptr(), bt.data_ptr(), bt.shape[1],
                   ctx.data_ptr(), out.data_ptr(), H * hd)
        assert st.code == 0, st.message
        torch.cuda.synchronize()
        assert rel_err(out.float().cpu().numpy(), want) < TOL, f"call {call}"
    W.device_check()
