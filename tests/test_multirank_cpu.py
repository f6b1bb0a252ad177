"""The multi-GPU decomposition on CPU: world_size-2 gloo process groups.

On N GPUs each rank mounts the heads welvet_b200.head_shard gives it (Wq/Wk/Wv rows
and Wo columns of those heads), runs attention and its KV cache locally, and the
per-rank outputs of the O projection are summed by one all-reduce (NCCL on the
GPUs). Here each rank computes its shard with the CPU oracle on the same slices,
the sum is a gloo all_reduce, and rank 0 compares it with the unsharded oracle:
prefill (RoPE, causal) and one decode step over a KV cache, MHA and GQA. The
attention-output exchange (output mode 2) is restated the same way: the ranks'
attention rows go to the owners' receive slots, whose output projection over every
head must equal the unsharded layer's rows exactly. Rendezvous on 127.0.0.1.
"""
import datetime
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_weights(Ws, hb, hc, group, hd):
    Wq, Wk, Wv, Wo = Ws
    kb, kc = hb // group, hc // group
    return (Wq[hb * hd:(hb + hc) * hd], Wk[kb * hd:(kb + kc) * hd], Wv[kb * hd:(kb + kc) * hd],
            np.ascontiguousarray(Wo[:, hb * hd:(hb + hc) * hd]))


def _case(H, NK):
    import welvet_b200 as W
    d, hd, B, T = 64, 16, 2, 12
    Ws = W.xavier_weights(d, H * hd, NK * hd, seed=0)
    x = W.synthetic(B * T * d, 1, 1, 1.0).reshape(B * T, d)
    x_new = W.synthetic(B * d, 3, 1, 1.0).reshape(B, d)
    return d, hd, B, T, Ws, x, x_new


def _worker(rank, world, port, out_path, H, NK):
    import torch
    import torch.distributed as dist
    sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "welvet.metal_b200")]
    import oracle_py as O
    import welvet_b200 as W
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        d, hd, B, T, Ws, x, x_new = _case(H, NK)
        group = H // NK
        hb, hc = W.head_shard(H, NK, world, rank)
        sub = O.MhaCfg(d_model=d, num_heads=hc, num_kv_heads=hc // group, head_dim=hd, max_seq_len=64,
                       mask=1, pos=0, per_sequence=1)
        Wq, Wk, Wv, Wo = _shard_weights(Ws, hb, hc, group, hd)
        pre, post, _, k, v = O.mha_forward(sub, B, T, Wq, Wk, Wv, Wo, x, want_qkv=True)
        # decode one token per sequence over this rank's slice of the prefill KV cache
        kc = k.reshape(B, T, -1)
        vc = v.reshape(B, T, -1)
        dpre, dpost, _, _ = O.mha_decode(sub, np.full(B, T, np.int32), kc, vc, Wq, Wk, Wv, Wo, x_new)
        post_t, dpost_t = torch.from_numpy(post), torch.from_numpy(dpost)
        dist.all_reduce(post_t)
        dist.all_reduce(dpost_t)
        pres = [torch.zeros_like(torch.from_numpy(pre)) for _ in range(world)]
        dist.all_gather(pres, torch.from_numpy(pre))
        if rank == 0:
            np.savez(out_path, post=post_t.numpy(), dpost=dpost_t.numpy(),
                     pre=np.concatenate([p.numpy() for p in pres], axis=1))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("H,NK", [(4, 4), (4, 2), (8, 2)])
def test_head_shards_allreduce_to_full_layer(tmp_path, H, NK):
    import torch.multiprocessing as mp
    sys.path.insert(0, os.path.join(ROOT, "welvet.metal_b200"))
    import oracle_py as O
    out = str(tmp_path / "rank0.npz")
    mp.start_processes(_worker, args=(2, _free_port(), out, H, NK), nprocs=2, join=True, start_method="spawn")
    got = np.load(out)
    d, hd, B, T, Ws, x, x_new = _case(H, NK)
    cfg = O.MhaCfg(d_model=d, num_heads=H, num_kv_heads=NK, head_dim=hd, max_seq_len=64, mask=1, pos=0,
                   per_sequence=1)
    pre, post, _, k, v = O.mha_forward(cfg, B, T, *Ws, x, want_qkv=True)
    _, dpost, _, _ = O.mha_decode(cfg, np.full(B, T, np.int32), k.reshape(B, T, -1), v.reshape(B, T, -1), *Ws,
                                  x_new)
    rel = lambda a, b: float(np.abs(a - b).max() / np.abs(b).max())
    assert rel(got["pre"], pre) == 0.0      # heads are independent: the shards' pre is exact
    assert rel(got["post"], post) < 1e-5    # summation order differs from the full O projection
    assert rel(got["dpost"], dpost) < 1e-5


def _exchange_worker(rank, world, port, out_path, H, NK):
    """Output mode 2 on CPU: each rank's attention output (its heads' columns) is
    split by rows into the owners' receive slots, chunk by chunk, and each rank runs
    the output projection over every head for its own rows."""
    import torch
    import torch.distributed as dist
    sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "welvet.metal_b200")]
    import oracle_py as O
    import welvet_b200 as W
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        d, hd, B, T, Ws, x, _ = _case(H, NK)
        group = H // NK
        hb, hc = W.head_shard(H, NK, world, rank)
        sub = O.MhaCfg(d_model=d, num_heads=hc, num_kv_heads=hc // group, head_dim=hd, max_seq_len=64,
                       mask=1, pos=0, per_sequence=1)
        Wq, Wk, Wv, Wo = _shard_weights(Ws, hb, hc, group, hd)
        pre, _ = O.mha_forward(sub, B, T, Wq, Wk, Wv, Wo, x)
        qdl = hc * hd
        # every rank's attention rows and Wo columns (the copy engines' and the set-up
        # gather's part on the GPUs)
        pres = [torch.zeros_like(torch.from_numpy(pre)) for _ in range(world)]
        dist.all_gather(pres, torch.from_numpy(pre))
        wos = [torch.zeros_like(torch.from_numpy(Wo)) for _ in range(world)]
        dist.all_gather(wos, torch.from_numpy(Wo))
        wo_full = np.concatenate([w.numpy() for w in wos], axis=1)     # [d, q_dim], rank p's block at p*qdl
        rows = []
        for c0 in range(0, B * T, T):                                  # chunks of one sequence
            own = T // world
            recv = np.zeros((own, world * qdl), np.float32)            # this rank's receive slot
            for p in range(world):
                recv[:, p * qdl:(p + 1) * qdl] = pres[p].numpy()[c0 + rank * own:c0 + (rank + 1) * own]
            rows.append(O.dense(recv, wo_full))
        got = [torch.zeros(B * T // world, d) for _ in range(world)]
        dist.all_gather(got, torch.from_numpy(np.concatenate(rows)))
        if rank == 0:
            np.save(out_path, np.stack([g.numpy() for g in got]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("H,NK", [(4, 4), (8, 2)])
def test_attention_output_exchange_matches_full_layer(tmp_path, H, NK):
    """Rank r's rows [c0 + r*T/2, c0 + (r+1)*T/2) of each one-sequence chunk equal the
    unsharded layer's, bit for bit (one accumulation over every head)."""
    import torch.multiprocessing as mp
    sys.path.insert(0, os.path.join(ROOT, "welvet.metal_b200"))
    import oracle_py as O
    out = str(tmp_path / "xa.npy")
    mp.start_processes(_exchange_worker, args=(2, _free_port(), out, H, NK), nprocs=2, join=True,
                       start_method="spawn")
    got = np.load(out)
    d, hd, B, T, Ws, x, _ = _case(H, NK)
    cfg = O.MhaCfg(d_model=d, num_heads=H, num_kv_heads=NK, head_dim=hd, max_seq_len=64, mask=1, pos=0,
                   per_sequence=1)
    _, post = O.mha_forward(cfg, B, T, *Ws, x)
    own = T // 2
    for r in range(2):
        want = np.concatenate([post[c0 + r * own:c0 + (r + 1) * own] for c0 in range(0, B * T, T)])
        assert np.array_equal(got[r], want)


def test_head_shard_rules():
    sys.path.insert(0, os.path.join(ROOT, "welvet.metal_b200"))
    import welvet_b200 as W
    assert [W.head_shard(32, 32, 8, r) for r in (0, 7)] == [(0, 4), (28, 4)]
    assert W.head_shard(32, 8, 8, 3) == (12, 4)    # GQA 4: one KV head per rank
    with pytest.raises(ValueError):
        W.head_shard(32, 4, 8, 0)                  # 4 heads per rank split a KV group of 8
    with pytest.raises(ValueError):
        W.head_shard(12, 12, 8, 0)
    with pytest.raises(ValueError):
        W.head_shard(32, 32, 2, 2)
