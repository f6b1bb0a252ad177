"""Two ranks on two GPUs (skipped with fewer): head-sharded layers with an NCCL
communicator, the row-sharded host-buffer forward (welvet_b200_mha_forward_rows)
against the FP64 oracle's forward of the whole batch (per-sequence semantics, the
same FP32 or BF16-rounded weights and inputs). Each rank passes only its half of
the sequences and receives the summed output rows of that half. Then two decode
steps over each rank's KV heads, their outputs summed through the NVLink
peer-memory all-reduce, against the oracle's decode of the whole layer. The
device-buffer forward runs with the reduce-scatter output (mode 1) and with the
attention-output exchange (mode 2); each rank's own rows against the oracle."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir, precision):
    import datetime

    import torch
    import torch.distributed as dist

    import welvet_b200 as W
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    d, H, NK, B, T = 512, 8, 4, 8, 128
    dt = torch.float32 if precision == 0 else torch.bfloat16
    Ws = W.xavier_weights(d, d, NK * d // H, seed=0)
    x = torch.from_numpy(W.synthetic(B * T * d, 1, 1, 1.0).reshape(B * T, d)).to(dt)
    hb, hc = W.head_shard(H, NK, world, rank)
    layer = W.MhaLayer(W.MhaConfig.make(d, H, NK, precision=precision, head_begin=hb, head_count=hc), *Ws)
    uid = [W.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    layer.attach_comm(uid[0], world, rank)
    bl = B // world
    xl = x[rank * bl * T:(rank + 1) * bl * T].contiguous().pin_memory()
    post = torch.zeros(bl * T, d, dtype=dt).pin_memory()
    for _ in range(2):  # the second call reuses the staging buffers and events
        layer.forward_rows(bl, T, xl, post)
    np.save(os.path.join(out_dir, f"rows{rank}.npy"), post.float().numpy())
    # one sequence per rank: the forward runs as a single chunk
    x1 = x[rank * T:(rank + 1) * T].contiguous().pin_memory()
    p1 = torch.zeros(T, d, dtype=dt).pin_memory()
    layer.forward_rows(1, T, x1, p1)
    np.save(os.path.join(out_dir, f"one{rank}.npy"), p1.float().numpy())
    # device buffers, reduce-scatter output: the batch runs in 4 chunks of 2
    # sequences (256 rows); rank r keeps rows [c0 + 128 r, c0 + 128 (r + 1)) summed
    layer.set_output_mode(1)
    xd = x.cuda()
    pd = torch.zeros(B * T, d, device="cuda", dtype=dt)
    layer.forward(B, T, xd, None, pd)
    torch.cuda.synchronize()
    layer.check_device()
    own = np.concatenate([pd[c0 + rank * 128:c0 + (rank + 1) * 128].float().cpu().numpy()
                          for c0 in range(0, B * T, 256)])
    np.save(os.path.join(out_dir, f"rs{rank}.npy"), own)
    # device buffers, attention-output exchange (mode 2; FP32 layers run as mode 1):
    # the same rows, two calls so both call parities of the receive areas are used
    layer.set_output_mode(2)
    for call in range(2):
        pd = torch.full((B * T, d), float("nan"), device="cuda", dtype=dt)
        layer.forward(B, T, xd, None, pd)
        torch.cuda.synchronize()
        layer.check_device()
        own = np.concatenate([pd[c0 + rank * 128:c0 + (rank + 1) * 128].float().cpu().numpy()
                              for c0 in range(0, B * T, 256)])
        np.save(os.path.join(out_dir, f"xa{rank}_{call}.npy"), own)
    # the unsharded layer on this GPU (no communicator) over the same inputs: mode 2
    # sums every head in one accumulation, as this layer does
    full = W.MhaLayer(W.MhaConfig.make(d, H, NK, precision=precision), *Ws)
    pf = torch.zeros(B * T, d, device="cuda", dtype=dt)
    full.forward(B, T, xd, None, pf)
    torch.cuda.synchronize()
    own = np.concatenate([pf[c0 + rank * 128:c0 + (rank + 1) * 128].float().cpu().numpy()
                          for c0 in range(0, B * T, 256)])
    np.save(os.path.join(out_dir, f"full{rank}.npy"), own)
    full.close()
    if rank == 0:
        np.save(os.path.join(out_dir, "x.npy"), x.float().numpy())
    # decode: two steps over a paged KV cache holding this rank's KV heads; the
    # batch x d_model output is all-reduced over NVLink peer memory (one kernel),
    # the second step on the other parity of the peer workspace
    hd, L = d // H, 64
    kdf = NK * hd
    kc = torch.from_numpy(W.synthetic(B * L * kdf, 2, 1, 0.5).reshape(B, L, kdf)).to(dt)
    vc = torch.from_numpy(W.synthetic(B * L * kdf, 2, 1, 0.5, offset=B * L * kdf).reshape(B, L, kdf)).to(dt)
    kh0, khc = hb // (H // NK), hc // (H // NK)
    kv = W.KvCache(layer, B, L + 16)
    kv.fill(B, L, kc[:, :, kh0 * hd:(kh0 + khc) * hd].contiguous().cuda(),
            vc[:, :, kh0 * hd:(kh0 + khc) * hd].contiguous().cuda())
    for step in range(2):
        xs = torch.from_numpy(W.synthetic(B * d, 30 + step, 1, 1.0).reshape(B, d)).to(dt)
        pre_d = torch.zeros(B, hc * hd, device="cuda", dtype=dt)
        post_d = torch.zeros(B, d, device="cuda", dtype=dt)
        layer.decode(kv, B, xs.cuda(), pre_d, post_d)
        torch.cuda.synchronize()
        layer.check_device()
        np.save(os.path.join(out_dir, f"dec{rank}_{step}.npy"), post_d.float().cpu().numpy())
        if rank == 0:
            np.save(os.path.join(out_dir, f"decx{step}.npy"), xs.float().numpy())
    if rank == 0:
        np.save(os.path.join(out_dir, "kc.npy"), kc.float().numpy())
        np.save(os.path.join(out_dir, "vc.npy"), vc.float().numpy())
    layer.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("precision", [0, 1])
def test_forward_rows_two_ranks(tmp_path, precision):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path), precision), nprocs=2, join=True,
                       start_method="spawn")
    import oracle_py as O
    import welvet_b200 as W
    from conftest import bf16_round, rel_err
    d, H, NK, B, T = 512, 8, 4, 8, 128
    Ws = W.xavier_weights(d, d, NK * d // H, seed=0)
    if precision == 1:
        Ws = [bf16_round(w) for w in Ws]
    x = np.load(tmp_path / "x.npy")  # the inputs as the device held them
    oc = O.MhaCfg(d_model=d, num_heads=H, num_kv_heads=NK, per_sequence=1)
    _, want = O.mha_forward(oc, B, T, *Ws, x)
    got = np.concatenate([np.load(tmp_path / f"rows{r}.npy") for r in range(2)])
    tol = 1e-4 if precision == 0 else 2e-2
    assert rel_err(got, want) < tol, rel_err(got, want)
    for r in range(2):  # one sequence per rank: sequence r
        one = np.load(tmp_path / f"one{r}.npy")
        assert rel_err(one, want[r * T:(r + 1) * T]) < tol, (r, rel_err(one, want[r * T:(r + 1) * T]))
    for r in range(2):  # reduce-scatter output: each rank's row slices of each chunk
        rows = np.concatenate([np.arange(c0 + r * 128, c0 + (r + 1) * 128) for c0 in range(0, B * T, 256)])
        rs = np.load(tmp_path / f"rs{r}.npy")
        assert rel_err(rs, want[rows]) < tol, (r, rel_err(rs, want[rows]))
        full = np.load(tmp_path / f"full{r}.npy")
        for call in range(2):  # attention-output exchange: the same rows
            xa = np.load(tmp_path / f"xa{r}_{call}.npy")
            assert np.isfinite(xa).all()
            assert rel_err(xa, want[rows]) < tol, (r, call, rel_err(xa, want[rows]))
            print(f"precision {precision} rank {r} call {call}: exchange vs oracle {rel_err(xa, want[rows]):.3e}, "
                  f"max |exchange - unsharded layer| {np.abs(xa - full).max():.3e}")
    # decode steps: every rank holds the whole summed output
    kc, vc = np.load(tmp_path / "kc.npy"), np.load(tmp_path / "vc.npy")
    L = kc.shape[1]
    for step in range(2):
        xs = np.load(tmp_path / f"decx{step}.npy")
        _, want_d, kn, vn = O.mha_decode(oc, [L + step] * B, kc, vc, *Ws, xs)
        for r in range(2):
            got_d = np.load(tmp_path / f"dec{r}_{step}.npy")
            assert rel_err(got_d, want_d) < tol, (step, r, rel_err(got_d, want_d))
        if precision == 1:  # the cache holds the new rows in bf16
            kn, vn = bf16_round(kn), bf16_round(vn)
        kc = np.concatenate([kc, kn[:, None, :]], axis=1)
        vc = np.concatenate([vc, vn[:, None, :]], axis=1)
