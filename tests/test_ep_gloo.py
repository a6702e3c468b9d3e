"""Host side of expert parallelism on CPU with two gloo ranks: pair counts,
pair rows and slot rows reach the rank that owns their experts in
contiguous per-source blocks, and the returned partial rows come back in
send order (the NCCL path on GPUs runs the same exchange code)."""
import os
import tempfile

import torch
import torch.multiprocessing as mp


def _worker(rank, world, init_file, result_dir):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    from mlxr_moe.ep import TorchDistExchange

    ex = TorchDistExchange()
    D, K = 8, 4
    # rank r sends (r + 1) * (d + 1) pairs to rank d; pair i is tagged
    # 64 * src + 16 * dst + i (exact in bf16), its slots with 1000 * src + 10 * dst + i
    pairs = [(rank + 1) * (d + 1) for d in range(world)]
    counts = torch.tensor([[p, 3 * p] for p in pairs], dtype=torch.int32)
    rows, metas = [], []
    for d in range(world):
        for i in range(pairs[d]):
            rows.append(torch.full((D,), float(64 * rank + 16 * d + i)))
            metas.append(torch.full((K,), 1000 * rank + 10 * d + i, dtype=torch.int32))
    x_send = torch.stack(rows).to(torch.bfloat16)
    meta_send = torch.stack(metas)
    recv_counts = ex.counts(counts)
    assert recv_counts.tolist() == [[(s + 1) * (rank + 1), 3 * (s + 1) * (rank + 1)] for s in range(world)]
    rp = recv_counts[:, 0].tolist()
    x_recv = ex.rows(x_send, pairs, rp)
    meta_recv = ex.rows(meta_send, pairs, rp)
    k = 0
    for s in range(world):
        for i in range(rp[s]):
            assert x_recv[k, 0].item() == float(64 * s + 16 * rank + i), (rank, s, i)
            assert int(meta_recv[k, K - 1]) == 1000 * s + 10 * rank + i
            k += 1
    # a receiver-side transform, then the reverse exchange restores send order
    back = ex.rows(x_recv.float().mul(2).to(torch.bfloat16), rp, pairs)
    assert torch.equal(back, x_send.float().mul(2).to(torch.bfloat16))
    with open(os.path.join(result_dir, f"ok{rank}"), "w") as f:
        f.write("ok")
    dist.destroy_process_group()


def test_ep_exchange_two_gloo_ranks():
    d = tempfile.mkdtemp()
    init_file = os.path.join(d, "init")
    mp.spawn(_worker, args=(2, init_file, d), nprocs=2, join=True)
    assert os.path.exists(os.path.join(d, "ok0")) and os.path.exists(os.path.join(d, "ok1"))
