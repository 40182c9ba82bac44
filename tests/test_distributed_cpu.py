"""Multi-rank host logic on CPU ranks (gloo, world size 2): batch sharding
and the head / token importance all-reduces give every rank the decision a
single process takes on the whole batch (spatten_bert.py:120-130, 136-150)."""
import os
import socket

import numpy as np
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, ctx, q):
    import torch.distributed as dist
    from spatten_b200 import distributed as sd
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        local = sd.shard_batch(ctx, rank, world)          # [B_local, H, S, D]
        B, H, S, D = local.shape
        head = sd.allreduce_head_importance(local.abs().sum(dim=(0, 2, 3)), B * S * D)
        # heads split (whole batch on every rank): partial sums over my heads
        tok_part = ctx[:, rank::world].abs().sum(dim=(1, 3))
        tok = sd.allreduce_token_importance(tok_part.clone())
        q.put((rank, head.numpy(), tok.numpy(), (B, sd.shard_range(ctx.shape[0], rank, world))))
    finally:
        dist.destroy_process_group()


def test_shard_range_covers_everything():
    from spatten_b200.distributed import shard_range
    for n in (1, 5, 8, 33):
        for w in (1, 2, 3, 8):
            spans = [shard_range(n, r, w) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1


def test_gloo_two_ranks_importance_allreduce():
    g = torch.Generator().manual_seed(0)
    ctx = torch.randn(5, 4, 7, 8, generator=g)
    world = 2
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _free_port()
    procs = [mpc.Process(target=_worker, args=(r, world, port, ctx, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # single-process decisions on the whole batch
    head_ref = ctx.abs().mean(dim=(0, 2, 3)).numpy()
    for rank, head, tok, _ in out:
        np.testing.assert_allclose(head, head_ref, rtol=1e-6)
        # same kept heads on every rank
        assert np.array_equal(np.sort(np.argsort(-head)[:3]), np.sort(np.argsort(-head_ref)[:3]))
    sizes = sorted(o[3][0] for o in out)
    assert sizes == [2, 3]
    # token importance: partial sums over each rank's heads add up to all heads
    expect = ctx.abs().sum(dim=(1, 3)).numpy()
    for _, _, tok, _ in out:
        np.testing.assert_allclose(tok, expect, rtol=1e-5)


def test_head_batch_shards_partition():
    """Every (batch, head) unit of the B8 H12 op workload lands on exactly one
    rank; heads split over up to 4 ranks, the batch over the rest."""
    from spatten_b200.distributed import HeadBatchShards
    for world, (hr, br) in {1: (1, 1), 2: (2, 1), 4: (4, 1), 8: (4, 2)}.items():
        seen = np.zeros((8, 12), int)
        for r in range(world):
            p = HeadBatchShards(8, 12, r, world)
            assert (p.head_ranks, p.batch_ranks) == (hr, br)
            seen[p.b0:p.b1, p.h0:p.h1] += 1
        assert (seen == 1).all(), world


def _head_group_worker(rank, world, port, x, q):
    import torch.distributed as dist
    from spatten_b200.distributed import HeadBatchShards, allreduce_token_importance
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = HeadBatchShards(x.shape[0], x.shape[1], rank, world, max_head_ranks=2)
        part = plan.take(x).sum(dim=1).contiguous()  # [B_local, S]: my heads' partial sums
        tok = allreduce_token_importance(part, plan.groups())
        q.put((rank, plan.b0, plan.b1, tok.numpy()))
    finally:
        dist.destroy_process_group()


def test_gloo_four_ranks_head_group_allreduce():
    """Four ranks as 2 head ranks x 2 batch ranks: each head group's
    all-reduce gives the sum over all heads for its own batch rows only."""
    g = torch.Generator().manual_seed(1)
    x = torch.rand(4, 6, 9, generator=g)
    world = 4
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _free_port()
    procs = [mpc.Process(target=_head_group_worker, args=(r, world, port, x, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    full = x.sum(dim=1).numpy()
    for rank, b0, b1, tok in out:
        np.testing.assert_allclose(tok, full[b0:b1], rtol=1e-6)


def _cpu_topk(x, k):
    """Ascending indices of the k largest, ties to the smaller index (the
    order spatten_topk_indices gives)."""
    idx = torch.argsort(-x, dim=1, stable=True)[:, :k]
    return torch.sort(idx, dim=1).values


def _batch_split_worker(rank, world, port, parts, k, q):
    import torch.distributed as dist
    from spatten_b200 import distributed as sd
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        kept, mine = sd.topk_by_batch_shard(parts[rank].clone(), k, topk=_cpu_topk)
        q.put((rank, kept.numpy(), mine.numpy()))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_decode_topk_by_batch_shard():
    """The decode selection split over the batch (reduce-scatter of the
    per-rank importance, top-k of each rank's rows, all-gather of the kept
    indices) gives every rank the kept keys of the summed importance of all
    batch rows, as one process selecting on the full sum."""
    g = torch.Generator().manual_seed(3)
    world, B, n, k = 2, 6, 40, 9
    parts = [torch.round(torch.rand(B, n, generator=g) * 8) / 8 for _ in range(world)]  # with ties
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _free_port()
    procs = [mpc.Process(target=_batch_split_worker, args=(r, world, port, parts, k, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    total = parts[0] + parts[1]
    ref = _cpu_topk(total, k).numpy()
    for rank, kept, mine in out:
        assert np.array_equal(kept, ref), rank
        np.testing.assert_allclose(mine, total[rank * B // world:(rank + 1) * B // world].numpy(), rtol=0)
