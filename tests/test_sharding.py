"""Host-side multi-GPU logic on CPU: zig-zag row plan and the gloo reassembly
of row / batch shards (world_size 2 processes, 127.0.0.1 rendezvous)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gsa_gdn_benchmarkstudy_b200.sharding import (RowBlockGather, causal_row_cost, gather_batch,
                                                  gather_rows, unshard_rows, zigzag_blocks,
                                                  zigzag_order)


@pytest.mark.parametrize("T,world", [(16384, 1), (16384, 2), (16384, 8), (65536, 8), (64, 4)])
def test_zigzag_covers_every_row_once_and_balances(T, world):
    rows = []
    costs = []
    for r in range(world):
        blocks = zigzag_blocks(T, world, r)
        assert len(blocks) == 2
        for s, e in blocks:
            rows += list(range(s, e))
        costs.append(causal_row_cost(blocks, 2048))
    assert sorted(rows) == list(range(T))
    # Indexer and bitmask-attention work both grow with t+1 (every causal key
    # tile is visited), so zig-zag pairs balance them to within one row.
    idx = [c[0] for c in costs]
    assert max(idx) - min(idx) <= T
    # A gather formulation (work min(t+1, k)) would be balanced far less well.
    att = [c[1] for c in costs]
    assert max(att) / min(att) < 2.0


def test_zigzag_rejects_ragged_lengths():
    with pytest.raises(ValueError):
        zigzag_blocks(1000, 3, 0)


@pytest.mark.parametrize("T,world", [(64, 1), (64, 2), (4096, 8), (96, 3)])
def test_zigzag_order_unshards_a_rank_major_gather(T, world):
    """zigzag_order maps every sequence row to its row in the rank-major
    concatenation of the ranks' local shards; unshard_rows applies it."""
    full = torch.arange(T * 2, dtype=torch.float32).view(1, T, 2)
    shards = torch.stack([torch.cat([full[0, s:e] for s, e in zigzag_blocks(T, world, r)])
                          for r in range(world)])            # [world, T/world, 2]
    order = zigzag_order(T, world, torch.device("cpu"))
    assert sorted(order.tolist()) == list(range(T))
    assert torch.equal(unshard_rows(shards, order), full)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, T, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = torch.arange(T * 3, dtype=torch.float32).view(1, T, 3)
        local = torch.cat([full[:, s:e] for s, e in zigzag_blocks(T, world, rank)], dim=1)
        got = gather_rows(local, T, dist.group.WORLD)
        ok_rows = torch.equal(got, full)
        # the per-block form the sharded forward uses: block 0 gathered first
        gat = RowBlockGather(T, world, 3, torch.float32, torch.device("cpu"))
        for i, (s, e) in enumerate(zigzag_blocks(T, world, rank)):
            gat.add(i, full[0, s:e], dist.group.WORLD)
        ok_rows = ok_rows and torch.equal(gat.finish(), full)
        xb = torch.arange(4 * 5 * 2, dtype=torch.float32).view(4, 5, 2)
        per = 4 // world
        gb = gather_batch(xb[rank * per:(rank + 1) * per], dist.group.WORLD)
        q.put((rank, ok_rows, torch.equal(gb, xb)))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_reassembles_row_and_batch_shards():
    world, T = 2, 40
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok_r and ok_b for _, ok_r, ok_b in res), res


def _adaptive_worker(rank, world, port, T, q):
    """Each rank holds its zig-zag rows' variances; ShardedGSA's all-reduce of
    their sums must give every rank the batch-wide mean that adaptive k uses."""
    from gsa_gdn_benchmarkstudy_b200.sharding import ShardedGSA
    from oracle import gsa_oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(11)
        s = torch.randn(1, T, T, generator=g) * torch.linspace(0.5, 2.0, T).view(1, T, 1)
        s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), float("-inf"))
        var = O.score_variance(s)
        runner = ShardedGSA(None, dist.group.WORLD, T=T, B=1)
        mine = torch.cat([var[:, a:b] for a, b in runner.blocks], dim=1)
        total = mine.double().sum().reshape(1)
        runner._sum_over_ranks(total)
        mean_ok = abs(total.item() / T - var.double().mean().item()) <= 1e-6 * var.mean().item()
        ks = O.adaptive_k_from_variance(mine, 32, 4, 64, avg_var=(total / T).float().clamp(min=1e-6))
        ref = O.adaptive_k_from_variance(var, 32, 4, 64)
        ref_mine = torch.cat([ref[:, a:b] for a, b in runner.blocks], dim=1)
        q.put((rank, mean_ok, int((ks != ref_mine).sum())))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_adaptive_k_variance_reduce():
    world, T = 2, 64
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_adaptive_worker, args=(r, world, port, T, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in res), res
    # k from the reduced mean matches the single-process rule (fp32 vs fp64
    # means may move a row across a floor boundary; none does for this input)
    assert all(bad == 0 for _, _, bad in res), res
