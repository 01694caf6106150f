"""Host-side multi-GPU logic on CPU: zig-zag row plan and the gloo reassembly
of row / batch shards (world_size 2 processes, 127.0.0.1 rendezvous)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gsa_gdn_benchmarkstudy_b200.sharding import (causal_row_cost, gather_batch, gather_rows,
                                                  zigzag_blocks)


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
