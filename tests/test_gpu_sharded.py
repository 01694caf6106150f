"""Sharded forward on the GPU against the unsharded one.

A single-process NCCL group (world_size 1) still cuts the sequence into two
zig-zag blocks, so this exercises the row-block path (query rows at q_pos0 > 0
against keys [0, block end)), the per-block kernels and the NCCL all-gather
reassembly on one GPU.  Multi-GPU runs use the same code with more ranks."""
import os
import socket

import pytest
import torch
import torch.distributed as dist

from gsa_gdn_benchmarkstudy_b200 import GatedSparseAttention, _lib
from gsa_gdn_benchmarkstudy_b200.build import build
from gsa_gdn_benchmarkstudy_b200.sharding import ShardedGSA
from gsa_gdn_benchmarkstudy_b200.workloads import CONFIGS, TEST_CONFIGS, init_weights_, make_input

pytestmark = pytest.mark.gpu
torch.set_grad_enabled(False)


@pytest.fixture(scope="module")
def group():
    build()
    _lib.load()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", 0))
    yield dist.group.WORLD
    dist.destroy_process_group()


def _model(cfg, adaptive=False):
    m = GatedSparseAttention(**cfg.module_kwargs(), adaptive_k=adaptive)
    init_weights_(m, seed=1)
    m = m.to(cfg.torch_dtype).cuda().eval()
    m.fuse_projections()
    return m


@pytest.mark.parametrize("name", ["small_bf16", "cfg2"])
def test_row_sharded_matches_unsharded(group, name):
    cfg = TEST_CONFIGS.get(name) or CONFIGS[name]
    m = _model(cfg)
    x = make_input(cfg).cuda()
    ref = m(x)
    runner = ShardedGSA(m, group, T=cfg.T, B=cfg.B)
    assert runner.blocks == [(0, cfg.T // 2), (cfg.T // 2, cfg.T)]
    got = runner(runner.local_input(x))
    assert got.shape == ref.shape
    err = (got.float() - ref.float()).abs().max().item()
    rel = ((got.float() - ref.float()).norm() / ref.float().norm()).item()
    # the row-block GEMMs may round differently from the whole-sequence GEMM
    assert err < 2e-2 and rel < 1e-2, (err, rel)
    assert _lib.device_error() == 0


def test_batch_sharded_matches_unsharded(group):
    cfg = TEST_CONFIGS["tiny_bf16"]
    m = _model(cfg)
    x = make_input(cfg).cuda()
    ref = m(x)
    runner = ShardedGSA(m, group, T=cfg.T, B=cfg.B)
    got = runner(runner.local_input(x))
    assert torch.equal(got, ref)


@pytest.mark.parametrize("name", ["small_bf16", "tiny_bf16"])
def test_forward_host_returns_this_ranks_rows(group, name):
    """forward_host: pinned host share in, this rank's output rows out (in the
    order of local_input), equal to those rows of the device-resident result.
    With row shards it projects and outputs block by block, so its GEMMs may
    round differently from the whole-share ones (bf16 output bound); with batch
    shards it runs the same GEMMs (bit-equal)."""
    cfg = TEST_CONFIGS[name]
    m = _model(cfg)
    x = make_input(cfg)
    runner = ShardedGSA(m, group, T=cfg.T, B=cfg.B)
    full = runner(runner.local_input(x.cuda())).cpu()
    for _ in range(2):  # the second call reuses the pinned output and the streams
        got = runner.forward_host(runner.local_input(x).pin_memory())
        assert not got.is_cuda
        ref = runner.local_input(full)
        if runner.mode == "batch":
            assert torch.equal(got, ref)
        else:
            err = (got.float() - ref.float()).abs().max().item()
            rel = ((got.float() - ref.float()).norm() / ref.float().norm()).item()
            assert err < 2e-2 and rel < 1e-2, (err, rel)


@pytest.mark.parametrize("name", ["small_bf16", "tiny_bf16"])
def test_adaptive_k_sharded_matches_unsharded(group, name):
    """Adaptive k under sharding: the blocks' (row shards') or the local batch's
    row-variance sums are all-reduced before any row picks its k, so the
    sharded forward selects as the unsharded one does."""
    cfg = TEST_CONFIGS[name]
    m = _model(cfg, adaptive=True)
    x = make_input(cfg).cuda()
    ref = m(x)
    runner = ShardedGSA(m, group, T=cfg.T, B=cfg.B)
    got = runner(runner.local_input(x))
    if runner.mode == "batch":
        assert torch.equal(got, ref)  # same GEMMs, same selection
    err = (got.float() - ref.float()).abs().max().item()
    rel = ((got.float() - ref.float()).norm() / ref.float().norm()).item()
    assert err < 2e-2 and rel < 1e-2, (err, rel)
    assert _lib.device_error() == 0

