"""Seeded workloads, work model figures and the module's host-side behaviour (CPU)."""
import pytest
import torch

from conftest import load_golden
from gsa_gdn_benchmarkstudy_b200 import GatedSparseAttention
from gsa_gdn_benchmarkstudy_b200.workloads import (CONFIGS, TEST_CONFIGS, WorkModel, causal_pairs,
                                                   init_weights_, make_input)


def test_causal_pair_counts():
    # P(T, k) = k(k+1)/2 + (T-k)k for the benchmark configurations
    assert causal_pairs(1024, 256) == 229_504
    assert causal_pairs(4096, 2048) == 6_292_480
    assert causal_pairs(16384, 2048) == 31_458_304
    assert causal_pairs(8192, 2048) == 14_681_088
    assert causal_pairs(65536, 2048) == 132_121_600


def test_work_model_cfg3():
    w = WorkModel(CONFIGS["cfg3"])
    assert w.indexer_flops == 2 * 4 * 64 * 16384 * 16385 // 2  # 68.7 GFLOP
    assert abs(w.attn_gather_bytes / 1e9 - 258.0) < 0.5


def test_inputs_are_seeded_and_shaped():
    c4 = CONFIGS["cfg4"]
    small = c4.__class__(**{**c4.__dict__, "T": 16, "D": 8})
    x = make_input(small)
    assert x.shape == (8, 16, 8) and x.dtype == torch.bfloat16
    # per-sequence seeds: sequence b equals a single-sequence draw with seed b
    one = torch.randn(16, 8, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    assert torch.equal(x[3], one)
    c5 = CONFIGS["cfg5"]
    small5 = c5.__class__(**{**c5.__dict__, "T": 64, "D": 4})
    x5 = make_input(small5, dtype=torch.float32)
    base = torch.randn(1, 64, 4, generator=torch.Generator().manual_seed(0))
    assert not torch.equal(x5, base)
    assert torch.allclose((x5 - base).mean(-1)[0, 4], torch.tensor(0.5), atol=1e-5)


def test_state_dict_contract_matches_reference():
    g = load_golden("tiny_bf16")
    cfg = TEST_CONFIGS["tiny_bf16"]
    m = GatedSparseAttention(**cfg.module_kwargs()).to(torch.bfloat16)
    ours = [(k, tuple(t.shape), str(t.dtype)) for k, t in m.state_dict().items()]
    assert ours == g["state_keys"]


def test_weight_init_is_deterministic():
    cfg = TEST_CONFIGS["tiny_fp32"]
    a = init_weights_(GatedSparseAttention(**cfg.module_kwargs()))
    b = init_weights_(GatedSparseAttention(**cfg.module_kwargs()))
    for (ka, ta), (kb, tb) in zip(a.state_dict().items(), b.state_dict().items()):
        assert ka == kb and torch.equal(ta, tb)
    sd = a.state_dict()
    assert torch.all(sd["value_gate.gate_proj.bias"] == 0.5)
    assert torch.all(sd["indexer.idx_bias"] == 0)


def test_forward_refuses_cpu_tensors():
    cfg = TEST_CONFIGS["tiny_fp32"]
    m = GatedSparseAttention(**cfg.module_kwargs())
    with pytest.raises(RuntimeError, match="CUDA"):
        m(make_input(cfg))


def test_graphed_forward_refuses_cpu_device():
    cfg = TEST_CONFIGS["tiny_fp32"]
    m = GatedSparseAttention(**cfg.module_kwargs())
    with pytest.raises(RuntimeError, match="CUDA"):
        m.graphed((cfg.B, cfg.T, cfg.D), device="cpu")
    with pytest.raises(RuntimeError, match="CUDA"):
        m.graphed_host((cfg.B, cfg.T, cfg.D), device="cpu")


def test_fused_projection_layout():
    cfg = TEST_CONFIGS["tiny_fp32"]
    m = init_weights_(GatedSparseAttention(**cfg.module_kwargs()))
    m.fuse_projections()
    w, b = m._fused_weight, m._fused_bias
    assert w.shape[0] % 64 == 0 and w.shape[0] >= 5 * cfg.D + 4 * 64 + 64 + 4
    o = m._proj_offsets
    assert torch.equal(w[o[5]:o[5] + 256], m.indexer.idx_q_proj.weight)
    assert torch.equal(b[o[3]:o[3] + cfg.D], m.value_gate.gate_proj.bias)
    assert torch.all(w[m._proj_total:] == 0) and torch.all(b[m._proj_total:] == 0)
    # every column block starts 16-byte aligned in bf16
    assert all(off % 8 == 0 for off in o[:7])
