"""Seeded synthetic workloads: the configurations the GSA forward is measured on.

The reference measures on ``torch.randn`` inputs (gsa_triton/benchmark.py:127,177)
with the module's own random init; the configurations below fix every seed so
that the reference, the CPU oracle and the CUDA path see identical numbers:

* weights: every ``*.weight`` ~ N(0, 0.02) drawn in ``state_dict`` key order
  from ``torch.Generator().manual_seed(seed)`` (seed 1); the value/output
  gate biases are 0.5; the indexer's weight-projection bias and its
  threshold bias (``idx_bias``) are 0; buffers (``rotary_emb.inv_freq``) keep
  their deterministic construction value;
* inputs: x ~ N(0, 1) from seed 0, or one seed per sequence (0..B-1) for the
  batched-serving config, plus a 0.5-amplitude sinusoid of 4 periods along T
  for the long-context config.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


@dataclass(frozen=True)
class GSAConfig:
    name: str
    B: int
    T: int
    D: int
    H: int
    k_base: int
    k_min: int
    k_max: int
    d_indexer: int = 64
    n_idx_heads: int = 4
    dtype: str = "bf16"
    per_seq_seed: bool = False
    sinusoid: float = 0.0      # amplitude of the low-frequency component along T
    sinusoid_periods: int = 4
    note: str = ""

    @property
    def d_head(self) -> int:
        return self.D // self.H

    @property
    def k_eff(self) -> int:
        return min(self.k_base, self.k_max, self.T)

    @property
    def torch_dtype(self) -> torch.dtype:
        return torch.bfloat16 if self.dtype == "bf16" else torch.float32

    def module_kwargs(self) -> dict:
        return dict(hidden_size=self.D, num_heads=self.H, k_max=self.k_max,
                    d_indexer=self.d_indexer, n_idx_heads=self.n_idx_heads,
                    k_base=self.k_base, k_min=self.k_min)


# The five configurations of the benchmark study (cfg1 runs on CPU in fp32).
CONFIGS: dict[str, GSAConfig] = {
    "cfg1": GSAConfig("cfg1", 1, 1024, 512, 4, 256, 64, 512, dtype="fp32",
                      note="fp32, CPU-runnable reference case"),
    "cfg2": GSAConfig("cfg2", 1, 4096, 2048, 16, 2048, 256, 4096),
    "cfg3": GSAConfig("cfg3", 1, 16384, 2048, 16, 2048, 256, 4096,
                      note="indexer-dominated; headline metric config"),
    "cfg4": GSAConfig("cfg4", 8, 8192, 2048, 16, 2048, 256, 4096, per_seq_seed=True,
                      note="batched serving"),
    "cfg5": GSAConfig("cfg5", 1, 65536, 2048, 16, 2048, 256, 4096, sinusoid=0.5,
                      note="long context"),
}

# Small configurations for parity tests (k_eff < T so selection is real).
TEST_CONFIGS: dict[str, GSAConfig] = {
    "tiny_bf16": GSAConfig("tiny_bf16", 2, 160, 256, 2, 48, 16, 4096),
    "tiny_fp32": GSAConfig("tiny_fp32", 2, 160, 256, 2, 48, 16, 4096, dtype="fp32"),
    "small_bf16": GSAConfig("small_bf16", 1, 1024, 1024, 8, 256, 64, 4096),
}


def init_weights_(module: torch.nn.Module, seed: int = 1) -> torch.nn.Module:
    """Overwrite the module's parameters with the seeded benchmark init (in place)."""
    g = torch.Generator().manual_seed(seed)
    sd = module.state_dict()
    new = {}
    for name, t in sd.items():
        if name.endswith(".weight"):
            v = torch.randn(tuple(t.shape), generator=g, dtype=torch.float32) * 0.02
        elif name in ("value_gate.gate_proj.bias", "output_gate.gate_proj.bias"):
            v = torch.full(tuple(t.shape), 0.5)
        elif name in ("indexer.idx_w_proj.bias", "indexer.idx_bias"):
            v = torch.zeros(tuple(t.shape))
        else:
            continue
        new[name] = v.to(dtype=t.dtype, device=t.device)
    module.load_state_dict(new, strict=False)
    return module


def make_input(cfg: GSAConfig, device: str | torch.device = "cpu",
               dtype: torch.dtype | None = None, seed: int = 0) -> torch.Tensor:
    """Seeded input x [B, T, D] for a configuration (generated on the CPU, then moved)."""
    dtype = dtype or cfg.torch_dtype
    if cfg.per_seq_seed:
        x = torch.stack([
            torch.randn(cfg.T, cfg.D, generator=torch.Generator().manual_seed(seed + b))
            for b in range(cfg.B)
        ])
    else:
        x = torch.randn(cfg.B, cfg.T, cfg.D, generator=torch.Generator().manual_seed(seed))
    if cfg.sinusoid:
        t = torch.arange(cfg.T, dtype=torch.float32)
        wave = cfg.sinusoid * torch.sin(2.0 * math.pi * cfg.sinusoid_periods * t / cfg.T)
        x = x + wave.view(1, cfg.T, 1)
    return x.to(device=device, dtype=dtype)


def causal_pairs(T: int, k: int) -> int:
    """Number of (query, selected key) pairs of one sequence: k(k+1)/2 + (T-k)k."""
    k = min(k, T)
    return k * (k + 1) // 2 + (T - k) * k


@dataclass
class WorkModel:
    """Algorithmic work of one forward (the units behind the roofline figures)."""
    cfg: GSAConfig
    extra: dict = field(default_factory=dict)

    @property
    def indexer_flops(self) -> int:
        c = self.cfg
        return c.B * 2 * c.n_idx_heads * c.d_indexer * c.T * (c.T + 1) // 2

    @property
    def attn_dense_flops(self) -> int:
        """QK^T + PV flops over the causal key range (what the bitmask kernel computes)."""
        c = self.cfg
        return c.B * 4 * c.D * c.T * (c.T + 1) // 2

    @property
    def attn_sparse_flops(self) -> int:
        """QK^T + PV flops over the selected pairs only."""
        c = self.cfg
        return c.B * 4 * c.D * causal_pairs(c.T, c.k_eff)

    @property
    def attn_gather_bytes(self) -> int:
        """K+V rows of every selected pair + Q in + O out + int32 indices."""
        c = self.cfg
        return (c.B * causal_pairs(c.T, c.k_eff) * 2 * c.D * 2 + c.B * c.T * c.D * 2 * 2
                + c.B * c.T * c.k_eff * 4)

    @property
    def proj_flops(self) -> int:
        c = self.cfg
        n = 5 * c.D + c.n_idx_heads * c.d_indexer + c.d_indexer + c.n_idx_heads
        return 2 * c.B * c.T * c.D * n + 2 * c.B * c.T * c.D * c.D
