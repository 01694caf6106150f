"""B200-native Gated Sparse Attention forward (sm_100a CUDA behind a C ABI).

Public API mirrors gsa_triton/gsa_ref.py and gsa_triton/gsa_opt.py of
nirmalpratheep/GSA_GDN_BenchmarkStudy:

    from gsa_gdn_benchmarkstudy_b200 import GatedSparseAttention
    model = GatedSparseAttention(hidden_size=2048, num_heads=16).cuda().bfloat16().eval()
    model.fuse_projections()
    y = model(x)            # x: [B, T, 2048] bf16 on an sm_100 GPU

The compute runs in ``libgsa_b200.so`` (built by ``python -m
gsa_gdn_benchmarkstudy_b200.build``); there is no CPU fallback.
"""
from .gsa import (  # noqa: F401
    AdaptiveTopKSelector,
    GatedLightningIndexer,
    GatedSparseAttention,
    GraphedForward,
    GraphedForwardHost,
    OutputGate,
    RotaryEmbedding,
    ValueGate,
    apply_rotary_pos_emb,
)
from .ops import fused_gated_indexer, fused_sparse_attention, sparse_attention_ref  # noqa: F401

__all__ = [
    "GatedSparseAttention", "GraphedForward", "GraphedForwardHost", "GatedLightningIndexer",
    "AdaptiveTopKSelector", "ValueGate", "OutputGate", "RotaryEmbedding", "apply_rotary_pos_emb", "fused_gated_indexer",
    "fused_sparse_attention", "sparse_attention_ref",
]
