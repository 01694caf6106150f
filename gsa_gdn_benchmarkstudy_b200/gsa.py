"""GatedSparseAttention for B200: the reference module's interface over sm_100a kernels.

Drop-in for ``gsa_triton/gsa_ref.py::GatedSparseAttention`` (gsa_ref.py:243-325)
and ``gsa_triton/gsa_opt.py::GatedSparseAttention`` (gsa_opt.py:512-730):
same constructor arguments, sub-module names and ``state_dict`` keys,
``forward(x, attention_mask=None)`` (the mask is accepted and ignored, as in
the reference) and ``fuse_projections()``.

Forward pipeline (bf16):
  1. one cuBLAS GEMM over the fused, zero-padded weight
     [q | k | v | value_gate | output_gate | idx_q | idx_k | idx_w | pad]
     (the reference's separate projections, gsa_ref.py:283-285,100-102,164,178);
  2. ``gsa_rope_gates``: RoPE on q/k + v * sigmoid(value gate);
  3. ``gsa_indexer_scores``: tcgen05 gated indexer over causal key tiles;
  4. ``gsa_topk_select``: per-row top-k -> selection bitmask;
  5. ``gsa_masked_attention``: tcgen05 attention over the selected keys with
     the output gate fused into its epilogue;
  6. o_proj on cuBLAS.
fp32 modules use the same steps with the CUDA-core indexer and the
index-gather attention kernel.  There is no CPU path.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops

try:  # NVTX ranges per stage, no-ops without CUDA (gsa_ref.py:17-24)
    from torch.cuda import nvtx as _nvtx

    _nvtx_push = _nvtx.range_push
    _nvtx_pop = _nvtx.range_pop
except Exception:  # pragma: no cover
    def _nvtx_push(msg: str) -> None:
        pass

    def _nvtx_pop() -> None:
        pass


class _Stage:
    """NVTX range around one stage; with ``module._stage_events`` set to a list it
    also records a CUDA event pair on the current stream (used by bench.py to
    time each kernel inside the timed region)."""

    __slots__ = ("mod", "name", "nvtx", "a", "launches")

    def __init__(self, mod, name: str, nvtx: str, launches: int = 1):
        self.mod, self.name, self.nvtx, self.a = mod, name, nvtx, None
        self.launches = launches  # kernels this stage launches

    def __enter__(self):
        _nvtx_push(self.nvtx)
        if self.mod._stage_events is not None:
            self.a = torch.cuda.Event(enable_timing=True)
            self.a.record()
        return self

    def __exit__(self, *exc):
        if self.a is not None:
            b = torch.cuda.Event(enable_timing=True)
            b.record()
            self.mod._stage_events.append((self.name, self.a, b, self.launches))
        _nvtx_pop()
        return False


# ── Rotary embeddings ──────────────────────────────────────────────────────

class RotaryEmbedding(nn.Module):
    """Rotary table holder with the reference's buffers and cache semantics.

    Mirrors gsa_ref.py:43-70: ``inv_freq`` is a persistent buffer (so it is
    rounded to the module dtype by ``.to(dtype)``), ``cos_cached`` /
    ``sin_cached`` are non-persistent and built for 8192 positions at
    construction.  A longer sequence rebuilds the cache from the *current*
    ``inv_freq`` in float32 on the host, exactly as the reference's
    ``_set_cos_sin_cache`` does on CPU (on CUDA the reference's rebuild mixes
    a CPU ``arange`` with a CUDA ``inv_freq`` and raises).  Tables are returned
    in the requested dtype.
    """

    def __init__(self, dim: int, max_seq_len: int = 8192, base: float = 10000.0):
        super().__init__()
        self.dim = dim
        inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2).float() / dim))
        self.register_buffer("inv_freq", inv_freq)
        self._set_cos_sin_cache(max_seq_len)

    def _set_cos_sin_cache(self, seq_len: int) -> None:
        inv = self.inv_freq.detach().cpu()
        t = torch.arange(seq_len, dtype=torch.float32)
        freqs = torch.outer(t, inv)
        emb = torch.cat((freqs, freqs), dim=-1)
        self.register_buffer("cos_cached", emb.cos(), persistent=False)
        self.register_buffer("sin_cached", emb.sin(), persistent=False)

    def forward(self, seq_len: int, device: torch.device, dtype: torch.dtype = None
                ) -> Tuple[torch.Tensor, torch.Tensor]:
        if seq_len > self.cos_cached.shape[0]:
            self._set_cos_sin_cache(seq_len)
            self.cos_cached = self.cos_cached.to(device)
            self.sin_cached = self.sin_cached.to(device)
        # the converted tables are kept until the cache tensors change (rebuild,
        # .to(), in-place edits), so a steady forward launches no conversion kernels
        key = (seq_len, torch.device(device), dtype, self.cos_cached.data_ptr(),
               self.cos_cached._version, self.sin_cached.data_ptr(), self.sin_cached._version)
        hit = getattr(self, "_tables", None)
        if hit is not None and hit[0] == key:
            return hit[1], hit[2]
        cos = self.cos_cached[:seq_len].to(device)
        sin = self.sin_cached[:seq_len].to(device)
        if dtype is not None:
            cos = cos.to(dtype)
            sin = sin.to(dtype)
        self._tables = (key, cos, sin)
        return cos, sin


def apply_rotary_pos_emb(q, k, cos, sin):
    """Reference signature (gsa_ref.py:35-40), computed by the CUDA RoPE kernel."""
    return ops.apply_rotary_pos_emb(q, k, cos, sin)


# ── Gated lightning indexer ────────────────────────────────────────────────

class GatedLightningIndexer(nn.Module):
    """score[q,k] = sum_h sigmoid(w[q,h]) * sigmoid(q_I[q,h].k_I[k] * scale + b[h]), causal.

    Same parameters and initialisation as gsa_ref.py:75-95; ``forward`` returns
    the [B, T, T] float32 score matrix with -inf above the diagonal
    (gsa_ref.py:97-126), computed by ``gsa_indexer_scores``."""

    def __init__(self, hidden_size: int, d_indexer: int = 64, n_idx_heads: int = 4):
        super().__init__()
        self.d_indexer = d_indexer
        self.n_idx_heads = n_idx_heads
        self.scale = 1.0 / math.sqrt(d_indexer)

        self.idx_q_proj = nn.Linear(hidden_size, n_idx_heads * d_indexer, bias=False)
        self.idx_k_proj = nn.Linear(hidden_size, d_indexer, bias=False)
        self.idx_w_proj = nn.Linear(hidden_size, n_idx_heads, bias=True)
        self.idx_bias = nn.Parameter(torch.zeros(n_idx_heads))

        nn.init.xavier_uniform_(self.idx_q_proj.weight, gain=1.0)
        nn.init.xavier_uniform_(self.idx_k_proj.weight, gain=1.0)
        nn.init.xavier_uniform_(self.idx_w_proj.weight, gain=0.1)

    def bias_f32(self) -> torch.Tensor:
        """idx_bias as contiguous float32 (what the kernels read), converted once
        per change of the parameter rather than on every call."""
        p = self.idx_bias
        key = (p.data_ptr(), p._version, p.device, p.dtype)
        hit = getattr(self, "_bias32", None)
        if hit is None or hit[0] != key:
            hit = (key, p.detach().to(torch.float32).contiguous())
            self._bias32 = hit
        return hit[1]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, T, _ = x.shape
        q_idx = self.idx_q_proj(x).view(B, T, self.n_idx_heads, self.d_indexer)
        k_idx = self.idx_k_proj(x)
        w = self.idx_w_proj(x)
        return ops.fused_gated_indexer(q_idx, k_idx, w, self.idx_bias, self.scale, causal=True)


# ── Top-k selector ─────────────────────────────────────────────────────────

class AdaptiveTopKSelector(nn.Module):
    """Fixed k_eff = min(k_base, k_max, T_kv) selection, as gsa_ref.py:131-150.

    ``forward(scores)`` returns (indices int64 [B,T,k], mask bool [B,T,k], k_eff).
    Indices come back in ascending order (the order gsa_opt.py:674-677 sorts
    into); valid slots precede masked filler slots; ties go to the lower index.
    In the default mode ``k_min`` is stored for interface parity; the
    reference never reads it.

    ``adaptive=True`` (opt-in; not part of the reference module) gives each row
    its own k by the variance rule of the reference's notebook
    (gsa_explained.ipynb:575-592): k_r = clamp(floor(k_base * mean_var /
    max(var_r, 1e-6)), k_min, k_max), var_r the variance of row r's valid
    scores and mean_var their mean over the batch (clamped to >= 1e-6).
    ``forward`` then returns (indices int64 [B,T,min(k_max,T_kv)], mask, k per
    row as an int64 [B,T] tensor)."""

    def __init__(self, k_base: int = 2048, k_min: int = 256, k_max: int = 4096,
                 adaptive: bool = False):
        super().__init__()
        self.k_base = k_base
        self.k_min = k_min
        self.k_max = k_max
        self.adaptive = adaptive

    def k_effective(self, t_kv: int) -> int:
        return min(self.k_base, self.k_max, t_kv)

    def forward(self, scores: torch.Tensor):
        B, T, T_kv = scores.shape
        if self.adaptive:
            sc = scores.float().contiguous()
            row_var, var_sum = ops.row_variance(sc, q_pos0=T_kv)
            idx, mask, _, row_k = ops.topk_select_adaptive(
                sc, self.k_base, self.k_min, self.k_max, row_var, var_sum, B * T,
                q_pos0=T_kv, want_bitmask=False)
            return idx.long(), mask, row_k.long()
        k_eff = self.k_effective(T_kv)
        # Every column is a candidate; -inf scores rank last and come back
        # with mask False, whatever the pattern of -inf in the rows.
        idx, mask, _ = ops.topk_select(scores.float().contiguous(), k_eff, q_pos0=T_kv,
                                       want_bitmask=False)
        return idx.long(), mask, k_eff


# ── Gates ──────────────────────────────────────────────────────────────────

class ValueGate(nn.Module):
    """G2: v * sigmoid(W x + b), bias init 0.5 (gsa_ref.py:155-166)."""

    def __init__(self, hidden_size: int):
        super().__init__()
        self.gate_proj = nn.Linear(hidden_size, hidden_size, bias=True)
        nn.init.constant_(self.gate_proj.bias, 0.5)

    def forward(self, v: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        B, T, H, d = v.shape
        return ops.output_gate(v, self.gate_proj(x)).view(B, T, H, d)


class OutputGate(nn.Module):
    """G1: o * sigmoid(W x + b), bias init 0.5 (gsa_ref.py:169-180)."""

    def __init__(self, hidden_size: int):
        super().__init__()
        self.gate_proj = nn.Linear(hidden_size, hidden_size, bias=True)
        nn.init.constant_(self.gate_proj.bias, 0.5)

    def forward(self, output: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        B, T, H, d = output.shape
        return ops.output_gate(output, self.gate_proj(x)).view(B, T, H, d)


# ── Row blocks of the host-buffer forward ───────────────────────────────────

def host_row_block_bounds(T: int, chunks: Optional[int] = None, graphed: bool = False) -> list:
    """Block edges [0, r1, ..., T] of ``forward_host`` for one sequence of T rows.

    Edges sit on 128-row tiles (the kernels' query tile) except the last, and
    the first and last blocks are half the size of the others: nothing overlaps
    the first copy in or the last copy out.  By default there are at most 5
    blocks and at most one per 2048 rows: below that Python's issue of each
    block's launches costs more than the overlap saves (T=4096: 0.96 ms with 2
    blocks, 1.72 ms with 5).  Replayed from a CUDA graph (``graphed``) nothing
    waits on Python, and finer blocks start the computation sooner behind the
    copies in: at most 9 blocks and one per 1024 rows (T=16384: 2.95 ms with 5
    blocks, 2.78 ms with 9, 2.84 ms with 12; T=4096: 0.73 ms with 2, 0.66 ms
    with 4, 0.72 ms with 6)."""
    tiles = (T + 127) // 128
    if chunks is None:
        chunks = max(1, min(9, T // 1024)) if graphed else max(1, min(5, T // 2048))
    n = max(1, min(chunks, tiles))
    if n <= 2:
        cuts = [tiles * i / n for i in range(n + 1)]
    else:
        unit = tiles / (n - 1)
        cuts = [0.0] + [unit * (i - 0.5) for i in range(1, n)] + [float(tiles)]
    return sorted({min(T, 128 * int(round(c))) for c in cuts} | {0, T})


# ── Main module ────────────────────────────────────────────────────────────

class GatedSparseAttention(nn.Module):
    """Gated Sparse Attention forward on B200 (see the module docstring)."""

    def __init__(self, hidden_size: int, num_heads: int, k_max: int = 4096,
                 d_indexer: int = 64, n_idx_heads: int = 4, k_base: int = 2048,
                 k_min: int = 256, adaptive_k: bool = False):
        super().__init__()
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.d_head = hidden_size // num_heads
        self.scale = self.d_head ** -0.5

        self.q_proj = nn.Linear(hidden_size, hidden_size, bias=False)
        self.k_proj = nn.Linear(hidden_size, hidden_size, bias=False)
        self.v_proj = nn.Linear(hidden_size, hidden_size, bias=False)
        self.o_proj = nn.Linear(hidden_size, hidden_size, bias=False)

        self.indexer = GatedLightningIndexer(hidden_size, d_indexer, n_idx_heads)
        # adaptive_k (opt-in, no state): per-row k by the variance rule of
        # AdaptiveTopKSelector(adaptive=True); the default is the reference's fixed k.
        self.topk_selector = AdaptiveTopKSelector(k_base, k_min, k_max, adaptive=adaptive_k)
        self.value_gate = ValueGate(hidden_size)
        self.output_gate = OutputGate(hidden_size)
        self.rotary_emb = RotaryEmbedding(self.d_head)

        self._fused_weight: Optional[torch.Tensor] = None
        self._fused_bias: Optional[torch.Tensor] = None
        # packed weight / bias of the projection GEMM with RoPE and the value
        # gate in its epilogue (bf16, d_head 128); built on first use
        self._packed: Optional[tuple] = None
        # bf16 forwards take that fused projection when the sizes allow; False
        # selects cuBLAS addmm + the separate RoPE/gate kernel
        self.use_fused_epilogue = True
        self._stage_events: Optional[list] = None
        self._streams: dict = {}
        self._workspaces: dict = {}  # (device, stream, slot) -> indexer/top-k scratch
        D, hi, di = hidden_size, n_idx_heads, d_indexer
        # Column layout of the fused projection output (gsa_opt.py:562-571 order).
        self._proj_sizes = [D, D, D, D, D, hi * di, di, hi]
        offs, o = [], 0
        for sz in self._proj_sizes:
            offs.append(o)
            o += sz
        self._proj_offsets = offs
        self._proj_total = o
        # Padded so that every row of the GEMM output is 64-element aligned.
        self._proj_padded = (o + 63) // 64 * 64

    # ---------------------------------------------------------------- weights
    def fuse_projections(self) -> None:
        """Build the fused projection weight/bias.  Call again after changing weights."""
        D = self.hidden_size
        w = torch.cat([
            self.q_proj.weight, self.k_proj.weight, self.v_proj.weight,
            self.value_gate.gate_proj.weight, self.output_gate.gate_proj.weight,
            self.indexer.idx_q_proj.weight, self.indexer.idx_k_proj.weight,
            self.indexer.idx_w_proj.weight,
        ], dim=0).detach()
        pad = self._proj_padded - self._proj_total
        if pad:
            w = torch.cat([w, w.new_zeros(pad, D)], dim=0)
        b = w.new_zeros(self._proj_padded)
        o = self._proj_offsets
        b[o[3]:o[3] + D] = self.value_gate.gate_proj.bias.detach()
        b[o[4]:o[4] + D] = self.output_gate.gate_proj.bias.detach()
        hi = self.indexer.n_idx_heads
        b[o[7]:o[7] + hi] = self.indexer.idx_w_proj.bias.detach()
        self._fused_weight = w.contiguous()
        self._fused_bias = b.contiguous()
        self._packed = None

    def _get_fused_weight(self):
        p = self.q_proj.weight
        if (self._fused_weight is None or self._fused_weight.device != p.device
                or self._fused_weight.dtype != p.dtype):
            self.fuse_projections()
        return self._fused_weight, self._fused_bias

    # ---------------------------------------------------------------- forward
    def project(self, x: torch.Tensor) -> torch.Tensor:
        """Fused projection GEMM: [B, T, D] -> [B, T, padded width] (cuBLAS)."""
        B, T, D = x.shape
        w, b = self._get_fused_weight()
        out = torch.addmm(b, x.reshape(B * T, D), w.t())
        return out.view(B, T, self._proj_padded)

    def split(self, proj: torch.Tensor):
        """Named column views of a fused projection output (no copies)."""
        o, D = self._proj_offsets, self.hidden_size
        hi, di = self.indexer.n_idx_heads, self.indexer.d_indexer
        B, T, _ = proj.shape
        return {
            "q": proj[..., o[0]:o[0] + D], "k": proj[..., o[1]:o[1] + D],
            "v": proj[..., o[2]:o[2] + D], "vg": proj[..., o[3]:o[3] + D],
            "og": proj[..., o[4]:o[4] + D],
            "iq": proj[..., o[5]:o[5] + hi * di].unflatten(-1, (hi, di)),
            "ik": proj[..., o[6]:o[6] + di], "iw": proj[..., o[7]:o[7] + hi],
        }

    def fused_epilogue_ok(self, dtype: torch.dtype) -> bool:
        """Whether ``project_fused`` serves inputs of ``dtype``: bf16 modules with
        128-channel heads and a hidden size that is a multiple of 256."""
        return (self.use_fused_epilogue and dtype == torch.bfloat16
                and self.q_proj.weight.dtype == torch.bfloat16 and self.d_head == 128
                and self.hidden_size % 256 == 0)

    def _get_packed(self):
        p = self.q_proj.weight
        if (self._packed is None or self._packed[0].device != p.device
                or self._packed[0].dtype != p.dtype):
            ix = self.indexer
            self._packed = ops.fused_projection_pack(
                {"q": self.q_proj.weight, "k": self.k_proj.weight, "v": self.v_proj.weight,
                 "vg": self.value_gate.gate_proj.weight, "og": self.output_gate.gate_proj.weight,
                 "iq": ix.idx_q_proj.weight, "ik": ix.idx_k_proj.weight,
                 "iw": ix.idx_w_proj.weight, "vg_bias": self.value_gate.gate_proj.bias,
                 "og_bias": self.output_gate.gate_proj.bias, "iw_bias": ix.idx_w_proj.bias},
                ix.n_idx_heads, ix.d_indexer)
        return self._packed

    def project_fused(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                      pos0: int = 0, seq_len: Optional[int] = None, out: Optional[tuple] = None):
        """Projection GEMM with RoPE and the value gate in its epilogue (one kernel).

        Returns (q, k, v, parts): q, k, v [B, T, D] after RoPE / the value gate,
        and ``parts`` the og / iq / ik / iw views of the rest columns.  Row t of
        a sequence takes row pos0 + t of the rotary tables cos / sin."""
        wp, bp = self._get_packed()
        ix = self.indexer
        q, k, v, rest = ops.fused_projection(x, wp, bp, self.num_heads, ix.n_idx_heads,
                                             ix.d_indexer, cos, sin, pos0, seq_len, out)
        return q, k, v, self.split_rest(rest)

    def split_rest(self, rest: torch.Tensor) -> dict:
        """og / iq / ik / iw views of a fused projection's rest columns."""
        D = self.hidden_size
        hi, di = self.indexer.n_idx_heads, self.indexer.d_indexer
        o_iq, o_ik = D, D + hi * di
        o_iw = o_ik + di
        return {"og": rest[..., :D], "iq": rest[..., o_iq:o_ik].unflatten(-1, (hi, di)),
                "ik": rest[..., o_ik:o_iw], "iw": rest[..., o_iw:o_iw + hi]}

    def select_rows(self, parts: dict, ik_all: torch.Tensor, q_pos0: int,
                    tkv: Optional[int] = None, bitmask_out: Optional[torch.Tensor] = None):
        """Indexer + top-k for a block of query rows (``parts`` = the block's projection views).

        Returns the selection: a bitmask [B, Tq, W] for the tensor-core attention
        (bf16, d_head = 128; written into ``bitmask_out`` when given, else into
        scratch kept per stream), else (indices, mask) for the index-gather path."""
        Tkv = ik_all.shape[1] if tkv is None else tkv
        bf16_tc = parts["iq"].dtype == torch.bfloat16 and self.d_head == 128
        B, Tq = parts["iq"].shape[:2]
        sel = self.topk_selector
        if sel.adaptive:
            need = ops.indexer_topk_adaptive_workspace_size(B, Tq, Tkv)
            ws, bm = self._scratch(parts["iq"].device, B, Tq, Tkv, bf16_tc and bitmask_out is None,
                                   need)
            bm = bitmask_out if bitmask_out is not None else bm
            with _Stage(self, "k:indexer_topk", "gsa_b200/indexer_topk", launches=4):
                idx, mask, bitmask, _ = ops.indexer_topk_adaptive(
                    parts["iq"], ik_all, parts["iw"], self.indexer.bias_f32(), self.indexer.scale,
                    sel.k_base, sel.k_min, sel.k_max, q_pos0=q_pos0, tkv=Tkv,
                    want_indices=not bf16_tc, want_mask=not bf16_tc, want_bitmask=bf16_tc,
                    workspace=ws, bitmask_out=bm)
            return bitmask if bf16_tc else (idx, mask)
        k_eff = sel.k_effective(Tkv)
        ws, bm = self._scratch(parts["iq"].device, B, Tq, Tkv, bf16_tc and bitmask_out is None,
                               ops.indexer_topk_workspace_size(B, Tq, Tkv))
        bm = bitmask_out if bitmask_out is not None else bm
        with _Stage(self, "k:indexer_topk", "gsa_b200/indexer_topk", launches=2):
            idx, mask, bitmask = ops.indexer_topk(
                parts["iq"], ik_all, parts["iw"], self.indexer.bias_f32(), self.indexer.scale, k_eff,
                q_pos0=q_pos0, tkv=Tkv, want_indices=not bf16_tc, want_mask=not bf16_tc,
                want_bitmask=bf16_tc, workspace=ws, bitmask_out=bm)
        return bitmask if bf16_tc else (idx, mask)

    def select_blocks(self, blocks, var_reduce=None, var_rows: Optional[int] = None) -> list:
        """Selections for several blocks of query rows: ``blocks`` is a list of
        (parts, ik_all, q_pos0, tkv) as ``select_rows`` takes them.

        With a fixed k the blocks are independent.  With adaptive k every row's
        k depends on the mean row variance of the whole batch, so all blocks'
        scores and variances are computed first, their variance sums added,
        ``var_reduce(total)`` (e.g. an all-reduce over the ranks holding the rest
        of the batch) applied in place, and the blocks selected with
        ``var_rows`` rows in the mean (default: the blocks' own rows)."""
        sel = self.topk_selector
        if not sel.adaptive or (len(blocks) == 1 and var_reduce is None):
            return [self.select_rows(p, ik, q0, tkv) for p, ik, q0, tkv in blocks]
        staged, total, rows = [], None, 0
        for slot, (p, ik, q0, tkv) in enumerate(blocks):
            B, Tq = p["iq"].shape[:2]
            bf16_tc = p["iq"].dtype == torch.bfloat16 and self.d_head == 128
            need = ops.indexer_topk_adaptive_workspace_size(B, Tq, tkv)
            ws, bm = self._scratch(p["iq"].device, B, Tq, tkv, bf16_tc, need, slot=slot)
            scores, row_var, var_sum = ops.adaptive_workspace_views(ws, B, Tq, tkv)
            with _Stage(self, "k:indexer_topk", "gsa_b200/indexer_topk", launches=3):
                ops.indexer_scores(p["iq"], ik, p["iw"], self.indexer.bias_f32(),
                                   self.indexer.scale, q_pos0=q0, tkv=tkv, fill_upper=False,
                                   out=scores)
                ops.row_variance(scores[:, :, :tkv], q_pos0=q0, out=(row_var, var_sum))
            total = var_sum.clone() if total is None else total + var_sum
            rows += B * Tq
            staged.append((scores[:, :, :tkv], row_var, q0, bf16_tc, bm))
        if var_reduce is not None:
            var_reduce(total)
        out = []
        for scores, row_var, q0, bf16_tc, bm in staged:
            with _Stage(self, "k:topk_adaptive", "gsa_b200/indexer_topk"):
                idx, mask, bitmask, _ = ops.topk_select_adaptive(
                    scores, sel.k_base, sel.k_min, sel.k_max, row_var, total,
                    var_rows if var_rows is not None else rows, q_pos0=q0,
                    want_indices=not bf16_tc, want_mask=not bf16_tc, want_bitmask=bf16_tc,
                    bitmask_out=bm)
            out.append(bitmask if bf16_tc else (idx, mask))
        return out

    def attend_selected(self, parts: dict, selection, k_all: torch.Tensor, v_all: torch.Tensor,
                        q_rows: torch.Tensor, q_pos0: int) -> torch.Tensor:
        """Sparse attention (+ output gate) of a block of query rows over its selection."""
        B, Tq, D = q_rows.shape
        Tkv = k_all.shape[1]
        H, d = self.num_heads, self.d_head
        if torch.is_tensor(selection):
            with _Stage(self, "k:masked_attention", "gsa_b200/sparse_attn"):
                return ops.masked_attention(q_rows, k_all, v_all, selection, self.scale, H,
                                            og=parts["og"], q_pos0=q_pos0)
        idx, mask = selection
        with _Stage(self, "k:gather_attention", "gsa_b200/sparse_attn"):
            attn = ops.gather_attention(q_rows.view(B, Tq, H, d), k_all.view(B, Tkv, H, d),
                                        v_all.view(B, Tkv, H, d), idx, mask, self.scale)
        with _Stage(self, "k:output_gate", "gsa_b200/output_gate"):
            return ops.output_gate(attn.view(B, Tq, D), parts["og"])

    def attend_rows(self, parts: dict, k_all: torch.Tensor, v_all: torch.Tensor,
                    ik_all: torch.Tensor, q_rows: torch.Tensor, q_pos0: int) -> torch.Tensor:
        """Indexer -> top-k -> sparse attention (+ output gate) for a block of query rows.

        ``parts`` holds the block's own projection views (``iq``, ``iw``, ``og``);
        ``q_rows`` its RoPE'd queries [B, Tq, D]; ``k_all``/``v_all``/``ik_all``
        cover keys [0, Tkv).  Row r of the block is sequence position q_pos0 + r.
        Returns the gated attention output [B, Tq, D] (before o_proj)."""
        sel = self.select_rows(parts, ik_all, q_pos0, tkv=k_all.shape[1])
        return self.attend_selected(parts, sel, k_all, v_all, q_rows, q_pos0)

    def _scratch(self, device: torch.device, B: int, Tq: int, Tkv: int, want_bitmask: bool,
                 need: int, slot: int = 0):
        """Score scratch (``need`` bytes) and selection bitmask for indexer + top-k,
        kept per (device, current stream, slot); blocks whose selections must
        coexist use different slots.

        Reusing them keeps a 1 GiB-scale allocation (T=16K) out of every
        forward.  Work on one stream runs in order, so a later call cannot
        overwrite scores an earlier call still reads.  The bitmask is read by
        the attention of the same forward; a later selection on the side
        stream waits for that attention (``side.wait_stream(main)`` at the top
        of ``forward``), and ``attend_rows`` selects and attends on one stream."""
        key = (device, torch.cuda.current_stream(device).cuda_stream, slot)
        ws, bm = self._workspaces.get(key, (None, None))
        if ws is None or ws.numel() < need:
            ws = torch.empty(need, dtype=torch.uint8, device=device)
        shape = (B, Tq, ops.bitmask_words(Tkv))
        n_words = B * Tq * shape[2]
        if want_bitmask and (bm is None or bm.numel() < n_words):
            bm = torch.empty(n_words, dtype=torch.int32, device=device)
        self._workspaces[key] = (ws, bm)
        return ws, (bm[:n_words].view(shape) if want_bitmask else None)

    def _side_stream(self, device: torch.device) -> torch.cuda.Stream:
        """The stream of indexer + top-k.  It has high priority: that branch is
        the longer of the two that follow the projection (RoPE + gates is the
        other), so its blocks go first whenever both have blocks waiting."""
        s = self._streams.get(device)
        if s is None:
            s = torch.cuda.Stream(device=device, priority=-1)
            self._streams[device] = s
        return s

    def forward(self, x: torch.Tensor, attention_mask: Optional[torch.Tensor] = None
                ) -> torch.Tensor:
        return self._forward_impl(x)

    def graphed(self, shape, dtype: Optional[torch.dtype] = None, device=None,
                warmup: int = 2) -> "GraphedForward":
        """The forward for inputs of ``shape`` captured as a CUDA graph
        (``GraphedForward``); ``dtype`` defaults to the parameters' dtype."""
        p = self.q_proj.weight
        return GraphedForward(self, shape, p.dtype if dtype is None else dtype,
                              p.device if device is None else device, warmup)

    def _forward_impl(self, x: torch.Tensor, var_reduce=None,
                      var_rows: Optional[int] = None,
                      side: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """``forward``; ``var_reduce`` / ``var_rows`` as in ``select_blocks`` let a
        caller whose batch spans several processes average adaptive k's row
        variances over all of it.  ``side`` replaces the module's side stream
        (a captured graph keeps its own, and with it its own scratch)."""
        if not x.is_cuda:
            raise RuntimeError("gsa_b200.GatedSparseAttention runs on CUDA only (no CPU path)")
        if x.dtype not in (torch.bfloat16, torch.float32):
            raise RuntimeError(f"unsupported dtype {x.dtype}")
        B, T, D = x.shape
        x = x.contiguous()
        _nvtx_push("gsa_b200/forward")
        cos, sin = self.rotary_emb(T, x.device, x.dtype)
        main = torch.cuda.current_stream(x.device)
        side = self._side_stream(x.device) if side is None else side
        if self.fused_epilogue_ok(x.dtype):
            # RoPE and the value gate run in the projection GEMM's epilogue; the
            # indexer + top-k then run alone (gsa_opt.py:654-711 runs them beside
            # the element-wise track_B work)
            with _Stage(self, "k:proj_rope_gates", "gsa_b200/fused_proj_rope"):
                q, k, v, parts = self.project_fused(x, cos, sin)
            side.wait_stream(main)
            with torch.cuda.stream(side):
                sel = self.select_blocks([(parts, parts["ik"], 0, T)], var_reduce, var_rows)[0]
        else:
            with _Stage(self, "lib:proj_gemm", "gsa_b200/fused_proj"):
                proj = self.project(x)
            parts = self.split(proj)
            # Two streams, as the reference's pipeline (gsa_opt.py:654-711): the
            # indexer + top-k (tensor/MUFU-bound) run beside RoPE + value gate
            # (HBM-bound); the attention waits for both.
            side.wait_stream(main)
            with torch.cuda.stream(side):
                sel = self.select_blocks([(parts, parts["ik"], 0, T)], var_reduce, var_rows)[0]
            with _Stage(self, "k:rope_gates", "gsa_b200/rope_gates"):
                q, k, v = ops.rope_gates(parts["q"], parts["k"], cos, sin, self.num_heads,
                                         v_src=parts["v"], vg_src=parts["vg"])
        main.wait_stream(side)
        if isinstance(sel, tuple):  # index lists are new tensors; the bitmask is kept scratch
            for t in sel:
                t.record_stream(main)
        attn = self.attend_selected(parts, sel, k, v, q, q_pos0=0)
        with _Stage(self, "lib:o_proj", "gsa_b200/o_proj"):
            out = F.linear(attn.view(B, T, D), self.o_proj.weight)
        _nvtx_pop()
        return out

    def graphed_host(self, shape, dtype: Optional[torch.dtype] = None, device=None,
                     chunks: Optional[int] = None, warmup: int = 2) -> "GraphedForwardHost":
        """``forward_host`` for host inputs of ``shape`` captured as a CUDA graph
        (``GraphedForwardHost``); ``dtype`` defaults to the parameters' dtype."""
        p = self.q_proj.weight
        return GraphedForwardHost(self, shape, p.dtype if dtype is None else dtype,
                                  p.device if device is None else device, chunks, warmup)

    # ------------------------------------------------------- host-buffer forward
    def forward_host(self, x_host: torch.Tensor, out: Optional[torch.Tensor] = None,
                     chunks: Optional[int] = None) -> torch.Tensor:
        """Forward from host memory to host memory with the PCIe copies hidden.

        For callers whose activations live in host memory.  ``x_host`` [B, T, D]
        (pinned; pageable input is pinned first) is copied to the current device
        in ``chunks`` pieces on a copy stream while earlier pieces compute, and
        each piece of the output is copied back into ``out`` (a pinned [B, T, D]
        host tensor, allocated if None) as soon as it is done.  Returns ``out``
        after the copies have completed.

        With B == 1 the pieces are blocks of query rows: attention is causal, so
        rows [r0, r1) need only keys [0, r1), which earlier pieces have already
        projected; the kernels take the block through ``q_pos0``.  The first and
        last blocks are half the size of the others, since the first copy in and
        the last copy out are the ones nothing overlaps.  ``chunks`` defaults to
        5, and to fewer for short sequences (at least 2048 rows per block).  With B > 1
        the pieces are groups of whole sequences.  The result equals
        ``forward`` up to the rounding of the projection GEMMs, which cuBLAS may
        block differently for a smaller problem."""
        if x_host.is_cuda:
            raise RuntimeError("forward_host takes a host tensor; use forward for device tensors")
        if x_host.dtype not in (torch.bfloat16, torch.float32):
            raise RuntimeError(f"unsupported dtype {x_host.dtype}")
        B, T, D = x_host.shape
        dev = torch.device("cuda", torch.cuda.current_device())
        x_host = x_host.contiguous()
        if not x_host.is_pinned():
            x_host = x_host.pin_memory()
        if out is None:
            out = torch.empty(B, T, D, dtype=x_host.dtype).pin_memory()
        elif out.shape != (B, T, D) or out.dtype != x_host.dtype or out.is_cuda:
            raise ValueError(f"out must be a host [{B}, {T}, {D}] {x_host.dtype} tensor")
        compute = torch.cuda.current_stream(dev)
        h2d, d2h = self._copy_streams(dev)
        self._issue_host(x_host, out, chunks, dev, compute, h2d, d2h, self._side_stream(dev))
        d2h.synchronize()
        return out

    def _issue_host(self, x_host, out, chunks, dev, compute, h2d, d2h, side, keep=None,
                    graphed=False):
        """Queue ``forward_host``'s copies and kernels without waiting for them;
        on return ``compute`` is ordered after the last copy out.  With ``keep``
        (a list; CUDA-graph capture) the device buffers are appended to it
        instead of being handed to the allocator's cross-stream tracking."""
        B, T, D = x_host.shape
        h2d.wait_stream(compute)  # device buffers below come from the compute stream's pool
        adaptive = self.topk_selector.adaptive
        if B > 1 or adaptive:
            # adaptive k averages row variances over the whole batch: one piece
            groups = 1 if adaptive else max(1, min(5 if chunks is None else chunks, B))
            bounds = [B * i // groups for i in range(groups + 1)]
            x_dev = torch.empty(B, T, D, device=dev, dtype=x_host.dtype)
            for b0, b1 in zip(bounds[:-1], bounds[1:]):
                with torch.cuda.stream(h2d):
                    x_dev[b0:b1].copy_(x_host[b0:b1], non_blocking=True)
                compute.wait_stream(h2d)
                y = self._forward_impl(x_dev[b0:b1], side=side)
                d2h.wait_stream(compute)
                with torch.cuda.stream(d2h):
                    out[b0:b1].copy_(y, non_blocking=True)
                if keep is None:
                    y.record_stream(d2h)
                else:
                    keep.append(y)
            if keep is not None:
                keep.append(x_dev)
        else:
            self._forward_host_rows(x_host, out, chunks, dev, compute, h2d, d2h, side, keep,
                                    graphed)
        compute.wait_stream(d2h)

    def _copy_streams(self, device: torch.device):
        key = ("copy", device)
        pair = self._streams.get(key)
        if pair is None:
            pair = (torch.cuda.Stream(device=device), torch.cuda.Stream(device=device))
            self._streams[key] = pair
        return pair

    def _forward_host_rows(self, x_host, out, chunks, dev, compute, h2d, d2h, side, keep,
                           graphed):
        """B == 1: row blocks [r0, r1) in sequence order, keys [0, r1) for each.

        Two compute streams: the side stream prepares block c (projection GEMM,
        indexer + top-k into block c's rows of a whole-sequence bitmask, RoPE +
        value gate) as soon as its input has arrived, and the current stream
        runs block c's attention and o_proj once block c is prepared.  The
        preparation of block c+1 therefore fills the SMs that the tail of
        block c's attention leaves idle."""
        _, T, D = x_host.shape
        H = self.num_heads
        bounds = host_row_block_bounds(T, chunks, graphed)
        # the copies in go first: everything else waits on them
        x_dev = torch.empty(1, T, D, device=dev, dtype=x_host.dtype)
        done_in = []
        for r0, r1 in zip(bounds[:-1], bounds[1:]):
            with torch.cuda.stream(h2d):
                x_dev[:, r0:r1].copy_(x_host[:, r0:r1], non_blocking=True)
                e = torch.cuda.Event()
                e.record(h2d)
                done_in.append(e)
        fused = self.fused_epilogue_ok(x_host.dtype)
        cos, sin = self.rotary_emb(T, dev, x_host.dtype)
        if fused:  # RoPE and the value gate in the projection GEMM's epilogue
            self._get_packed()
            ix = self.indexer
            proj = torch.empty(1, T, ops.fused_projection_rest_width(D, ix.n_idx_heads,
                                                                     ix.d_indexer),
                               device=dev, dtype=x_host.dtype)
            parts_all = self.split_rest(proj)
        else:
            w, bias = self._get_fused_weight()
            proj = torch.empty(1, T, self._proj_padded, device=dev, dtype=x_host.dtype)
            parts_all = self.split(proj)
        q = torch.empty(1, T, D, device=dev, dtype=x_host.dtype)
        k = torch.empty_like(q)
        v = torch.empty_like(q)
        attn = torch.empty_like(q)
        y = torch.empty_like(q)
        bf16_tc = x_host.dtype == torch.bfloat16 and self.d_head == 128
        # one contiguous [1, r1 - r0, bitmask_words(r1)] selection per block, all alive at once
        bm_sizes = [(r1 - r0) * ops.bitmask_words(r1) for r0, r1 in zip(bounds[:-1], bounds[1:])]
        bm_flat = (torch.empty(sum(bm_sizes), device=dev, dtype=torch.int32) if bf16_tc
                   else None)
        bm_offs = [sum(bm_sizes[:i]) for i in range(len(bm_sizes))]
        if keep is not None:
            keep.extend([x_dev, proj, q, k, v, attn, y, bm_flat])
        side.wait_stream(compute)  # the buffers above come from the current stream's pool
        blocks = list(zip(bounds[:-1], bounds[1:]))

        def prepare(c):
            r0, r1 = blocks[c]
            with torch.cuda.stream(side):
                side.wait_event(done_in[c])
                if fused:
                    with _Stage(self, "k:proj_rope_gates", "gsa_b200/fused_proj_rope"):
                        self.project_fused(x_dev[:, r0:r1], cos, sin, pos0=r0, seq_len=r1 - r0,
                                           out=(q[:, r0:r1], k[:, r0:r1], v[:, r0:r1],
                                                proj[:, r0:r1]))
                else:
                    with _Stage(self, "lib:proj_gemm", "gsa_b200/fused_proj"):
                        torch.addmm(bias, x_dev[0, r0:r1], w.t(), out=proj[0, r0:r1])
                rows = {name: t[:, r0:r1] for name, t in parts_all.items()}
                bm_c = (bm_flat[bm_offs[c]:bm_offs[c] + bm_sizes[c]].view(
                    1, r1 - r0, ops.bitmask_words(r1)) if bf16_tc else None)
                sel = self.select_rows(rows, parts_all["ik"][:, :r1], q_pos0=r0, tkv=r1,
                                       bitmask_out=bm_c)
                if not fused:
                    with _Stage(self, "k:rope_gates", "gsa_b200/rope_gates"):
                        ops.rope_gates(rows["q"], rows["k"], cos[r0:r1], sin[r0:r1], H,
                                       v_src=rows["v"], vg_src=rows["vg"],
                                       out=(q[:, r0:r1], k[:, r0:r1], v[:, r0:r1]))
                e = torch.cuda.Event()
                e.record(side)
            return e, rows, sel

        # issue order: the preparation of block c+1 is queued before the attention
        # of block c, so neither stream waits on the host
        prepared = [prepare(0)]
        for c, (r0, r1) in enumerate(blocks):
            if c + 1 < len(blocks):
                prepared.append(prepare(c + 1))
            e, rows, sel = prepared[c]
            compute.wait_event(e)
            if isinstance(sel, tuple):
                for t in sel:
                    if keep is None:
                        t.record_stream(compute)
                    else:
                        keep.append(t)
            if torch.is_tensor(sel):
                with _Stage(self, "k:masked_attention", "gsa_b200/sparse_attn"):
                    ops.masked_attention(q[:, r0:r1], k[:, :r1], v[:, :r1], sel, self.scale, H,
                                         og=rows["og"], q_pos0=r0, out=attn[:, r0:r1])
            else:
                attn[:, r0:r1] = self.attend_selected(rows, sel, k[:, :r1], v[:, :r1],
                                                      q[:, r0:r1], q_pos0=r0)
            with _Stage(self, "lib:o_proj", "gsa_b200/o_proj"):
                torch.mm(attn[0, r0:r1], self.o_proj.weight.t(), out=y[0, r0:r1])
            d2h.wait_stream(compute)
            with torch.cuda.stream(d2h):
                out[:, r0:r1].copy_(y[:, r0:r1], non_blocking=True)
        compute.wait_stream(side)
        if keep is None:
            y.record_stream(d2h)


# ── CUDA-graph replay ──────────────────────────────────────────────────────

class GraphedForward:
    """``module(x)`` for one input shape, captured once as a CUDA graph.

    No counterpart in the reference, which launches every step from Python.
    One forward issues about a dozen kernels and copies on two streams, plus
    the Python around them; for short sequences (T of a few thousand and
    below) that host work, not the GPU, sets the step time.  A replay issues
    the whole forward as one graph launch on the caller's current stream.

    The graph owns its input buffer ``x`` and its output ``out``: a call copies
    its argument into ``x`` (skip it by writing ``x`` directly and calling with
    no argument), replays, and returns ``out``, which the next replay
    overwrites.  The captured side stream is private to the graph, and so is
    the indexer/top-k scratch, so replays and eager calls of the module do not
    share buffers.  Weights are captured by address: after changing them call
    ``module.fuse_projections()`` and capture again.
    """

    def __init__(self, module: "GatedSparseAttention", shape, dtype: torch.dtype,
                 device=None, warmup: int = 2):
        device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("GraphedForward needs a CUDA device")
        if module._stage_events is not None:
            raise RuntimeError("per-stage timing events cannot be captured; disable them first")
        self.module = module
        self.x = torch.zeros(tuple(shape), dtype=dtype, device=device)
        self._main = torch.cuda.Stream(device=device)
        self._side = torch.cuda.Stream(device=device, priority=-1)  # as the module's side stream
        self._main.wait_stream(torch.cuda.current_stream(device))
        with torch.no_grad(), torch.cuda.stream(self._main):
            # eager warm-up on the capture streams: builds the fused weight,
            # the rotary tables and this graph's scratch outside the graph pool
            for _ in range(max(1, warmup)):
                module._forward_impl(self.x, side=self._side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph, stream=self._main):
            self.out = module._forward_impl(self.x, side=self._side)
        # the graph reads these by address: hold them even if the module later
        # replaces its caches (new sequence length, dtype, re-fused weights)
        self._held = (module._fused_weight, module._fused_bias, module._packed,
                      getattr(module.indexer, "_bias32", None),
                      getattr(module.rotary_emb, "_tables", None), dict(module._workspaces))

    def __call__(self, x: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x is not None:
            if x.shape != self.x.shape or x.dtype != self.x.dtype:
                raise RuntimeError(f"captured for {tuple(self.x.shape)} {self.x.dtype}, "
                                   f"got {tuple(x.shape)} {x.dtype}")
            self.x.copy_(x, non_blocking=True)
        self.graph.replay()
        return self.out


class GraphedForwardHost:
    """``module.forward_host`` for one input shape, captured once as a CUDA graph.

    The graph holds the whole host-to-host pipeline: the pinned copies in, the
    row-block (or batch-group) computation on its two streams and the pinned
    copies out.  Its buffers are pinned host tensors of its own: write the
    activations into ``x`` (or pass them to the call, which copies them there on
    the host: a CPU memcpy of the whole input, which a producer that writes into
    ``x`` directly avoids), and read the result from ``out`` once the call
    returns; the next call overwrites it.  A replay issues the pipeline as one graph launch, so the
    GPU no longer waits for Python to issue each block's kernels while the
    first blocks' inputs arrive.  Captured by address, as ``GraphedForward``.
    """

    def __init__(self, module: "GatedSparseAttention", shape, dtype: torch.dtype,
                 device=None, chunks: Optional[int] = None, warmup: int = 2):
        device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("GraphedForwardHost needs a CUDA device")
        if module._stage_events is not None:
            raise RuntimeError("per-stage timing events cannot be captured; disable them first")
        if dtype not in (torch.bfloat16, torch.float32):
            raise RuntimeError(f"unsupported dtype {dtype}")
        self.module, self.device = module, device
        self.x = torch.zeros(tuple(shape), dtype=dtype).pin_memory()
        self.out = torch.zeros(tuple(shape), dtype=dtype).pin_memory()
        self._main = torch.cuda.Stream(device=device)
        self._side = torch.cuda.Stream(device=device, priority=-1)
        self._h2d = torch.cuda.Stream(device=device)
        self._d2h = torch.cuda.Stream(device=device)
        streams = (self._main, self._h2d, self._d2h, self._side)
        self._main.wait_stream(torch.cuda.current_stream(device))
        with torch.no_grad(), torch.cuda.stream(self._main):
            for _ in range(max(1, warmup)):
                module._issue_host(self.x, self.out, chunks, device, *streams, graphed=True)
        self._main.synchronize()
        self._keep: list = []
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph, stream=self._main):
            module._issue_host(self.x, self.out, chunks, device, *streams, keep=self._keep,
                               graphed=True)
        self._held = (module._fused_weight, module._fused_bias, module._packed,
                      getattr(module.indexer, "_bias32", None),
                      getattr(module.rotary_emb, "_tables", None), dict(module._workspaces))

    def __call__(self, x_host: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x_host is not None:
            if x_host.shape != self.x.shape or x_host.dtype != self.x.dtype or x_host.is_cuda:
                raise RuntimeError(f"captured for a host {tuple(self.x.shape)} {self.x.dtype} "
                                   f"tensor, got {tuple(x_host.shape)} {x_host.dtype} "
                                   f"on {x_host.device}")
            self.x.copy_(x_host)
        stream = torch.cuda.current_stream(self.device)
        self.graph.replay()
        stream.synchronize()
        return self.out
