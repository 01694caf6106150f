"""Multi-GPU GSA forward: one process per GPU, torch.distributed (NCCL) plumbing.

The reference runs on one device only; this module partitions the forward.

* B == 1 (long sequences): causally load-balanced query-row sharding.  The
  sequence is cut into 2P equal blocks and rank r owns blocks r and 2P-1-r
  (a cheap early block and an expensive late one: indexer work per row grows
  with the row position, so the pair costs the same on every rank).  Each rank
  projects only its own rows, applies RoPE / value gate, then all-gathers the
  keys, values and indexer keys (k, v, k_I) so every rank holds [0, T).  Each
  row's indexer, top-k and attention need nothing else, so there is no further
  exchange until the output rows are all-gathered at the end.
* B > 1 (batched serving): sequences are independent; rank r runs B/P of them
  and the outputs are all-gathered.

Only NCCL collectives cross GPUs (no peer-memory loads of any kind).
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import ops
from .gsa import _Stage

Block = Tuple[int, int]


def zigzag_blocks(T: int, world: int, rank: int) -> List[Block]:
    """Blocks [start, end) owned by ``rank``: r and 2P-1-r of 2P equal blocks."""
    nb = 2 * world
    if T % nb:
        raise ValueError(f"T={T} must be a multiple of 2*world={nb} for row sharding")
    b = T // nb
    return [(rank * b, (rank + 1) * b), ((nb - 1 - rank) * b, (nb - rank) * b)]


def causal_row_cost(blocks: Sequence[Block], k: int) -> Tuple[int, int]:
    """(indexer pairs, attention pairs) of a set of row blocks: sum of t+1 and min(t+1, k)."""
    idx = att = 0
    for s, e in blocks:
        idx += (e * (e + 1) - s * (s + 1)) // 2
        # rows t in [s, e): min(t+1, k)
        lo, hi = s, min(e, k)
        if hi > lo:
            att += (hi * (hi + 1) - lo * (lo + 1)) // 2
        att += max(0, e - max(s, k)) * k
    return idx, att


def all_gather_equal(t: torch.Tensor, group) -> torch.Tensor:
    """All-gather equally shaped tensors -> [world, *t.shape] (NCCL or gloo)."""
    world = dist.get_world_size(group)
    t = t.contiguous()
    out = torch.empty((world, *t.shape), dtype=t.dtype, device=t.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, t, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), t, group=group)
    return out


def all_gather_async(out: torch.Tensor, t: torch.Tensor, group):
    """Start an all-gather of equally shaped ``t`` into ``out`` [world, *t.shape]
    (contiguous); returns the work handle (NCCL or gloo)."""
    t = t.contiguous()
    if dist.get_backend(group) == "nccl":
        return dist.all_gather_into_tensor(out, t, group=group, async_op=True)
    return dist.all_gather(list(out.unbind(0)), t, group=group, async_op=True)


class RowBlockGather:
    """The full [1, T, W] output from every rank's two zig-zag row blocks,
    gathered one block at a time so that a block's all-gather overlaps the
    work that follows it.

    Rank r's first block is sequence block r, so the ranks' first blocks
    gathered rank-major are sequence blocks 0..P-1 and land in place; rank r's
    second block is sequence block 2P-1-r, so the second gather comes in
    reverse order and is copied into place once it has arrived."""

    def __init__(self, T: int, world: int, width: int, dtype, device):
        self.world, self.n = world, T // (2 * world)
        self.out = torch.empty(1, T, width, dtype=dtype, device=device)
        self.late = torch.empty(world, self.n, width, dtype=dtype, device=device)
        self.works = []

    def add(self, i: int, block: torch.Tensor, group) -> None:
        """Start gathering this rank's block ``i`` (0 or 1), [n, W]."""
        P, n = self.world, self.n
        target = self.out[0, :P * n].view(P, n, -1) if i == 0 else self.late
        self.works.append(all_gather_async(target, block, group))

    def finish(self) -> torch.Tensor:
        for w in self.works:
            w.wait()
        P, n = self.world, self.n
        self.out[0, P * n:].copy_(self.late.flip(0).reshape(P * n, -1))
        return self.out


def zigzag_order(T: int, world: int, device) -> torch.Tensor:
    """For each sequence row, its row in the rank-major all-gather of zig-zag shards."""
    src = torch.empty(T, dtype=torch.long)
    tl = T // world
    for r in range(world):
        off = 0
        for s, e in zigzag_blocks(T, world, r):
            src[s:e] = torch.arange(r * tl + off, r * tl + off + (e - s))
            off += e - s
    return src.to(device)


def unshard_rows(g: torch.Tensor, order: torch.Tensor) -> torch.Tensor:
    """[world, Tl, W] gathered shards -> [1, T, W] in sequence order (one gather kernel)."""
    return g.reshape(-1, g.shape[-1]).index_select(0, order).unsqueeze(0)


def gather_rows(local: torch.Tensor, T: int, group, order: torch.Tensor = None) -> torch.Tensor:
    """Reassemble zig-zag row shards [1, Tl, W] from every rank into [1, T, W] in sequence order."""
    world = dist.get_world_size(group)
    g = all_gather_equal(local[0], group)  # [world, Tl, W]
    if order is None:
        order = zigzag_order(T, world, local.device)
    return unshard_rows(g, order)


def gather_batch(local: torch.Tensor, group) -> torch.Tensor:
    """Reassemble batch shards [B/P, T, W] into [B, T, W]."""
    g = all_gather_equal(local, group)
    return g.reshape(-1, *local.shape[1:])


class ShardedGSA:
    """Runs a GatedSparseAttention forward sharded over the ranks of ``group``.

    ``local_input(x)`` picks this rank's share of a full input; ``__call__``
    takes that share (on this rank's GPU) and returns the FULL output on every
    rank.  ``forward_host(x_local_host)`` runs the same forward from this rank's
    share in pinned host memory and returns this rank's rows of the output in
    host memory (the whole output is the union of the ranks' returns)."""

    def __init__(self, model, group, T: int, B: int):
        self.model = model
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.T, self.B = T, B
        self.mode = "rows" if B == 1 else "batch"
        if self.mode == "rows":
            self.blocks = zigzag_blocks(T, self.world, self.rank)
        else:
            if B % self.world:
                raise ValueError(f"B={B} must be a multiple of world={self.world}")
            per = B // self.world
            self.b0, self.b1 = self.rank * per, (self.rank + 1) * per
        self._pos = None
        self._order = None
        self._host_out = None
        self._bitmasks = None
        # K/V all-gathers run on a high-priority NCCL stream of their own group, beside
        # the indexer + top-k (new_group is collective: every rank builds it here)
        self.kv_group = group
        if self.mode == "rows" and dist.get_backend(group) == "nccl":
            opts = dist.ProcessGroupNCCL.Options()
            opts.is_high_priority_stream = True
            self.kv_group = dist.new_group(ranks=dist.get_process_group_ranks(group),
                                           backend="nccl", pg_options=opts)

    # ---------------------------------------------------------------- inputs
    def local_input(self, x: torch.Tensor) -> torch.Tensor:
        if self.mode == "rows":
            return torch.cat([x[:, s:e] for s, e in self.blocks], dim=1).contiguous()
        return x[self.b0:self.b1].contiguous()

    def _row_order(self, device) -> torch.Tensor:
        if self._order is None or self._order.device != device:
            self._order = zigzag_order(self.T, self.world, device)
        return self._order

    def _block_bitmasks(self, device):
        """One selection bitmask per row block, alive together (both blocks select
        before either attends)."""
        key = (device, tuple(self.blocks))
        if self._bitmasks is None or self._bitmasks[0] != key:
            bms = [torch.empty(1, e - s, ops.bitmask_words(e), device=device, dtype=torch.int32)
                   for s, e in self.blocks]
            self._bitmasks = (key, bms)
        return self._bitmasks[1]

    def _positions(self, device) -> torch.Tensor:
        if self._pos is None or self._pos.device != device:
            self._pos = torch.cat([torch.arange(s, e) for s, e in self.blocks]).to(device)
        return self._pos

    # ---------------------------------------------------------------- forward
    def __call__(self, x_local: torch.Tensor, gather: bool = True) -> torch.Tensor:
        """Sharded forward of this rank's share.  Returns the full output on every
        rank, or with ``gather=False`` only this rank's rows (in the order of
        ``local_input``), which skips the output all-gather."""
        return self._forward(x_local, gather=gather)

    def _sum_over_ranks(self, t: torch.Tensor) -> None:
        """In-place sum over the group: adaptive k's row-variance total."""
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def _forward(self, x_local: torch.Tensor, gather: bool) -> torch.Tensor:
        if self.mode == "batch":
            if self.model.topk_selector.adaptive:
                y = self.model._forward_impl(x_local, var_reduce=self._sum_over_ranks,
                                             var_rows=self.B * self.T)
            else:
                y = self.model(x_local)
            if not gather:
                return y
            with _Stage(self.model, "comm:out_allgather", "gsa_b200/out_allgather"):
                return gather_batch(y, self.group)
        return self._forward_rows(x_local, gather)

    def _forward_rows(self, x_loc: torch.Tensor, gather: bool = True) -> torch.Tensor:
        m = self.model
        if m.fused_epilogue_ok(x_loc.dtype):
            # RoPE and the value gate in the projection's epilogue, with the
            # rotary table rows of this rank's positions
            cos, sin = m.rotary_emb(self.T, x_loc.device, x_loc.dtype)
            pos = self._positions(x_loc.device)
            with _Stage(m, "k:proj_rope_gates", "gsa_b200/fused_proj_rope"):
                proj = m.project_fused(x_loc, cos.index_select(0, pos), sin.index_select(0, pos))
        else:
            with _Stage(m, "lib:proj_gemm", "gsa_b200/fused_proj"):
                proj = m.project(x_loc)
        if not gather:
            outs = self._rows_from_projection(proj, x_loc.dtype)
            with _Stage(m, "lib:o_proj", "gsa_b200/o_proj"):
                return F.linear(torch.cat(outs, dim=1), m.o_proj.weight)
        # o_proj and the output all-gather per block: the first (early, light)
        # block's gather runs while the second block computes
        gat = RowBlockGather(self.T, self.world, m.hidden_size, x_loc.dtype, x_loc.device)

        def block_out(i, o, n, a):
            with _Stage(m, "lib:o_proj", "gsa_b200/o_proj"):
                y = F.linear(a[0], m.o_proj.weight)
            gat.add(i, y, self.kv_group)

        self._rows_from_projection(proj, x_loc.dtype, per_block=block_out)
        with _Stage(m, "comm:out_allgather_wait", "gsa_b200/out_allgather"):
            return gat.finish()

    def _rows_from_projection(self, proj, dtype, per_block=None) -> list:
        """Everything after the projection GEMM of this rank's rows: gathers,
        RoPE + value gate (unless ``proj`` is the (q, k, v, parts) of
        ``project_fused``, which ran them in its epilogue), selection and
        attention.  Returns the gated attention output of each block ([1, n, D],
        in the order of ``self.blocks``); with ``per_block(i, o, n, attn)`` that
        callback receives each block as soon as it is computed."""
        m = self.model
        T, H = self.T, m.num_heads
        fused = isinstance(proj, tuple)
        parts = proj[3] if fused else m.split(proj)
        dev = parts["ik"].device
        order = self._row_order(dev)
        # the selection needs only the indexer keys of the whole sequence (2 MB at
        # T=16K): gathered while RoPE runs
        ik_loc = parts["ik"][0]
        g_ik = torch.empty((self.world, *ik_loc.shape), dtype=ik_loc.dtype, device=dev)
        w_ik = all_gather_async(g_ik, ik_loc, self.group)
        if fused:
            q, k, v = proj[:3]
        else:
            cos, sin = m.rotary_emb(T, dev, dtype)
            pos = self._positions(dev)
            with _Stage(m, "k:rope_gates", "gsa_b200/rope_gates"):
                q, k, v = ops.rope_gates(parts["q"], parts["k"], cos.index_select(0, pos),
                                         sin.index_select(0, pos), H, v_src=parts["v"],
                                         vg_src=parts["vg"])
        # keys and values of the whole sequence: gathered while the blocks select
        gk = torch.empty((self.world, *k.shape[1:]), dtype=k.dtype, device=dev)
        gv = torch.empty_like(gk)
        if dist.get_backend(self.kv_group) == "nccl":
            wk = dist.all_gather_into_tensor(gk, k[0], group=self.kv_group, async_op=True)
            wv = dist.all_gather_into_tensor(gv, v[0], group=self.kv_group, async_op=True)
        else:
            wk = dist.all_gather(list(gk.unbind(0)), k[0].contiguous(), group=self.kv_group,
                                 async_op=True)
            wv = dist.all_gather(list(gv.unbind(0)), v[0].contiguous(), group=self.kv_group,
                                 async_op=True)
        with _Stage(m, "comm:ik_allgather_wait", "gsa_b200/ik_allgather"):
            w_ik.wait()
            ik_full = unshard_rows(g_ik, order)
        blocks, off = [], 0
        for s, e in self.blocks:
            n = e - s
            pb = {key: parts[key][:, off:off + n] for key in ("iq", "iw", "og")}
            blocks.append((pb, s, e, off, n))
            off += n
        if m.topk_selector.adaptive:
            # every row's k needs the mean row variance over all ranks' rows
            sels = m.select_blocks([(pb, ik_full[:, :e], s, e) for pb, s, e, _, _ in blocks],
                                   var_reduce=self._sum_over_ranks, var_rows=self.B * T)
        else:
            bms = self._block_bitmasks(dev)
            sels = [m.select_rows(pb, ik_full[:, :e], s, tkv=e, bitmask_out=bm)
                    for (pb, s, e, _, _), bm in zip(blocks, bms)]
        # the part of the K/V all-gathers that the selection did not hide
        with _Stage(m, "comm:kv_allgather_wait", "gsa_b200/kv_allgather_wait"):
            wk.wait()
            wv.wait()
            k_full = unshard_rows(gk, order)
            v_full = unshard_rows(gv, order)
        outs = []
        for i, ((pb, s, e, o, n), sel) in enumerate(zip(blocks, sels)):
            a = m.attend_selected(pb, sel, k_full[:, :e], v_full[:, :e], q[:, o:o + n], q_pos0=s)
            if per_block is not None:
                per_block(i, o, n, a)
            outs.append(a)
        return outs

    def forward_host(self, x_local_host: torch.Tensor) -> torch.Tensor:
        """This rank's input share from pinned host memory -> device, sharded forward,
        this rank's output rows read back into a pinned host buffer (returned).

        Rows come back in the order of ``local_input`` (this rank's blocks, or
        its sequences); no output all-gather is needed, so each rank copies
        back 1/P of the output.  With row shards the copies overlap the work:
        each block's rows are projected as soon as they have arrived, and each
        block's output rows are copied back while the next block computes."""
        dev = torch.device("cuda", torch.cuda.current_device())
        if not x_local_host.is_pinned():
            x_local_host = x_local_host.pin_memory()
        if self._host_out is None or self._host_out.shape != x_local_host.shape:
            self._host_out = torch.empty(x_local_host.shape,
                                         dtype=x_local_host.dtype).pin_memory()
        if self.mode == "batch":
            out = self._forward(x_local_host.to(dev, non_blocking=True), gather=False)
            self._host_out.copy_(out, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()
            return self._host_out
        m = self.model
        compute = torch.cuda.current_stream(dev)
        h2d, d2h = m._copy_streams(dev)
        h2d.wait_stream(compute)  # device buffers below come from the current stream's pool
        _, Tl, D = x_local_host.shape
        x_dev = torch.empty(1, Tl, D, device=dev, dtype=x_local_host.dtype)
        arrived, off = [], 0
        for s, e in self.blocks:
            with torch.cuda.stream(h2d):
                x_dev[:, off:off + e - s].copy_(x_local_host[:, off:off + e - s],
                                                non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(h2d)
            arrived.append((ev, off, e - s))
            off += e - s
        if m.fused_epilogue_ok(x_local_host.dtype):
            # each block's rows hold the consecutive positions s..e-1
            ix = m.indexer
            rest = torch.empty(1, Tl, ops.fused_projection_rest_width(D, ix.n_idx_heads,
                                                                      ix.d_indexer),
                               device=dev, dtype=x_local_host.dtype)
            q = torch.empty(1, Tl, D, device=dev, dtype=x_local_host.dtype)
            k, v = torch.empty_like(q), torch.empty_like(q)
            cos, sin = m.rotary_emb(self.T, dev, x_local_host.dtype)
            for (ev, o, n), (s, _) in zip(arrived, self.blocks):
                compute.wait_event(ev)
                m.project_fused(x_dev[:, o:o + n], cos, sin, pos0=s, seq_len=n,
                                out=(q[:, o:o + n], k[:, o:o + n], v[:, o:o + n],
                                     rest[:, o:o + n]))
            proj = (q, k, v, m.split_rest(rest))
        else:
            w, bias = m._get_fused_weight()
            proj = torch.empty(1, Tl, m._proj_padded, device=dev, dtype=x_local_host.dtype)
            for ev, o, n in arrived:
                compute.wait_event(ev)
                torch.addmm(bias, x_dev[0, o:o + n], w.t(), out=proj[0, o:o + n])
        y = torch.empty(1, Tl, D, device=dev, dtype=x_local_host.dtype)

        def block_out(i, o, n, a):
            torch.mm(a[0], m.o_proj.weight.t(), out=y[0, o:o + n])
            d2h.wait_stream(compute)
            with torch.cuda.stream(d2h):
                self._host_out[:, o:o + n].copy_(y[:, o:o + n], non_blocking=True)

        self._rows_from_projection(proj, x_local_host.dtype, per_block=block_out)
        y.record_stream(d2h)
        compute.wait_stream(d2h)
        d2h.synchronize()
        return self._host_out
