"""Tensor-level wrappers over the C ABI (``include/gsa_b200.h``).

Each function takes CUDA tensors, checks layouts, allocates its outputs with
torch on the tensors' device and launches on ``torch.cuda.current_stream()``.
There is no CPU path: a CPU tensor or a missing ``libgsa_b200.so`` raises.

The op-level functions of the reference are mirrored with the same names and
argument meaning:
  * ``fused_gated_indexer``  — gsa_triton/gsa_opt.py:143-176
  * ``fused_sparse_attention`` — gsa_triton/gsa_opt.py:349-383
  * ``sparse_attention_ref`` — gsa_triton/gsa_ref.py:202-238 (same kernel)
  * ``apply_rotary_pos_emb`` — gsa_triton/gsa_ref.py:35-40
"""
from __future__ import annotations

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.GSA_DTYPE_BF16, torch.float32: _lib.GSA_DTYPE_F32}


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise RuntimeError(f"gsa_b200 supports bfloat16 and float32, got {t.dtype}") from None


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("gsa_b200 runs only on CUDA tensors (no CPU fallback)")


def _rows(t: torch.Tensor, width: int, name: str) -> int:
    """Row stride (elements) of a [B, T, width]-shaped view with unit inner stride.

    The batch stride must equal T * row stride (the C ABI convention)."""
    if t.dim() != 3:
        raise ValueError(f"{name}: expected 3 dims [B, T, {width}], got {tuple(t.shape)}")
    B, T, W = t.shape
    if W != width or t.stride(2) != 1:
        raise ValueError(f"{name}: inner dim must be {width} contiguous elements")
    rs = t.stride(1)
    if B > 1 and t.stride(0) != T * rs:
        raise ValueError(f"{name}: batch stride must equal T * row stride")
    return rs


def _flat_heads(t: torch.Tensor, name: str) -> torch.Tensor:
    """View [B, T, H, d] (inner two dims contiguous) as [B, T, H*d]."""
    if t.dim() == 3:
        return t
    if t.dim() != 4:
        raise ValueError(f"{name}: expected [B, T, H, d] or [B, T, H*d]")
    B, T, H, d = t.shape
    if t.stride(3) != 1 or t.stride(2) != d:
        t = t.contiguous()
    return t.as_strided((B, T, H * d), (t.stride(0), t.stride(1), 1))


def bitmask_words(tkv: int) -> int:
    return int(_lib.load().gsa_bitmask_words(int(tkv)))


def indexer_topk_workspace_size(B: int, Tq: int, Tkv: int) -> int:
    """Bytes of scratch ``indexer_topk`` needs (the fp32 score rows)."""
    return int(_lib.load().gsa_indexer_topk_workspace_size(int(B), int(Tq), int(Tkv)))


# --------------------------------------------------------------------------- RoPE + G2
def rope_gates(q_src: torch.Tensor, k_src: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
               num_heads: int, v_src: torch.Tensor | None = None,
               vg_src: torch.Tensor | None = None, out: tuple | None = None):
    """RoPE on q/k and (optionally) v * sigmoid(vg); all sources [B, T, H*d] with one row stride.

    Returns (q, k, v) as contiguous [B, T, H*d] tensors (v is None without v_src); ``out``
    = (q, k, v) supplies them (contiguous, the sources' shape and dtype)."""
    _cuda(q_src, k_src, cos, sin, v_src, vg_src)
    B, T, W = q_src.shape
    d = W // num_heads
    code = _dtype_code(q_src)
    rs = _rows(q_src, W, "q_src")
    for name, t in (("k_src", k_src), ("v_src", v_src), ("vg_src", vg_src)):
        if t is not None:
            if t.shape != q_src.shape or t.dtype != q_src.dtype or _rows(t, W, name) != rs:
                raise ValueError(f"{name} must match q_src in shape, dtype and row stride")
    if cos.shape != (T, d) or sin.shape != (T, d):
        raise ValueError(f"cos/sin must be [T, d] = [{T}, {d}]")
    cos = cos.to(q_src.dtype).contiguous()
    sin = sin.to(q_src.dtype).contiguous()
    if out is None:
        q = torch.empty(B, T, W, device=q_src.device, dtype=q_src.dtype)
        k = torch.empty_like(q)
        v = torch.empty_like(q) if v_src is not None else None
    else:
        q, k, v = out
        for t in (q, k) + ((v,) if v_src is not None else ()):
            if (t is None or t.shape != (B, T, W) or t.dtype != q_src.dtype
                    or not t.is_contiguous() or t.device != q_src.device):
                raise ValueError(f"out tensors must be contiguous [{B}, {T}, {W}] "
                                 f"{q_src.dtype} on the sources' device")
        if v_src is None:
            v = None
    rc = _lib.load().gsa_rope_gates(
        q_src.data_ptr(), k_src.data_ptr(),
        v_src.data_ptr() if v_src is not None else None,
        vg_src.data_ptr() if vg_src is not None else None,
        rs, code, B, T, num_heads, d, cos.data_ptr(), sin.data_ptr(),
        q.data_ptr(), k.data_ptr(), v.data_ptr() if v is not None else None, _stream())
    _lib.check(rc, "gsa_rope_gates")
    return q, k, v


def fused_projection_rows(hidden: int, n_idx_heads: int, d_indexer: int) -> int:
    """Rows of the packed weight ``fused_projection`` takes (0: unsupported sizes)."""
    return int(_lib.load().gsa_fused_projection_rows(hidden, n_idx_heads, d_indexer))


def fused_projection_rest_width(hidden: int, n_idx_heads: int, d_indexer: int) -> int:
    """Row width of the ``rest`` output (og | iq | ik | iw, padded to 64 columns)."""
    return int(_lib.load().gsa_fused_projection_rest_width(hidden, n_idx_heads, d_indexer))


def fused_projection_pack(weights: dict, n_idx_heads: int, d_indexer: int):
    """Packed (weight [rows, D] bf16, bias [rows] fp32) for ``fused_projection``.

    ``weights`` maps q, k, v, vg, og, iq, ik, iw to the nn.Linear weights and
    vg_bias, og_bias, iw_bias to the biases (bf16, on one device)."""
    w = {n: weights[n].detach().contiguous() for n in ("q", "k", "v", "vg", "og", "iq", "ik", "iw")}
    b = {n: weights[n].detach().float().contiguous() for n in ("vg_bias", "og_bias", "iw_bias")}
    _cuda(*w.values(), *b.values())
    D = w["q"].shape[1]
    if any(t.dtype != torch.bfloat16 for t in w.values()):
        raise ValueError("fused_projection_pack takes bf16 weights")
    rows = fused_projection_rows(D, n_idx_heads, d_indexer)
    if rows == 0:
        raise ValueError(f"unsupported sizes for the fused projection: D={D}")
    wp = torch.empty(rows, D, device=w["q"].device, dtype=torch.bfloat16)
    bp = torch.empty(rows, device=w["q"].device, dtype=torch.float32)
    rc = _lib.load().gsa_fused_projection_pack(
        *(w[n].data_ptr() for n in ("q", "k", "v", "vg", "og", "iq", "ik", "iw")),
        *(b[n].data_ptr() for n in ("vg_bias", "og_bias", "iw_bias")),
        D, n_idx_heads, d_indexer, wp.data_ptr(), bp.data_ptr(), _stream())
    _lib.check(rc, "gsa_fused_projection_pack")
    return wp, bp


def fused_projection(x: torch.Tensor, w_packed: torch.Tensor, b_packed: torch.Tensor,
                     num_heads: int, n_idx_heads: int, d_indexer: int, cos: torch.Tensor,
                     sin: torch.Tensor, pos0: int = 0, seq_len: int | None = None,
                     out: tuple | None = None):
    """Projection GEMM with RoPE and the value gate in its epilogue (bf16).

    x [B, T, D] (unit inner stride); cos / sin [rows, 128] bf16 tables; row t of
    a sequence takes table row pos0 + t (``seq_len`` = rows per sequence,
    default T).  Returns (q, k, v, rest): q, k, v [B, T, D] contiguous (RoPE'd,
    gated) and rest [B, T, rest width] = og | iq | ik | iw | padding.  ``out``
    = (q, k, v, rest) supplies them."""
    _cuda(x, w_packed, b_packed, cos, sin)
    B, T, D = x.shape
    M = B * T
    if x.dtype != torch.bfloat16 or w_packed.dtype != torch.bfloat16:
        raise ValueError("fused_projection is bf16")
    xs = _rows(x, D, "x")
    if B > 1 and x.stride(0) != T * xs:
        raise ValueError("x must have uniform row strides across the batch")
    rw = fused_projection_rest_width(D, n_idx_heads, d_indexer)
    if out is None:
        q = torch.empty(B, T, D, device=x.device, dtype=x.dtype)
        k, v = torch.empty_like(q), torch.empty_like(q)
        rest = torch.empty(B, T, rw, device=x.device, dtype=x.dtype)
    else:
        q, k, v, rest = out
    cos = cos.to(torch.bfloat16).contiguous()
    sin = sin.to(torch.bfloat16).contiguous()
    rc = _lib.load().gsa_fused_projection(
        x.data_ptr(), xs, w_packed.data_ptr(), b_packed.data_ptr(), M, D, num_heads,
        D // num_heads, n_idx_heads, d_indexer, T if seq_len is None else seq_len, pos0,
        cos.data_ptr(), sin.data_ptr(), cos.shape[0], q.data_ptr(), k.data_ptr(), v.data_ptr(),
        rest.data_ptr(), rest.stride(-2), _stream())
    _lib.check(rc, "gsa_fused_projection")
    return q, k, v, rest


def apply_rotary_pos_emb(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """Reference-compatible RoPE: q, k [B, T, H, d]; cos, sin broadcastable to [1, T, 1, d]."""
    B, T, H, d = q.shape
    cos2 = cos.reshape(-1, d)[-T:] if cos.dim() != 2 else cos
    sin2 = sin.reshape(-1, d)[-T:] if sin.dim() != 2 else sin
    qe, ke, _ = rope_gates(_flat_heads(q, "q"), _flat_heads(k, "k"), cos2, sin2, H)
    return qe.view(B, T, H, d), ke.view(B, T, H, d)


# --------------------------------------------------------------------------- indexer
def indexer_scores(q_idx: torch.Tensor, k_idx: torch.Tensor, w: torch.Tensor, bias: torch.Tensor,
                   scale: float, q_pos0: int = 0, tkv: int | None = None,
                   fill_upper: bool = True, out: torch.Tensor | None = None) -> torch.Tensor:
    """Gated indexer scores [B, Tq, Tkv] fp32 (row stride padded to a multiple of 4).

    q_idx [B, Tq, H_I, d_I] (or [B, Tq, H_I*d_I]), k_idx [B, Tkv, d_I], w [B, Tq, H_I];
    query row r sits at sequence position q_pos0 + r."""
    _cuda(q_idx, k_idx, w, bias)
    if q_idx.dim() == 4:
        B, Tq, H_I, d_I = q_idx.shape
        if q_idx.stride(3) != 1 or q_idx.stride(2) != d_I:
            q_idx = q_idx.contiguous()
        q3 = q_idx.as_strided((B, Tq, H_I * d_I), (q_idx.stride(0), q_idx.stride(1), 1))
    else:
        raise ValueError("q_idx must be [B, Tq, H_I, d_I]")
    Tkv = k_idx.shape[1] if tkv is None else tkv
    d_code = _dtype_code(q_idx)
    if k_idx.dtype != q_idx.dtype or w.dtype != q_idx.dtype:
        raise ValueError("q_idx, k_idx and w must share a dtype")
    qs = _rows(q3, H_I * d_I, "q_idx")
    ks = _rows(k_idx, d_I, "k_idx")
    ws = _rows(w, H_I, "w")
    bias32 = bias.detach().to(torch.float32).contiguous()
    stride = (Tkv + 3) // 4 * 4
    if out is None:
        out = torch.empty(B, Tq, stride, device=q_idx.device, dtype=torch.float32)
    rc = _lib.load().gsa_indexer_scores(
        q3.data_ptr(), qs, k_idx.data_ptr(), ks, w.data_ptr(), ws, bias32.data_ptr(),
        float(scale), d_code, B, Tq, Tkv, int(q_pos0), H_I, d_I, out.data_ptr(), out.stride(1),
        1 if fill_upper else 0, _stream())
    _lib.check(rc, "gsa_indexer_scores")
    return out[:, :, :Tkv]


def fused_gated_indexer(q_idx, k_idx, w, bias, scale: float, causal: bool = True) -> torch.Tensor:
    """Drop-in for gsa_opt.fused_gated_indexer: [B, T, T] fp32 with -inf above the diagonal.

    causal=False places every query past the last key, so each row sees all keys."""
    B, T = q_idx.shape[0], q_idx.shape[1]
    Tkv = k_idx.shape[1]
    s = indexer_scores(q_idx, k_idx, w, bias, scale, q_pos0=0 if causal else Tkv, tkv=Tkv,
                       fill_upper=True)
    return s.contiguous() if s.stride(1) != Tkv else s


def _indexer_inputs(q_idx, k_idx, w, bias):
    """Checked [B, Tq, H_I*d_I] view of q_idx, row strides, fp32 bias and dtype code."""
    _cuda(q_idx, k_idx, w, bias)
    B, Tq, H_I, d_I = q_idx.shape
    if q_idx.stride(3) != 1 or q_idx.stride(2) != d_I:
        q_idx = q_idx.contiguous()
    q3 = q_idx.as_strided((B, Tq, H_I * d_I), (q_idx.stride(0), q_idx.stride(1), 1))
    code = _dtype_code(q_idx)
    if k_idx.dtype != q_idx.dtype or w.dtype != q_idx.dtype:
        raise ValueError("q_idx, k_idx and w must share a dtype")
    qs, ks, ws = _rows(q3, H_I * d_I, "q_idx"), _rows(k_idx, d_I, "k_idx"), _rows(w, H_I, "w")
    bias32 = bias.detach().to(torch.float32).contiguous()
    return q3, qs, ks, ws, bias32, code, (B, Tq, H_I, d_I)


def _selection_outputs(dev, B: int, Tq: int, width: int, Tkv: int, want_indices: bool,
                       want_mask: bool, want_bitmask: bool, bitmask_out=None):
    idx = torch.empty(B, Tq, width, device=dev, dtype=torch.int32) if want_indices else None
    msk = torch.empty(B, Tq, width, device=dev, dtype=torch.uint8) if want_mask else None
    W = bitmask_words(Tkv)
    bm = None
    if want_bitmask:
        if bitmask_out is not None:
            if (bitmask_out.shape != (B, Tq, W) or bitmask_out.dtype != torch.int32
                    or not bitmask_out.is_contiguous() or bitmask_out.device != dev):
                raise ValueError(f"bitmask_out must be a contiguous int32 [{B}, {Tq}, {W}] "
                                 "tensor on the inputs' device")
            bm = bitmask_out
        else:
            bm = torch.empty(B, Tq, W, device=dev, dtype=torch.int32)
    return idx, msk, bm, W


def _ptr(t):
    return t.data_ptr() if t is not None else None


def _workspace(workspace, need: int, dev):
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    return workspace


def indexer_topk(q_idx: torch.Tensor, k_idx: torch.Tensor, w: torch.Tensor, bias: torch.Tensor,
                 scale: float, k_sel: int, q_pos0: int = 0, tkv: int | None = None,
                 want_indices: bool = False, want_mask: bool = False, want_bitmask: bool = True,
                 workspace: torch.Tensor | None = None, bitmask_out: torch.Tensor | None = None):
    """Indexer + top-k in one C call; the scores live only in a scratch workspace.

    Same inputs as ``indexer_scores``; outputs as ``topk_select``
    (indices int32, mask bool, bitmask int32 words), unrequested ones None.
    ``bitmask_out`` (int32 [B, Tq, bitmask_words(Tkv)], contiguous) receives the
    bitmask instead of a new tensor."""
    q3, qs, ks, ws, bias32, code, (B, Tq, H_I, d_I) = _indexer_inputs(q_idx, k_idx, w, bias)
    Tkv = k_idx.shape[1] if tkv is None else tkv
    lib = _lib.load()
    workspace = _workspace(workspace, int(lib.gsa_indexer_topk_workspace_size(B, Tq, Tkv)),
                           q_idx.device)
    idx, msk, bm, W = _selection_outputs(q_idx.device, B, Tq, k_sel, Tkv, want_indices,
                                         want_mask, want_bitmask, bitmask_out)
    rc = lib.gsa_indexer_topk(
        q3.data_ptr(), qs, k_idx.data_ptr(), ks, w.data_ptr(), ws, bias32.data_ptr(), float(scale),
        code, B, Tq, Tkv, int(q_pos0), H_I, d_I, int(k_sel), workspace.data_ptr(),
        workspace.numel() * workspace.element_size(), _ptr(idx), _ptr(msk), _ptr(bm), W,
        _stream())
    _lib.check(rc, "gsa_indexer_topk")
    return idx, (msk.bool() if msk is not None else None), bm


# --------------------------------------------------------------------------- adaptive k
def adaptive_k_width(k_max: int, tkv: int) -> int:
    """Slots per row of adaptive-mode index / mask outputs: min(k_max, Tkv)."""
    return int(_lib.load().gsa_adaptive_k_width(int(k_max), int(tkv)))


def indexer_topk_adaptive_workspace_size(B: int, Tq: int, Tkv: int) -> int:
    return int(_lib.load().gsa_indexer_topk_adaptive_workspace_size(int(B), int(Tq), int(Tkv)))


def adaptive_workspace_views(workspace: torch.Tensor, B: int, Tq: int, Tkv: int):
    """(scores [B, Tq, stride] fp32, row_var [B, Tq] fp32, var_sum [1] fp64) inside a
    uint8 workspace of ``indexer_topk_adaptive_workspace_size`` bytes, laid out as
    the C call lays it out."""
    stride = (Tkv + 3) // 4 * 4
    n_scores = B * Tq * stride * 4
    sum_off = (n_scores + B * Tq * 4 + 15) // 16 * 16
    scores = workspace[:n_scores].view(torch.float32).view(B, Tq, stride)
    row_var = workspace[n_scores:n_scores + B * Tq * 4].view(torch.float32).view(B, Tq)
    var_sum = workspace[sum_off:sum_off + 8].view(torch.float64)
    return scores, row_var, var_sum


def indexer_topk_adaptive(q_idx: torch.Tensor, k_idx: torch.Tensor, w: torch.Tensor,
                          bias: torch.Tensor, scale: float, k_base: int, k_min: int, k_max: int,
                          q_pos0: int = 0, tkv: int | None = None, want_indices: bool = False,
                          want_mask: bool = False, want_bitmask: bool = True,
                          workspace: torch.Tensor | None = None,
                          bitmask_out: torch.Tensor | None = None):
    """``indexer_topk`` with the per-row adaptive k, averaged over the call's rows.

    Returns (indices [B,Tq,adaptive_k_width], mask, bitmask, row_k int32 [B,Tq])."""
    q3, qs, ks, ws, bias32, code, (B, Tq, H_I, d_I) = _indexer_inputs(q_idx, k_idx, w, bias)
    Tkv = k_idx.shape[1] if tkv is None else tkv
    lib = _lib.load()
    workspace = _workspace(workspace, indexer_topk_adaptive_workspace_size(B, Tq, Tkv),
                           q_idx.device)
    width = adaptive_k_width(k_max, Tkv)
    idx, msk, bm, W = _selection_outputs(q_idx.device, B, Tq, width, Tkv, want_indices,
                                         want_mask, want_bitmask, bitmask_out)
    row_k = torch.empty(B, Tq, device=q_idx.device, dtype=torch.int32)
    rc = lib.gsa_indexer_topk_adaptive(
        q3.data_ptr(), qs, k_idx.data_ptr(), ks, w.data_ptr(), ws, bias32.data_ptr(), float(scale),
        code, B, Tq, Tkv, int(q_pos0), H_I, d_I, int(k_base), int(k_min), int(k_max),
        workspace.data_ptr(), workspace.numel() * workspace.element_size(), row_k.data_ptr(),
        _ptr(idx), _ptr(msk), _ptr(bm), W, _stream())
    _lib.check(rc, "gsa_indexer_topk_adaptive")
    return idx, (msk.bool() if msk is not None else None), bm, row_k


def _check_scores(scores: torch.Tensor):
    _cuda(scores)
    if scores.dtype != torch.float32 or scores.dim() != 3 or scores.stride(2) != 1:
        raise ValueError("scores must be float32 [B, Tq, Tkv] with unit inner stride")
    B, Tq, Tkv = scores.shape
    if B > 1 and scores.stride(0) != Tq * scores.stride(1):
        raise ValueError("scores batch stride must equal Tq * row stride")
    return B, Tq, Tkv


def row_variance(scores: torch.Tensor, q_pos0: int = 0, out=None):
    """Per-row variance of the valid (!= -inf) causal scores and its sum over the rows.

    Returns (row_var fp32 [B, Tq], var_sum fp64 [1]); ``out`` may supply that pair."""
    B, Tq, Tkv = _check_scores(scores)
    if out is None:
        row_var = torch.empty(B, Tq, device=scores.device, dtype=torch.float32)
        var_sum = torch.empty(1, device=scores.device, dtype=torch.float64)
    else:
        row_var, var_sum = out
    rc = _lib.load().gsa_row_variance(scores.data_ptr(), scores.stride(1), B, Tq, Tkv,
                                      int(q_pos0), row_var.data_ptr(), var_sum.data_ptr(),
                                      _stream())
    _lib.check(rc, "gsa_row_variance")
    return row_var, var_sum


def topk_select_adaptive(scores: torch.Tensor, k_base: int, k_min: int, k_max: int,
                         row_var: torch.Tensor, var_sum: torch.Tensor, var_rows: int,
                         q_pos0: int = 0, want_indices: bool = True, want_mask: bool = True,
                         want_bitmask: bool = True, bitmask_out: torch.Tensor | None = None):
    """Top-k with k per row from the row variances (``row_variance``); ``var_sum`` /
    ``var_rows`` give the batch mean of the variances (summed over every row block
    and rank of the batch).  Returns (indices, mask, bitmask, row_k int32 [B, Tq])."""
    B, Tq, Tkv = _check_scores(scores)
    _cuda(row_var, var_sum)
    if row_var.dtype != torch.float32 or row_var.numel() != B * Tq or not row_var.is_contiguous():
        raise ValueError("row_var must be a contiguous float32 tensor of B*Tq elements")
    if var_sum.dtype != torch.float64 or var_sum.numel() != 1:
        raise ValueError("var_sum must be a one-element float64 tensor")
    width = adaptive_k_width(k_max, Tkv)
    idx, msk, bm, W = _selection_outputs(scores.device, B, Tq, width, Tkv, want_indices,
                                         want_mask, want_bitmask, bitmask_out)
    row_k = torch.empty(B, Tq, device=scores.device, dtype=torch.int32)
    rc = _lib.load().gsa_topk_select_adaptive(
        scores.data_ptr(), scores.stride(1), B, Tq, Tkv, int(q_pos0), int(k_base), int(k_min),
        int(k_max), row_var.data_ptr(), var_sum.data_ptr(), int(var_rows), row_k.data_ptr(),
        _ptr(idx), _ptr(msk), _ptr(bm), W, _stream())
    _lib.check(rc, "gsa_topk_select_adaptive")
    return idx, (msk.bool() if msk is not None else None), bm, row_k


# --------------------------------------------------------------------------- top-k
def topk_select(scores: torch.Tensor, k_sel: int, q_pos0: int = 0, want_indices: bool = True,
                want_mask: bool = True, want_bitmask: bool = True,
                bitmask_out: torch.Tensor | None = None):
    """Top-k over causal rows of ``scores`` [B, Tq, Tkv] (fp32, unit inner stride).

    Returns (indices int32 [B,Tq,k] ascending + masked filler, mask bool [B,Tq,k],
    bitmask int32-storage uint32 words [B,Tq,W]); unrequested outputs are None."""
    B, Tq, Tkv = _check_scores(scores)
    idx, msk, bm, W = _selection_outputs(scores.device, B, Tq, k_sel, Tkv, want_indices,
                                         want_mask, want_bitmask, bitmask_out)
    rc = _lib.load().gsa_topk_select(
        scores.data_ptr(), scores.stride(1), B, Tq, Tkv, int(q_pos0), int(k_sel),
        _ptr(idx), _ptr(msk), _ptr(bm), W, _stream())
    _lib.check(rc, "gsa_topk_select")
    return idx, (msk.bool() if msk is not None else None), bm


# --------------------------------------------------------------------------- attention
def masked_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, bitmask: torch.Tensor,
                     scale: float, num_heads: int, og: torch.Tensor | None = None,
                     q_pos0: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """Tensor-core sparse attention over a selection bitmask (bf16, d = 128).

    q [B, Tq, H*d], k/v [B, Tkv, H*d], bitmask [B, Tq, W] from ``topk_select``;
    og (optional) output-gate logits [B, Tq, H*d] fused as o * sigmoid(og)."""
    q, k, v = _flat_heads(q, "q"), _flat_heads(k, "k"), _flat_heads(v, "v")
    _cuda(q, k, v, bitmask, og)
    B, Tq, W = q.shape
    Tkv = k.shape[1]
    d = W // num_heads
    for t in (q, k, v):
        if t.dtype != torch.bfloat16:
            raise RuntimeError("masked_attention runs in bfloat16")
    qs, ks, vs = _rows(q, W, "q"), _rows(k, W, "k"), _rows(v, W, "v")
    if bitmask.dim() != 3 or bitmask.stride(2) != 1 or bitmask.shape[:2] != (B, Tq):
        raise ValueError("bitmask must be [B, Tq, W] with unit inner stride")
    ogs = _rows(og, W, "og") if og is not None else 0
    if out is None:
        out = torch.empty(B, Tq, W, device=q.device, dtype=q.dtype)
    os_ = _rows(out, W, "out")
    rc = _lib.load().gsa_masked_attention(
        q.data_ptr(), qs, k.data_ptr(), ks, v.data_ptr(), vs, bitmask.data_ptr(),
        bitmask.stride(1), og.data_ptr() if og is not None else None, ogs, out.data_ptr(), os_,
        float(scale), B, Tq, Tkv, int(q_pos0), num_heads, d, _stream())
    _lib.check(rc, "gsa_masked_attention")
    return out


def gather_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor,
                     mask: torch.Tensor | None, scale: float) -> torch.Tensor:
    """Index-gather sparse attention; q [B,Tq,H,d], k/v [B,Tkv,H,d], indices [B,Tq,k]."""
    _cuda(q, k, v, indices, mask)
    B, Tq, H, d = q.shape
    Tkv = k.shape[1]
    code = _dtype_code(q)
    q3, k3, v3 = _flat_heads(q, "q"), _flat_heads(k, "k"), _flat_heads(v, "v")
    W = H * d
    qs, ks, vs = _rows(q3, W, "q"), _rows(k3, W, "k"), _rows(v3, W, "v")
    idx = indices.to(torch.int32).contiguous()
    k_sel = idx.shape[-1]
    m = mask.to(torch.uint8).contiguous() if mask is not None else None
    out = torch.empty(B, Tq, H, d, device=q.device, dtype=q.dtype)
    rc = _lib.load().gsa_gather_attention(
        q3.data_ptr(), qs, k3.data_ptr(), ks, v3.data_ptr(), vs, idx.data_ptr(),
        m.data_ptr() if m is not None else None, k_sel, out.data_ptr(), W, float(scale), code,
        B, Tq, Tkv, H, d, _stream())
    _lib.check(rc, "gsa_gather_attention")
    return out


def fused_sparse_attention(q, k, v, indices, mask, scale: float) -> torch.Tensor:
    """Drop-in for gsa_opt.fused_sparse_attention: [B, T, H, d] in q's dtype."""
    return gather_attention(q, k, v, indices, mask, scale)


def sparse_attention_ref(q, k, v, indices, mask, scale: float) -> torch.Tensor:
    """Drop-in for gsa_ref.sparse_attention_ref (gsa_ref.py:202-238), same arguments:
    q [B, T, H, d], k / v [B, T_kv, H, d], indices / mask [B, T, k_sel].  Runs the
    index-gather kernel; a row whose mask is all False comes out as zeros, as the
    reference's nan_to_num makes it."""
    return gather_attention(q, k, v, indices, mask, scale)


def output_gate(o: torch.Tensor, og: torch.Tensor) -> torch.Tensor:
    """o * sigmoid(og) element-wise (each op rounded to o's dtype); o, og [B, T, W]."""
    _cuda(o, og)
    if o.dim() == 4:
        o = _flat_heads(o, "o")
    B, T, W = o.shape
    og = og.reshape(B, T, W)
    code = _dtype_code(o)
    o_s, g_s = _rows(o, W, "o"), _rows(og, W, "og")
    out = torch.empty(B, T, W, device=o.device, dtype=o.dtype)
    rows = B * T
    rc = _lib.load().gsa_output_gate(o.data_ptr(), o_s, og.data_ptr(), g_s, out.data_ptr(), W,
                                     code, rows, W, _stream())
    _lib.check(rc, "gsa_output_gate")
    return out
