"""The projection GEMM with RoPE and the value gate in its epilogue
(gsa_fused_projection, proj_gemm.cu) against the unfused path it replaces:
cuBLAS addmm over the concatenated weights (gsa_opt.py:582-609) followed by
gsa_rope_gates, which matches torch's RoPE / gate rounding bit for bit
(test_gpu_kernels.py).

The two GEMMs accumulate in different orders, so a projection value can round
to a neighbouring bf16 value; the tests therefore bound the difference by a
few bf16 steps of the tensor's largest magnitude and require almost every
element (>= 98%) to be identical.  A layout error (wrong tile, head, partner
channel, gate column or bias) changes most elements and fails both."""
import pytest
import torch

from gsa_gdn_benchmarkstudy_b200 import ops
from gsa_gdn_benchmarkstudy_b200.gsa import GatedSparseAttention

pytestmark = pytest.mark.gpu
torch.set_grad_enabled(False)


def _module(D, H, seed):
    torch.manual_seed(seed)
    m = GatedSparseAttention(D, H).cuda().to(torch.bfloat16)
    for b in (m.value_gate.gate_proj.bias, m.output_gate.gate_proj.bias,
              m.indexer.idx_w_proj.bias):
        b.normal_(0.0, 0.5)  # non-zero biases, so a misplaced bias shows
    return m


def _unfused(m, x, cos, sin):
    parts = m.split(m.project(x))
    q, k, v = ops.rope_gates(parts["q"], parts["k"], cos, sin, m.num_heads,
                             v_src=parts["v"], vg_src=parts["vg"])
    return {"q": q, "k": k, "v": v, "og": parts["og"], "iq": parts["iq"], "ik": parts["ik"],
            "iw": parts["iw"]}


def _compare(got: dict, ref: dict):
    for name in ref:
        a, b = got[name].float(), ref[name].float()
        assert a.shape == b.shape, name
        assert torch.isfinite(a).all(), name
        scale = b.abs().max().item()
        err = (a - b).abs().max().item()
        assert err <= 2 ** -6 * scale, (name, err, scale)
        same = (got[name] == ref[name]).float().mean().item()
        assert same >= 0.98, (name, same)


@pytest.mark.parametrize("D,H,B,T", [(512, 4, 2, 300), (2048, 16, 1, 512), (512, 4, 1, 77)])
def test_fused_projection_matches_addmm_then_rope_gates(D, H, B, T):
    """Row tails (600 = 2*256 + 88 rows, 77 rows: one partial tile), batch
    entries sharing the rotary rows, and the full hidden size of the
    benchmarks (42 column tiles, a rest tile with two of four boxes stored)."""
    m = _module(D, H, seed=D + T)
    x = (torch.randn(B, T, D, device="cuda") * 0.8).bfloat16()
    cos, sin = m.rotary_emb(T, x.device, x.dtype)
    q, k, v, parts = m.project_fused(x, cos, sin)
    _compare({"q": q, "k": k, "v": v, **parts}, _unfused(m, x, cos, sin))


def test_fused_projection_block_positions():
    """A block of rows at positions pos0..pos0+n-1 (the row-block and sharded
    paths), written into views of larger buffers: rows outside the block stay
    as they were."""
    D, H, T, r0, r1 = 512, 4, 1200, 333, 1100
    m = _module(D, H, seed=5)
    x = (torch.randn(1, T, D, device="cuda") * 0.8).bfloat16()
    cos, sin = m.rotary_emb(T, x.device, x.dtype)
    rw = ops.fused_projection_rest_width(D, 4, 64)
    bufs = [torch.full((1, T, D), 3.0, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    rest = torch.full((1, T, rw), 3.0, device="cuda", dtype=torch.bfloat16)
    q, k, v, parts = m.project_fused(x[:, r0:r1], cos, sin, pos0=r0, seq_len=r1 - r0,
                                     out=tuple(t[:, r0:r1] for t in bufs) + (rest[:, r0:r1],))
    ref = _unfused(m, x[:, r0:r1], cos[r0:r1], sin[r0:r1])
    _compare({"q": q, "k": k, "v": v, **parts}, ref)
    for t in bufs + [rest]:
        assert (t[:, :r0] == 3.0).all() and (t[:, r1:] == 3.0).all()
    # padding columns of the rest rows past iw are not part of the contract,
    # but the columns it names are all written
    assert not (rest[:, r0:r1, :D + 256 + 64 + 4] == 3.0).all(dim=-1).any()


def test_fused_projection_pack_layout():
    """The packed weight rows are the module's weights in the documented tile
    order, copied bit for bit."""
    D, H = 512, 4
    m = _module(D, H, seed=9)
    wp, bp = m._get_packed()
    ix = m.indexer
    assert wp.shape == (ops.fused_projection_rows(D, 4, 64), D)
    assert torch.equal(wp[:D], m.q_proj.weight)
    assert torch.equal(wp[D:2 * D], m.k_proj.weight)
    for i in range(D // 128):
        t0 = 2 * D + 256 * i
        assert torch.equal(wp[t0:t0 + 128], m.v_proj.weight[128 * i:128 * i + 128])
        assert torch.equal(wp[t0 + 128:t0 + 256],
                           m.value_gate.gate_proj.weight[128 * i:128 * i + 128])
        assert torch.equal(bp[t0 + 128:t0 + 256],
                           m.value_gate.gate_proj.bias[128 * i:128 * i + 128].float())
        assert (bp[t0:t0 + 128] == 0).all()
    r = 4 * D
    rest_w = torch.cat([m.output_gate.gate_proj.weight, ix.idx_q_proj.weight,
                        ix.idx_k_proj.weight, ix.idx_w_proj.weight])
    assert torch.equal(wp[r:r + rest_w.shape[0]], rest_w)
    assert (wp[r + rest_w.shape[0]:] == 0).all()
    assert torch.equal(bp[r:r + D], m.output_gate.gate_proj.bias.float())
    o_iw = r + D + 256 + 64
    assert torch.equal(bp[o_iw:o_iw + 4], ix.idx_w_proj.bias.float())
    assert (bp[:2 * D] == 0).all() and (bp[r + D:o_iw] == 0).all() and (bp[o_iw + 4:] == 0).all()


def test_forward_same_with_and_without_the_fused_epilogue():
    """The module forward through the fused projection against the cuBLAS +
    separate RoPE path (cfg1-sized, 2048 rows)."""
    m = _module(1024, 8, seed=3)
    x = (torch.randn(1, 2048, 1024, device="cuda") * 0.8).bfloat16()
    assert m.fused_epilogue_ok(x.dtype)
    y_fused = m(x)
    m.use_fused_epilogue = False
    y_ref = m(x)
    d = (y_fused.float() - y_ref.float()).abs()
    scale = y_ref.float().abs().max().item()
    assert d.max().item() <= 2 ** -5 * scale, (d.max().item(), scale)
    assert d.mean().item() <= 2 ** -10 * scale
