"""Generate the golden fixtures in this folder by running the REFERENCE itself.

Run here, where the reference checkout is present:

    python tests/golden/make_golden.py --reference /path/to/GSA_GDN_BenchmarkStudy

It imports ``gsa_triton/gsa_ref.py`` from that checkout (read only), builds
``GatedSparseAttention`` with the seeded benchmark weights
(``gsa_gdn_benchmarkstudy_b200.workloads.init_weights_``), runs it on the seeded
inputs and stores, per configuration, the outputs and the intermediates of
its own stages (scores, top-k indices/mask, RoPE'd q/k, gated v, attention).
Stages are invoked exactly in the order of gsa_ref.py:276-325 and the final
result is asserted equal to ``model(x)``.

For cfg2 (T=4096, D=2048) the whole reference forward would materialise the
[B, T, k, H, d] gather (2 x 34 GB in bf16), so the fixture runs the
reference's full-sequence stages (projections, RoPE, indexer, top-k) and calls
``sparse_attention_ref`` on a sample of query rows only.
"""
from __future__ import annotations

import argparse
import hashlib
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from gsa_gdn_benchmarkstudy_b200.workloads import (  # noqa: E402
    CONFIGS, TEST_CONFIGS, GSAConfig, init_weights_, make_input)


def x_digest(x: torch.Tensor) -> str:
    return hashlib.sha256(x.float().contiguous().numpy().tobytes()).hexdigest()


def build(ref, cfg: GSAConfig):
    torch.manual_seed(1234)
    m = ref.GatedSparseAttention(**cfg.module_kwargs())
    init_weights_(m, seed=1)
    return m.to(cfg.torch_dtype).eval()


def stages(ref, m, x, rows=None):
    """The reference forward (gsa_ref.py:276-325) with its intermediates."""
    B, T, D = x.shape
    H, dh = m.num_heads, m.d_head
    q = m.q_proj(x).view(B, T, H, dh)
    k = m.k_proj(x).view(B, T, H, dh)
    v = m.v_proj(x).view(B, T, H, dh)
    v = m.value_gate(v, x)
    cos, sin = m.rotary_emb(T, x.device, x.dtype)
    q, k = ref.apply_rotary_pos_emb(q, k, cos.unsqueeze(0).unsqueeze(2), sin.unsqueeze(0).unsqueeze(2))
    scores = m.indexer(x)
    idx, mask, k_eff = m.topk_selector(scores)
    if rows is None:
        attn = ref.sparse_attention_ref(q, k, v, idx, mask, m.scale)
        attn = m.output_gate(attn, x)
        out = m.o_proj(attn.reshape(B, T, D))
    else:
        r = torch.as_tensor(rows)
        attn = ref.sparse_attention_ref(q[:, r], k, v, idx[:, r], mask[:, r], m.scale)
        og = m.output_gate.gate_proj(x[:, r])
        attn = attn * torch.sigmoid(og).view(B, len(rows), H, dh)
        out = m.o_proj(attn.reshape(B, len(rows), D))
    return dict(q=q, k=k, v=v, scores=scores, idx=idx, mask=mask, attn=attn, out=out, k_eff=k_eff)


def notebook_adaptive_k(reference: Path, scores: torch.Tensor, k_base: int, k_min: int,
                        k_max: int):
    """Runs the adaptive-k cell of the reference's notebook (gsa_explained.ipynb:575-592)
    on ``scores`` with its k_base / k_min / k_max set to the given values.

    The cell's own source is executed; only its three parameter assignments are
    replaced and its printing is discarded.  Returns (k_adaptive, variance)."""
    import contextlib
    import io
    import json
    import re
    nb = json.loads((reference / "gsa_explained.ipynb").read_text())
    cells = ["".join(c["source"]) for c in nb["cells"] if c["cell_type"] == "code"]
    src = next(c for c in cells if "k_adaptive = (k_base" in c)
    for name, val in (("k_base", k_base), ("k_min", k_min), ("k_max", k_max)):
        src, n = re.subn(rf"^{name} = \d+", f"{name} = {val}", src, count=1, flags=re.M)
        assert n == 1, name
    ns = {"torch": torch, "final_scores": scores, "T": scores.shape[1]}
    with contextlib.redirect_stdout(io.StringIO()):
        exec(compile(src, "gsa_explained.ipynb[adaptive-k cell]", "exec"), ns)
    return ns["k_adaptive"], ns["variance"]


def adaptive_edge_scores() -> torch.Tensor:
    """Seeded causal scores with the cases adaptive k must handle: a constant
    row (variance 0 -> the 1e-6 clamp), exact ties, rows with few valid
    scores and scattered -inf entries below the diagonal."""
    g = torch.Generator().manual_seed(7)
    B, T = 2, 96
    s = torch.randn(B, T, T, generator=g) * 2.0
    s[0, 40] = 0.25                                  # constant row
    s[1, 50, :30] = s[1, 50, 0]                      # tied block
    s[1, 60] = torch.round(s[1, 60] * 2) / 2         # many exact ties
    drop = torch.rand(B, T, T, generator=g) < 0.1
    s = s.masked_fill(drop, float("-inf"))           # scattered -inf
    causal = torch.triu(torch.ones(T, T, dtype=torch.bool), diagonal=1)
    return s.masked_fill(causal, float("-inf"))


ADAPTIVE_PARAMS = ((48, 16, 4096), (4, 2, 6), (32, 0, 64), (2048, 256, 4096))


def make_adaptive(reference: Path) -> None:
    """Adaptive-k fixture: the notebook cell's k and variance on the tiny
    configurations' reference scores and on the edge-case scores."""
    inputs = {"edge": adaptive_edge_scores()}
    for name in ("tiny_bf16", "tiny_fp32"):
        inputs[name] = torch.load(HERE / f"{name}.pt")["scores"].float()
    cases = []
    for name, scores in inputs.items():
        for kb, kmn, kmx in ADAPTIVE_PARAMS:
            k_ad, var = notebook_adaptive_k(reference, scores, kb, kmn, kmx)
            cases.append(dict(scores=name, k_base=kb, k_min=kmn, k_max=kmx,
                              k=k_ad.to(torch.int32), variance=var))
    torch.save(dict(edge_scores=inputs["edge"], cases=cases), HERE / "adaptive_k.pt")
    print("adaptive_k saved:", len(cases), "cases")


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="checkout of nirmalpratheep/GSA_GDN_BenchmarkStudy (read only)")
    ap.add_argument("--parts", default="all", choices=("all", "adaptive"),
                    help="'adaptive' regenerates only adaptive_k.pt (needs the tiny fixtures)")
    args = ap.parse_args()
    if args.parts == "adaptive":
        make_adaptive(Path(args.reference))
        return 0
    sys.path.insert(0, str(Path(args.reference) / "gsa_triton"))
    import gsa_ref as ref  # the reference implementation, unmodified
    torch.set_grad_enabled(False)

    # ---- tiny configs: whole forward + every intermediate
    for name in ("tiny_bf16", "tiny_fp32"):
        cfg = TEST_CONFIGS[name]
        m = build(ref, cfg)
        x = make_input(cfg)
        st = stages(ref, m, x)
        full = m(x)
        assert torch.equal(full, st["out"]), "stage replay differs from model(x)"
        fx = dict(config=name, x_sha256=x_digest(x), k_eff=st["k_eff"],
                  state_keys=[(k2, tuple(t.shape), str(t.dtype)) for k2, t in m.state_dict().items()],
                  out=st["out"], scores=st["scores"], idx=st["idx"].to(torch.int16),
                  mask=st["mask"], q=st["q"], k=st["k"], v=st["v"], attn=st["attn"])
        if name == "tiny_fp32":
            for key in ("q", "k", "v"):
                fx.pop(key)
        torch.save(fx, HERE / f"{name}.pt")
        print(name, "saved", {k: tuple(v.shape) for k, v in fx.items() if torch.is_tensor(v)})

    # ---- cfg1 (fp32, the reference's CPU-runnable case): whole forward
    cfg = CONFIGS["cfg1"]
    m = build(ref, cfg)
    x = make_input(cfg)
    st = stages(ref, m, x)
    assert torch.equal(m(x), st["out"])
    srows = list(range(0, cfg.T, cfg.T // 32))
    fx = dict(config="cfg1", x_sha256=x_digest(x), k_eff=st["k_eff"], out=st["out"],
              idx=st["idx"].to(torch.int16), mask=st["mask"], score_rows=torch.tensor(srows),
              scores=st["scores"][:, srows].contiguous())
    torch.save(fx, HERE / "cfg1.pt")
    print("cfg1 saved; mask.sum() =", int(st["mask"].sum()))

    # ---- cfg2 (bf16, T=4096): full-sequence stages, attention on sampled rows
    cfg = CONFIGS["cfg2"]
    m = build(ref, cfg)
    x = make_input(cfg)
    rows = [0, 1, 17, 511, 1023, 1500, 2046, 2047, 2048, 2049, 2600, 3071, 3333, 3900, 4094, 4095]
    st = stages(ref, m, x, rows=rows)
    r = torch.as_tensor(rows)
    fx = dict(config="cfg2", x_sha256=x_digest(x), k_eff=st["k_eff"], rows=r,
              out=st["out"].contiguous(), scores=st["scores"][:, r].contiguous(),
              idx=st["idx"][:, r].to(torch.int16).contiguous(),
              mask=st["mask"][:, r].contiguous())
    torch.save(fx, HERE / "cfg2_rows.pt")
    print("cfg2 saved")

    make_adaptive(Path(args.reference))
    return 0


if __name__ == "__main__":
    sys.exit(main())
