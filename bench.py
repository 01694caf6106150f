"""GSA forward benchmark on B200: tokens/s of GatedSparseAttention.forward.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg3] [--impl ours|reference]

One step = one forward of the configuration's whole batch (default cfg3:
B=1, T=16384, D=2048, H=16, k=2048, bf16) on synthetic seeded inputs and
weights.  For N > 1 the driver launches one rank per GPU under torchrun; B=1
configurations shard query rows zig-zag over the ranks (k_I, K and V are
all-gathered with NCCL, and the output rows at the end, so every rank holds the
whole output), batched ones shard sequences (outputs all-gathered likewise).

Rank 0 prints ONE JSON line.  ``value`` is whole-job tokens/s with inputs
resident in HBM, timed per step with CUDA events (max over ranks), L2 flushed
between steps outside the timed events; ``e2e`` repeats the measurement
through the public module API from pinned host memory with the host->device
copy of x and the device->host read of the output inside the timed region.
``roofline`` describes the dominant kernel (the tensor-core sparse attention),
timed live with events on its launch stream; ``cpu_baseline`` times the CPU
oracle (a restatement of gsa_ref.py) on a bounded row sample on this host.

``--impl reference`` times the reference's CPU algorithm (the oracle port of
gsa_ref.py) on all host cores for the same workload and prints the same JSON
line with impl=reference; like ``cpu_baseline`` it times a row sample and
extrapolates, and says so.

``--gpu-reference`` (single GPU) adds ``gpu_reference``: the reference's own
GPU module, gsa_triton/gsa_opt.py (Triton), unmodified and loaded from the
reference checkout installed under baseline/_ref, timed with the reference
harness's protocol (5 warm-up + 10 timed forwards, CUDA events) at cfg2 and at
the bench's configuration.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "GSA fwd tokens/s at D=2048,T=16K (1-8 B200); indexer TFLOP/s, sparse-attn GB/s"
UNIT = "tokens/s"
# dram__bytes_read.sum + dram__bytes_write.sum of one masked-attention launch at
# N=1, per configuration, each from an ncu capture of that configuration's
# bench command (the algorithmic bytes of a launch, for comparison: q, k, v, og
# and out read/written once plus the bitmask, B*T*(5*D*2 + 4*ceil(T/128)*4)).
ATTN_TRAFFIC_BYTES_PER_LAUNCH = {"cfg2": 71_964_672, "cfg3": 363_120_000, "cfg4": 1_379_490_560}


def workload_string(cfg) -> str:
    """The workload name both arms print (the driver compares them)."""
    return (f"{cfg.name}: B={cfg.B} T={cfg.T} D={cfg.D} H={cfg.H} d={cfg.d_head} "
            f"H_I={cfg.n_idx_heads} d_I={cfg.d_indexer} k={cfg.k_eff}")


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg3")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-rows", type=int, default=256)
    ap.add_argument("--unfused-projection", action="store_true",
                    help="cuBLAS addmm + the separate RoPE/gate kernel instead of the "
                         "projection GEMM with RoPE and the value gate in its epilogue")
    ap.add_argument("--adaptive-k", action="store_true",
                    help="opt-in variance-based k per row (not the reference module's fixed k)")
    ap.add_argument("--gpu-reference", action="store_true",
                    help="also time the reference's Triton module (gsa_opt.py) from baseline/_ref")
    ap.add_argument("--profile-window", action="store_true",
                    help="cudaProfilerStart/Stop around the timed device-resident steps, for "
                         "ncu --profile-from-start off (the reference's capture windows)")
    return ap.parse_args()


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        d["_source"] = "measured"
        return d
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "_source": "fallback"}


# ─────────────────────────────────────────────────────────────── clocks
class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def _lines(self) -> int:
        try:
            return len(Path(self.file.name).read_text().splitlines())
        except OSError:
            return 0

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.file, stderr=subprocess.DEVNULL)
            # the timed region starts once the sampler is producing samples
            t0 = time.time()
            while self._lines() < 1 and time.time() - t0 < 5.0:
                time.sleep(0.05)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            # one more sample that covers the end of the timed region
            n = self._lines()
            t0 = time.time()
            while self._lines() <= n and time.time() - t0 < 1.0:
                time.sleep(0.05)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        if self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(parts)
            except ValueError:
                continue
        try:
            os.unlink(self.file.name)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons,
                "samples": len(rows)}


# ─────────────────────────────────────────────────────────────── CPU baseline
class CpuSample:
    """The CPU oracle (restated gsa_ref.py) on a bounded row sample of a workload.

    Work shared by all rows (key/value/indexer-key projections + key RoPE over
    the full sequence) is timed whole; the per-row work is timed on
    ``sample_rows`` query rows spread uniformly over T and scaled by T/rows
    (and, for a batch, by B: its sequences cost the same).  The figure is an
    extrapolation from the sample, and every line that carries it says so."""

    def __init__(self, cfg, sample_rows: int, threads: int):
        from gsa_gdn_benchmarkstudy_b200.gsa import GatedSparseAttention
        from gsa_gdn_benchmarkstudy_b200.workloads import init_weights_, make_input
        from oracle import gsa_oracle as O

        self.O, self.cfg, self.threads = O, cfg, threads
        torch.set_num_threads(threads)
        m = GatedSparseAttention(**cfg.module_kwargs())
        init_weights_(m, seed=1)
        self.sd = m.to(cfg.torch_dtype).state_dict()
        self.x = make_input(cfg)[:1]
        self.rows = O.spread_rows(cfg.T, sample_rows)

    def seconds(self) -> float:
        """Extrapolated CPU seconds of one whole forward, from one timed sample."""
        cfg, tm = self.cfg, {}
        with torch.no_grad():
            self.O.forward_rows(self.sd, self.x, cfg.H, cfg.k_base, cfg.k_max, rows=self.rows,
                                row_chunk=1, timings=tm)
        return cfg.B * (tm["shared_s"] + tm["rows_s"] * cfg.T / len(self.rows))

    def describe(self, value: float) -> dict:
        cfg = self.cfg
        return {"value": value, "unit": UNIT, "cores": self.threads, "kind": "port",
                "extrapolated": True, "sample_rows": len(self.rows),
                "sample": (f"{len(self.rows)} query rows spread over T={cfg.T} of sequence 0 "
                           f"(+ full-sequence key/value projections), per-row time scaled by "
                           f"T/rows{' and by B' if cfg.B > 1 else ''}: an extrapolation; "
                           f"oracle restatement of gsa_ref.py in torch on the CPU, {cfg.dtype}")}


def cpu_baseline(cfg, sample_rows: int, threads: int) -> dict:
    s = CpuSample(cfg, sample_rows, threads)
    return s.describe(cfg.B * cfg.T / s.seconds())


# ─────────────────────────────────────────────────────────────── reference arm
def run_reference(args, cfg, rank: int):
    """The reference's CPU algorithm (oracle port of gsa_ref.py) on all host cores.
    Each step is one row sample of the workload (the same sample size as our
    line's cpu_baseline), extrapolated to the whole forward."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    sample = CpuSample(cfg, args.cpu_sample_rows, threads)
    secs = []
    for i in range(args.warmup + args.steps):
        t = sample.seconds()
        if i >= args.warmup:
            secs.append(t)
    ms = statistics.mean(secs) * 1e3
    v = cfg.B * cfg.T / (ms / 1e3)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16" if cfg.dtype == "bf16" else "f32",
        "data": "synthetic (seeded N(0,1) inputs, N(0,0.02) weights; no dataset in the reference)",
        "extrapolated": True,
        "config": {"workload": workload_string(cfg), "global_batch": cfg.B, "seq_len": cfg.T,
                   "l2": "n/a (CPU)"},
        "cpu_baseline": sample.describe(v),
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ─────────────────────────────────────────────────────────────── reference GPU row
def gpu_reference(cfg, device, names=("cfg2",)) -> dict:
    """The reference's own GPU module, gsa_triton/gsa_opt.py (Triton kernels,
    two streams), unmodified, loaded from the reference checkout installed under
    baseline/_ref, and timed with the reference harness's protocol
    (gsa_triton/benchmark.py:150-222: 5 warm-up + 10 timed forwards between two
    CUDA events, tok/s = B*T/s) on the same seeded weights and inputs as our
    arm.  Runs at each named configuration and at ``cfg``.

    The stock module raises for T > 8192 on a GPU (its RotaryEmbedding rebuilds
    the cos/sin cache from a CPU arange and the device's inv_freq,
    gsa_opt.py:410-421); that error is recorded as the configuration's result.
    A second entry then times the same module with its rotary cache built for
    T on the host before the module moves to the GPU (the constructor's own
    cache code, called with T; no reference code is changed), marked as such."""
    from gsa_gdn_benchmarkstudy_b200 import GatedSparseAttention as Ours
    from gsa_gdn_benchmarkstudy_b200.workloads import CONFIGS, init_weights_, make_input

    ref_dir = ROOT / "baseline" / "_ref"
    if not (ref_dir / "gsa_opt.py").exists():
        return {"unavailable": "baseline/_ref/gsa_opt.py not present (reference not installed)"}
    if str(ref_dir) not in sys.path:
        sys.path.insert(0, str(ref_dir))
    try:
        import gsa_opt  # noqa: F401  (the reference's own module)
    except Exception as exc:  # triton or the module itself failed to import
        return {"unavailable": f"import gsa_opt failed: {type(exc).__name__}: {exc}"[:300]}

    def one(c, prebuild_rotary: bool) -> dict:
        res = {"workload": workload_string(c), "impl": "gsa_triton/gsa_opt.py (unmodified)"}
        model = x = None
        try:
            kw = c.module_kwargs()
            ref = gsa_opt.GatedSparseAttention(**kw)
            ours = init_weights_(Ours(**kw))
            ref.load_state_dict(ours.state_dict(), strict=True)
            if prebuild_rotary:
                ref.rotary_emb._set_cos_sin_cache(c.T)
                res["note"] = (f"rotary cos/sin cache built for T={c.T} on the host before .to(cuda) "
                               "(the stock module raises for T > 8192 on a GPU)")
            model = ref.to(device).to(c.torch_dtype).eval()
            model.fuse_projections()
            x = make_input(c, device=device)
            with torch.no_grad():
                for _ in range(5):
                    model(x)
                torch.cuda.synchronize(device)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(10):
                    model(x)
                e1.record()
                torch.cuda.synchronize(device)
            ms = e0.elapsed_time(e1) / 10
            res.update({"ms_per_step": round(ms, 3), "value": round(c.B * c.T / (ms / 1e3), 1),
                        "unit": UNIT})
        except Exception as exc:
            res["error"] = f"{type(exc).__name__}: {exc}"[:300]
        finally:
            del model, x
            torch.cuda.synchronize(device)
            torch.cuda.empty_cache()
        return res

    out = {"protocol": "gsa_triton/benchmark.py:150-222 (5 warm-up + 10 timed, CUDA events)",
           "runs": []}
    todo = [CONFIGS[n] for n in names if n != cfg.name] + [cfg]
    for c in todo:
        r = one(c, prebuild_rotary=False)
        out["runs"].append(r)
        if "error" in r and c.T > 8192:
            out["runs"].append(one(c, prebuild_rotary=True))
    return out


# ─────────────────────────────────────────────────────────────── our arm
def build_model(cfg, device, adaptive_k: bool = False):
    from gsa_gdn_benchmarkstudy_b200 import GatedSparseAttention
    from gsa_gdn_benchmarkstudy_b200.workloads import init_weights_

    m = GatedSparseAttention(**cfg.module_kwargs(), adaptive_k=adaptive_k)
    init_weights_(m, seed=1)
    m = m.to(cfg.torch_dtype).to(device).eval()
    m.fuse_projections()
    return m


def run_ours(args, cfg, rank: int, world: int, device):
    from gsa_gdn_benchmarkstudy_b200 import _lib
    from gsa_gdn_benchmarkstudy_b200.build import build
    from gsa_gdn_benchmarkstudy_b200.workloads import WorkModel, make_input

    if rank == 0:
        build()
    if world > 1:
        dist.barrier()
    _lib.load()
    torch.set_grad_enabled(False)
    model = build_model(cfg, device, args.adaptive_k)
    model.use_fused_epilogue = not args.unfused_projection
    x_host = make_input(cfg).pin_memory()

    if world > 1:
        from gsa_gdn_benchmarkstudy_b200.sharding import ShardedGSA
        runner = ShardedGSA(model, dist.group.WORLD, T=cfg.T, B=cfg.B)
        x_local_host = runner.local_input(x_host).pin_memory()
        x_dev = x_local_host.to(device)
        # the whole step: every rank ends with the full output (the output rows
        # are all-gathered, as for the k_I / K / V rows before them)
        step = lambda: runner(x_dev)  # noqa: E731
        e2e_step = lambda: runner.forward_host(x_local_host)  # noqa: E731
    else:
        x_dev = x_host.to(device)
        step = lambda: model(x_dev)  # noqa: E731
        e2e_step = None

    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)  # > 126 MB L2
    stream = torch.cuda.current_stream()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---------------- device-resident timed region (K steps, per-step events)
    model._stage_events = []
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    with ClockSampler(device.index if device.index is not None else 0) as clocks:
        # the barrier comes after every rank's sampler has started: the samplers
        # start at different times, and a rank that entered the timed loop early
        # would count its wait for the others' first collective as step time
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        if args.profile_window:
            torch.cuda.profiler.start()
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record(stream)
            step()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        if args.profile_window:
            torch.cuda.profiler.stop()
    if world > 1:
        dist.barrier()
    step_ms = [a.elapsed_time(b) for a, b in ev]
    stage_events = model._stage_events
    model._stage_events = None
    local_ms = sum(step_ms)
    t = torch.tensor([local_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = t.item()
    ms_per_step = total_ms / args.steps
    value = cfg.B * cfg.T / (ms_per_step / 1e3)

    # per-kernel averages over the timed region (events on the launch stream)
    stage_ms: dict = {}
    own_launches = 0
    for name, a, b, n_launch in stage_events:
        stage_ms.setdefault(name, []).append(a.elapsed_time(b))
        if name.startswith("k:"):
            own_launches += n_launch
    stage_avg = {k: sum(v) / len(v) for k, v in stage_ms.items()}
    stage_step = {k: sum(v) / args.steps for k, v in stage_ms.items()}
    split = time_indexer_and_topk(model, x_dev if world == 1 else None, cfg)

    # ---------------- end-to-end through the public API, host buffers
    out_host = torch.empty(cfg.B, cfg.T, cfg.D, dtype=cfg.torch_dtype).pin_memory()
    eager_host = None
    e2e_path = "ShardedGSA.forward_host"
    if e2e_step is None:
        # one GPU: forward_host captured as one CUDA graph (GraphedForwardHost);
        # every replay copies the pinned input in and the output back out
        eager_host = lambda: model.forward_host(x_host, out=out_host)  # noqa: E731
        try:
            graphed = model.graphed_host(x_host.shape)
            graphed.x.copy_(x_host)
            e2e_step = graphed
            e2e_path = ("GatedSparseAttention.graphed_host: forward_host replayed as one CUDA "
                        "graph")
        except RuntimeError as exc:  # capture refused: time the eager pipeline instead
            torch.cuda.synchronize()
            e2e_step, eager_host = eager_host, None
            e2e_path = f"GatedSparseAttention.forward_host (graph capture failed: {exc})"[:300]

    def timed_host_steps(fn):
        ev_ = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        for _ in range(args.warmup):  # untimed, as for the device-resident steps
            fn()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(args.steps):
            flush.zero_()
            ev_[i][0].record(stream)
            fn()  # returns once the output is in host memory
            ev_[i][1].record(stream)
        torch.cuda.synchronize()
        return [a.elapsed_time(b) for a, b in ev_]

    e2e_steps = timed_host_steps(e2e_step)
    e2e_local = sum(e2e_steps)
    e2e_median = statistics.median(e2e_steps)
    t = torch.tensor([e2e_local], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = t.item() / args.steps
    eager_host_ms = (statistics.mean(timed_host_steps(eager_host)) if eager_host is not None
                     else None)
    # bytes copied per step by each rank: its input share in, its output rows out
    h2d = x_host.numel() * x_host.element_size() // world
    d2h = out_host.numel() * out_host.element_size() // world

    if rank != 0:
        return
    pk = peaks()
    wm = WorkModel(cfg)
    attn_ms = stage_avg.get("k:masked_attention")
    rl = None
    if attn_ms:
        # algorithmic work of one launch: QK^T + PV over the causal key range of the
        # launch's rows (the formulation the kernel computes), B sequences / world ranks
        n_at = stage_count(stage_ms, "k:masked_attention", args.steps)
        flops = wm.attn_dense_flops / world / n_at
        achieved = flops / (attn_ms / 1e3) / 1e12
        peak = pk["bf16_tflops"]
        traffic = ATTN_TRAFFIC_BYTES_PER_LAUNCH.get(cfg.name) if world == 1 else None
        rl = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
              "frac": round(achieved / peak, 4), "traffic": traffic,
              "kernel": "masked_attn_kernel (tcgen05)", "peak_kind": f"bf16 burst, {pk['_source']}",
              "ms_per_launch": round(attn_ms, 4),
              # the same launch time over the flops of the selected (query, key)
              # pairs only: the share of the tensor work the selection needs
              "useful_frac": round(wm.attn_sparse_flops / world / n_at / (attn_ms / 1e3) / 1e12
                                   / peak, 4),
              "traffic_source": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch "
                                 f"of this bench at {cfg.name}, N=1" if traffic is not None else
                                 "no ncu capture of this configuration and N")}
    extra = {}
    if split:
        extra["indexer_ms"] = round(split["indexer"], 4)
        extra["topk_ms"] = round(split["topk"], 4)
        extra["indexer_tflops"] = round(wm.indexer_flops / (split["indexer"] / 1e3) / 1e12, 2)
    if attn_ms:
        extra["sparse_attn_gather_equiv_gbs"] = round(
            wm.attn_gather_bytes / world / n_at / (attn_ms / 1e3) / 1e9, 1)
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16"
        if cfg.dtype == "bf16" else "f32",
        "data": "synthetic (seeded N(0,1) inputs, N(0,0.02) weights; no dataset in the reference)",
        "config": {"workload": workload_string(cfg),
                   "global_batch": cfg.B, "seq_len": cfg.T,
                   "parallelism": ("single GPU" if world == 1 else
                                   ("query-row zig-zag shards" if cfg.B == 1 else "batch shards")),
                   "l2": "flushed between steps (256 MB memset outside the step events)",
                   **({"adaptive_k": True} if args.adaptive_k else {})},
        "gpu_launches": own_launches,
        "clocks": clocks.summary(),
        "e2e": {"value": round(cfg.B * cfg.T / (e2e_ms / 1e3), 1), "unit": UNIT,
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "ms_per_step": round(e2e_ms, 4), "ms_per_step_median_rank0": round(e2e_median, 4),
                "path": e2e_path,
                **({"forward_host_ms_per_step": round(eager_host_ms, 4)}
                   if eager_host_ms is not None else {})},
        "roofline": rl,
        # per stage: device time summed over the stage's launches in one step
        # (events on the stream that issues it; rank 0)
        "stage_ms": {stage_label(k): round(v, 4) for k, v in stage_step.items()},
        **extra,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, args.cpu_sample_rows, os.cpu_count() or 1)
    if world == 1:
        ref_mod = None
        if args.gpu_reference:
            line["gpu_reference"] = gpu_reference(cfg, device)
            ref_mod = sys.modules.get("gsa_opt")
        line["gather_attention"] = time_gather_attention(device, reference=ref_mod)
    print(json.dumps(line), flush=True)


def time_gather_attention(device, name: str = "cfg2", iters: int = 3, reference=None) -> dict:
    """The index-gather attention kernel (the op-level fused_sparse_attention /
    sparse_attention_ref, gsa_opt.py:349-383) on a configuration's own q, k, v
    and top-k index lists, event-timed.  Its work is the gathered K and V rows
    of every selected (query, key) pair plus q in, out and the indices
    (WorkModel.attn_gather_bytes), reported as GB/s and as a fraction of the
    measured HBM peak; the rows mostly come from L2.  With ``reference`` (the
    gsa_opt module) the reference's Triton kernel is timed on the same inputs."""
    from gsa_gdn_benchmarkstudy_b200 import ops
    from gsa_gdn_benchmarkstudy_b200.workloads import CONFIGS, WorkModel, make_input

    c = CONFIGS[name]
    m = build_model(c, device)
    x = make_input(c, device=device)
    parts = m.split(m.project(x))
    cos, sin = m.rotary_emb(c.T, device, x.dtype)
    q, k, v = ops.rope_gates(parts["q"], parts["k"], cos, sin, c.H, v_src=parts["v"],
                             vg_src=parts["vg"])
    ix = m.indexer
    idx, mask, _ = ops.indexer_topk(parts["iq"], parts["ik"], parts["iw"], ix.bias_f32(),
                                    ix.scale, c.k_eff, want_indices=True, want_mask=True,
                                    want_bitmask=False)
    shape = (c.B, c.T, c.H, c.d_head)
    q4, k4, v4 = q.view(shape), k.view(shape), v.view(shape)

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters

    ms = timed(lambda: ops.fused_sparse_attention(q4, k4, v4, idx, mask, m.scale))
    gb = WorkModel(c).attn_gather_bytes / 1e9
    res = {"workload": workload_string(c), "kernel": "gather_attn_kernel", "ms": round(ms, 3),
           "gathered_gbs": round(gb / (ms / 1e3), 1),
           "frac_of_hbm": round(gb / (ms / 1e3) / peaks()["hbm_gbs"], 4)}
    if reference is not None:
        try:
            idx64 = idx.long()
            rms = timed(lambda: reference.fused_sparse_attention(q4, k4, v4, idx64, mask, m.scale))
            res["reference_triton_ms"] = round(rms, 3)
        except Exception as exc:  # the reference kernel failed to compile or run
            res["reference_triton_error"] = f"{type(exc).__name__}: {exc}"[:200]
    del m
    torch.cuda.empty_cache()
    return res


def time_indexer_and_topk(model, x, cfg, iters: int = 5):
    """Event-timed indexer and top-k kernels alone (the forward runs them fused
    in one C call), on this step's own projections; single-GPU runs only."""
    if x is None:
        return None
    from gsa_gdn_benchmarkstudy_b200 import ops

    parts = model.split(model.project(x))
    ix = model.indexer
    k_eff = model.topk_selector.k_effective(cfg.T)
    res = {}
    scores = ops.indexer_scores(parts["iq"], parts["ik"], parts["iw"], ix.idx_bias, ix.scale,
                                fill_upper=False)
    # one bitmask for every call: allocations do not land between the timing events
    bm = torch.empty(cfg.B, cfg.T, ops.bitmask_words(cfg.T), device=x.device, dtype=torch.int32)
    for name in ("indexer", "topk"):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            if name == "indexer":
                ops.indexer_scores(parts["iq"], parts["ik"], parts["iw"], ix.idx_bias, ix.scale,
                                   fill_upper=False, out=scores.as_strided(
                                       (cfg.B, cfg.T, scores.stride(1)),
                                       (scores.stride(0), scores.stride(1), 1)))
            else:
                ops.topk_select(scores, k_eff, want_indices=False, want_mask=False,
                                bitmask_out=bm)
        e1.record()
        torch.cuda.synchronize()
        res[name] = e0.elapsed_time(e1) / iters
    return res


def stage_label(name: str) -> str:
    """Stage names of the bench line: our kernels bare, library calls tagged."""
    kind, _, rest = name.partition(":")
    return {"k": rest, "lib": f"{rest} (cuBLAS)", "comm": f"{rest} (NCCL)"}.get(kind, name)


def stage_count(stage_ms: dict, name: str, steps: int) -> float:
    return len(stage_ms.get(name, [])) / steps


def main():
    args = parse_args()
    from gsa_gdn_benchmarkstudy_b200.workloads import CONFIGS

    cfg = CONFIGS[args.config]
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, cfg, rank)
        return
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    try:
        run_ours(args, cfg, rank, world, device)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
