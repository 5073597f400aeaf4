"""Benchmark of the column-sparse linear hot path on B200.

Headline workload (one "step"): one fused gather-GEMM of the standalone sweep's
reference point, y = x[:, alive] @ W'^T with x [4096, 4096] fp16, W [4096, 4096]
fp16 ~ N(0, 1/sqrt(K)) with 50 % of its input columns (seeded uniform choice)
zeroed, K' = 2048 alive columns found by the mask kernel and packed once.
Metric: useful TFLOP/s = 2*M*N*K' / time (dense-equivalent 2*M*N*K also shown).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload gemm|mlp-sharded|ghostlinear-fp32|gpt2|distilbert]
                  [--no-sweep] [--no-cpu-baseline]

* Inputs are resident in HBM: 4 independent layers (x, W', y) rotate so every
  step reads cold data (4 x 80 MB > 126 MB L2).
* Device time by CUDA events on the launching stream, barrier + synchronize on
  both sides, max over ranks. N > 1 (torchrun): every rank runs its own batch
  through its own copy of the layer ("scaling": "weak"); no collective on the
  data path. --workload mlp-sharded runs the sharded MLP projection instead:
  x [8192, 8192] bf16, W [28672, 8192] with 70 % dead 128-column blocks,
  output features split across ranks, NCCL all-gather of y ("strong").
* e2e: the same step through GhostLinear (frozen weight mask) with x copied
  from pinned host memory and y copied back inside the timed region.
* --impl reference: the reference's CPU path for this computation
  (A.float()[:, idx] @ W.float()[idx, :], tests/test_matmul.py:30-42 of
  ghostweight-triton), restated by the oracle in numpy on all host cores, on
  a bounded row sample per step; rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

import numpy as np  # noqa: E402
import torch  # noqa: E402

HEADLINE = dict(M=4096, N=4096, K=4096, sparsity=0.5, pattern="random", dtype="fp16")
MLP = dict(M=8192, N=28672, K=8192, sparsity=0.7, pattern="block128", dtype="bf16")
METRIC = "useful TFLOP/s of the fused gather-GEMM (2*M*N*K')"
N_SETS = 4
L2_FLUSH_BYTES = 2 * 126 * 2**20     # twice the B200 L2: rotated inputs summing past this come from HBM
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


# ---------------------------------------------------------------------------- helpers
def load_peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def dead_columns(K: int, sparsity: float, seed: int, pattern: str) -> np.ndarray:
    rng = np.random.default_rng(seed + 7919)
    if pattern == "random":
        return np.sort(rng.permutation(K)[: int(K * sparsity)])
    block = int(pattern.replace("block", ""))
    nb = K // block
    blocks = np.sort(rng.permutation(nb)[: int(nb * sparsity)])
    return (blocks[:, None] * block + np.arange(block)[None, :]).reshape(-1)


class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons while the GPU is busy."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.rows: list[list[str]] = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu_index), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return self

        def reader():
            for line in self.proc.stdout:
                self.rows.append([c.strip() for c in line.split(",")])

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()
        return self

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=5)
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1])); smax.append(float(r[2])); power.append(float(r[3]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def physical_gpu_index(local: int) -> int:
    cvd = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    parts = [p.strip() for p in cvd.split(",") if p.strip()]
    if local < len(parts) and parts[local].isdigit():
        return int(parts[local])
    return local


def gpu_local_cpus(device_index: int) -> set[int] | None:
    """CPUs that NVML reports as nearest the GPU (its NUMA node), within this
    process's allowed set; None when NVML or the affinity call is unavailable."""
    try:
        import pynvml

        uuid = str(torch.cuda.get_device_properties(device_index).uuid)
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            words = pynvml.nvmlDeviceGetCpuAffinity(h, ((os.cpu_count() or 64) + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = {64 * i + b for i, w in enumerate(words) for b in range(64) if (int(w) >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        return cpus or None
    except Exception:
        return None


class NearGpu:
    """Run a block on the CPUs nearest this rank's GPU, so that host buffers
    first touched inside it live on the GPU's NUMA node; the previous affinity
    comes back on exit."""

    def __init__(self, device_index: int):
        self.cpus = gpu_local_cpus(device_index)
        self.prev = None

    def __enter__(self):
        if self.cpus:
            self.prev = os.sched_getaffinity(0)
            os.sched_setaffinity(0, self.cpus)
        return self

    def __exit__(self, *exc):
        if self.prev:
            os.sched_setaffinity(0, self.prev)

    def describe(self) -> str:
        if not self.cpus:
            return "not bound (no NVML CPU affinity)"
        return f"{len(self.cpus)} CPUs NVML reports nearest the GPU (of {len(self.prev or self.cpus)} allowed)"


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        # NCCL's communicator set-up lines (the rank count of every communicator)
        # on stderr, so that stdout keeps only the JSON line; unless the caller
        # asked for more than INFO already.
        if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
            os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        if args.impl == "ours":
            torch.cuda.set_device(local)
        dist.init_process_group("nccl" if args.impl == "ours" else "gloo",
                                timeout=datetime.timedelta(seconds=300))
    elif args.impl == "ours":
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed(fn, steps: int, world: int, stream=None) -> float:
    """Seconds for `steps` calls of fn(i), CUDA events on the launching stream, max over ranks."""
    barrier(world)
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for i in range(steps):
        fn(i)
    e.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(s.elapsed_time(e) / 1e3, world)


def event_time(fn, iters: int = 10, warmup: int = 3) -> float:
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(iters):
        fn(i)
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / 1e3 / iters


# ---------------------------------------------------------------------------- CPU reference path
def cpu_reference_sample(M: int, N: int, K: int, sparsity: float, pattern: str, rows: int,
                         budget_s: float, max_reps: int, seed: int = 0,
                         exact: tuple[int, int] | None = None) -> dict:
    """Time the oracle (numpy, all cores) on `rows` rows of the workload.

    Default: up to max_reps timed calls within budget_s after one warm call.
    exact = (warmup, steps): that many untimed, then exactly that many timed
    calls; if they would take longer than budget_s, the sample shrinks to fewer
    rows (at least 16) instead."""
    from oracle import gw_oracle as O

    try:
        from threadpoolctl import threadpool_limits
    except Exception:  # pragma: no cover
        threadpool_limits = None
    cores = os.cpu_count() or 1
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, K), dtype=np.float32).astype(np.float16)
    w_kn = (rng.standard_normal((K, N), dtype=np.float32) / np.sqrt(K)).astype(np.float16)
    dead = dead_columns(K, sparsity, seed, pattern)
    w_kn[dead, :] = 0
    x[:, dead] = 0
    idx = np.setdiff1d(np.arange(K), dead)
    ctx = threadpool_limits(limits=cores) if threadpool_limits else None
    try:
        # The first untimed call also sizes the sample (it counts as one of the
        # warm-up calls when `exact` asks for a fixed number of them).
        t0 = time.perf_counter()
        O.ghostweight_matmul(x, w_kn, idx)
        t_warm = time.perf_counter() - t0
        times = []
        if exact is not None:
            warmup, steps = exact
            if (warmup + steps) * t_warm > budget_s:
                shrunk = max(16, int(rows * budget_s / ((warmup + steps) * t_warm)))
                x = np.ascontiguousarray(x[:min(rows, shrunk)])
            for _ in range(max(0, warmup - 1)):
                O.ghostweight_matmul(x, w_kn, idx)
            for _ in range(steps):
                t0 = time.perf_counter()
                O.ghostweight_matmul(x, w_kn, idx)
                times.append(time.perf_counter() - t0)
        else:
            t_end = time.perf_counter() + budget_s
            while len(times) < max_reps and (not times or time.perf_counter() < t_end):
                t0 = time.perf_counter()
                O.ghostweight_matmul(x, w_kn, idx)
                times.append(time.perf_counter() - t0)
    finally:
        if ctx is not None:
            ctx.__exit__(None, None, None)
    t = statistics.median(times)
    rows = x.shape[0]
    flops = 2.0 * rows * N * len(idx)
    return {"value": flops / t / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "seconds_per_sample": t, "reps": len(times), "rows": rows,
            "sample": f"{rows} of {M} rows of x through oracle.ghostweight_matmul "
                      f"(fp32 gather + numpy sgemm over K'={len(idx)}, N={N}), median of {len(times)}"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    cfg = HEADLINE
    rows = 256
    # W untimed and exactly K timed calls, each on a sample of the workload's
    # rows, bounded to about 150 s of CPU work in all.
    res = cpu_reference_sample(cfg["M"], cfg["N"], cfg["K"], cfg["sparsity"], cfg["pattern"], rows,
                               budget_s=150.0, max_reps=args.steps, exact=(args.warmup, args.steps))
    kp = cfg["K"] - int(cfg["K"] * cfg["sparsity"])
    line = {
        "impl": "reference", "metric": METRIC, "value": round(res["value"], 6), "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": res["reps"], "warmup": args.warmup,
        "ms_per_step": round(res["seconds_per_sample"] * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16 in, fp32 compute (CPU)",
        "data": "synthetic (seeded N(0,1) activations, N(0,1/sqrt(K)) weight, dead columns zeroed)",
        "config": {"workload": "gather-GEMM M=N=K=4096, 50% random dead input columns",
                   "M": cfg["M"], "N": cfg["N"], "K": cfg["K"], "K_alive": kp,
                   "sample_rows": res["rows"]},
        "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": round(res["value"], 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- reference's Triton kernels on the GPU
REF_DIR = REPO / "baseline" / "_ref"
REF_WARMUP, REF_ITERS = 10, 100              # benchmarks/bench_kernels.py:45-46 of the reference
# (name, M, N, K, dead fraction): the headline point, the standalone sweep's
# other row counts and 90%, and the reference benchmark's own layer shapes
# (benchmarks/bench_kernels.py:34-41) at 50%.
REF_MATMUL_CASES = [("headline_4096x4096x4096_s50", 4096, 4096, 4096, 0.5),
                    ("sweep_4096x4096x4096_s90", 4096, 4096, 4096, 0.9),
                    ("sweep_1024x4096x4096_s50", 1024, 4096, 4096, 0.5),
                    ("sweep_128x4096x4096_s50", 128, 4096, 4096, 0.5),
                    ("sweep_16x4096x4096_s50", 16, 4096, 4096, 0.5),
                    ("layer_1x3072x768_s50", 1, 3072, 768, 0.5),
                    ("layer_16x3072x768_s50", 16, 3072, 768, 0.5),
                    ("layer_128x3072x768_s50", 128, 3072, 768, 0.5),
                    ("layer_128x768x3072_s50", 128, 768, 3072, 0.5)]


def cuda_mean_ms(fn, warmup: int = REF_WARMUP, iters: int = REF_ITERS) -> float:
    """Mean per-call time of fn() by CUDA events, as the reference's benchmark measures it."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def _ref_inputs(device) -> dict:
    """Seeded inputs shared by the reference child process and the comparison."""
    g = torch.Generator(device=device).manual_seed(2026)
    out = {}
    for name, M, N, K, sp in REF_MATMUL_CASES:
        x = torch.randn(M, K, device=device, generator=g).half()
        w_kn = (torch.randn(K, N, device=device, generator=g) / K ** 0.5).half()
        dead = torch.from_numpy(dead_columns(K, sp, M + N, "random")).to(device)
        x[:, dead] = 0
        w_kn[dead, :] = 0
        out[name] = (x, w_kn)
    # Mask semantics cases: NaN handling (mask.py:55), the fp16 threshold
    # boundary (fp32 compare, mask.py:53-58), an fp32 matrix, all-dead rows.
    nan = torch.randn(64, 256, device=device, generator=g).half()
    nan[:, :64] = 0
    nan[5, 0] = float("nan")                     # NaN + zeros: dead
    nan[7, 1] = float("nan")
    nan[9, 1] = 0.5                              # NaN + a live value: alive
    nan[:, 2] = float("nan")                     # all NaN: dead
    bound = torch.zeros(16, 128, device=device).half()
    bound[3, :64] = 1.0133e-06                   # just above 1e-6 in fp32, not in fp16
    bound[4, 64:] = 9.5e-07
    f32 = torch.randn(200, 320, device=device, generator=g)
    f32[:, ::3] = 0
    out["mask_nan"] = (nan, 1e-6)
    out["mask_fp16_threshold_boundary"] = (bound, 1e-6)
    out["mask_f32"] = (f32, 0.0)
    return out


def reference_triton_child(outdir: str) -> None:
    """Runs in a separate process: the unmodified reference package from baseline/_ref.

    This repository also holds a package under the reference's import name, so
    the repository is taken off sys.path before the reference is imported.
    Times dead_neuron_mask, gather_compact and ghostweight_matmul (CUDA events,
    10 warm-up, 100 iterations) and saves their outputs for the comparison.
    """
    sys.path[:] = [p for p in sys.path if Path(p or ".").resolve() != REPO]
    sys.path.insert(0, str(REF_DIR))
    import triton

    import ghostweight_triton as ref
    from ghostweight_triton.kernels import dead_neuron_mask, gather_compact, ghostweight_matmul

    assert Path(ref.__file__).resolve().is_relative_to(REF_DIR.resolve()), ref.__file__
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    inp = _ref_inputs(device)
    res = {"triton": triton.__version__, "package": str(Path(ref.__file__).parent.relative_to(REPO)),
           "ms": {}, "outputs": {}}
    saved = {}
    for name, (x, thr) in [(k, v) for k, v in inp.items() if k.startswith("mask_")]:
        saved[name] = dead_neuron_mask(x, threshold=thr).cpu()
    x, w_kn = inp["headline_4096x4096x4096_s50"]
    res["ms"]["dead_neuron_mask_4096x4096_fp16"] = cuda_mean_ms(lambda: dead_neuron_mask(x, threshold=0.0))
    m = dead_neuron_mask(x, threshold=0.0)
    idx = torch.nonzero(m).squeeze(-1).to(torch.int64)
    saved["mask_headline"] = m.cpu()
    res["ms"]["gather_compact_4096x4096_s50_fp16"] = cuda_mean_ms(lambda: gather_compact(x, w_kn, idx))
    a_c, w_c = gather_compact(x, w_kn, idx)
    saved["gather_a"], saved["gather_w"] = a_c.cpu(), w_c.cpu()
    for name, M, N, K, sp in REF_MATMUL_CASES:
        x, w_kn = inp[name]
        m = dead_neuron_mask(x, threshold=0.0)
        idx = torch.nonzero(m).squeeze(-1).to(torch.int64)
        res["ms"][f"ghostweight_matmul_{name}"] = cuda_mean_ms(lambda: ghostweight_matmul(x, w_kn, idx))
        if M <= 1024:
            saved[f"matmul_{name}"] = ghostweight_matmul(x, w_kn, idx).cpu()
    torch.save(saved, Path(outdir) / "ref_outputs.pt")
    (Path(outdir) / "ref_times.json").write_text(json.dumps(res))


def reference_triton_record(timeout_s: float = 420.0) -> dict:
    """The reference's own Triton kernels timed on this GPU beside ours, outputs compared.

    Both sides run the same calls through the same Python surface
    (dead_neuron_mask, gather_compact, ghostweight_matmul) on the same seeded
    inputs; speed-up = reference time / our time. Masks and alive lists must
    be bit-identical (a NaN column and the fp16 threshold boundary included),
    gathers identical, matmul outputs within 1e-2.
    """
    import tempfile

    if not (REF_DIR / "ghostweight_triton" / "__init__.py").exists():
        return {"unavailable": "reference package not installed under baseline/_ref"}
    from ghostweight_triton_b200.kernels import dead_neuron_mask, gather_compact, ghostweight_matmul

    with tempfile.TemporaryDirectory() as td:
        env = dict(os.environ)
        env.pop("PYTHONPATH", None)
        try:
            proc = subprocess.run([sys.executable, str(REPO / "bench.py"), "--reference-triton-child", td],
                                  cwd=td, env=env, capture_output=True, text=True, timeout=timeout_s)
        except subprocess.TimeoutExpired:
            return {"unavailable": f"reference child did not finish in {timeout_s:.0f} s"}
        if proc.returncode != 0:
            return {"unavailable": "reference child failed: " + proc.stderr.strip().splitlines()[-1][:300]
                    if proc.stderr.strip() else f"reference child exit {proc.returncode}"}
        ref = json.loads((Path(td) / "ref_times.json").read_text())
        outs = torch.load(Path(td) / "ref_outputs.pt")
    device = torch.device("cuda", torch.cuda.current_device())
    inp = _ref_inputs(device)
    parity = {}
    for name in [k for k in inp if k.startswith("mask_")]:
        x, thr = inp[name]
        parity[name] = bool(torch.equal(dead_neuron_mask(x, threshold=thr).cpu(), outs[name]))
    ours = {}
    x, w_kn = inp["headline_4096x4096x4096_s50"]
    ours["dead_neuron_mask_4096x4096_fp16"] = cuda_mean_ms(lambda: dead_neuron_mask(x, threshold=0.0))
    m = dead_neuron_mask(x, threshold=0.0)
    parity["mask_headline"] = bool(torch.equal(m.cpu(), outs["mask_headline"]))
    idx = torch.nonzero(m).squeeze(-1).to(torch.int64)
    ours["gather_compact_4096x4096_s50_fp16"] = cuda_mean_ms(lambda: gather_compact(x, w_kn, idx))
    a_c, w_c = gather_compact(x, w_kn, idx)
    parity["gather_compact"] = bool(torch.equal(a_c.cpu(), outs["gather_a"]) and
                                    torch.equal(w_c.cpu(), outs["gather_w"]))
    worst = -float("inf")
    for name, M, N, K, sp in REF_MATMUL_CASES:
        x, w_kn = inp[name]
        idx = torch.nonzero(dead_neuron_mask(x, threshold=0.0)).squeeze(-1).to(torch.int64)
        ours[f"ghostweight_matmul_{name}"] = cuda_mean_ms(lambda: ghostweight_matmul(x, w_kn, idx))
        key = f"matmul_{name}"
        if key in outs:
            y = ghostweight_matmul(x, w_kn, idx).float().cpu()
            r = outs[key].float()
            worst = max(worst, float(((y - r).abs() - (1e-2 + 1e-2 * r.abs())).max()))
    parity["matmul_max_excess_vs_reference"] = round(worst, 6)
    parity["native_parity"] = all(v for k, v in parity.items() if isinstance(v, bool)) and worst <= 0.0
    kernels = {}
    for k, t_ref in ref["ms"].items():
        t_ours = ours.get(k)
        kernels[k] = {"reference_ms": round(t_ref, 5), "ours_ms": round(t_ours, 5) if t_ours else None,
                      "speedup": round(t_ref / t_ours, 3) if t_ours else None}
    return {"what": "the reference's Triton kernels (unmodified, baseline/_ref) JIT-compiled on this GPU, "
                    "and ours, through the same Python calls; CUDA events, 10 warm-up + 100 iterations, mean",
            "triton": ref["triton"], "kernels": kernels, "parity": parity,
            "native_parity": parity["native_parity"],
            "note": "ghostweight_matmul takes W as [K, N] per call on both sides, so ours packs W' "
                    "(the transposing gather) inside every call; a GhostLinear packs it once"}


# ---------------------------------------------------------------------------- ours: headline GEMM
def build_layer(M, N, K, sparsity, pattern, dtype, seed, device):
    from ghostweight_triton_b200.kernels.gather import pack_weight
    from ghostweight_triton_b200.kernels.mask import alive_indices

    g = torch.Generator(device=device).manual_seed(seed)
    w = (torch.randn(N, K, device=device, generator=g) / K ** 0.5).to(dtype)
    x = torch.randn(M, K, device=device, generator=g).to(dtype)
    dead = torch.from_numpy(dead_columns(K, sparsity, seed, pattern)).to(device)
    w[:, dead] = 0
    x[:, dead] = 0
    idx = alive_indices(w, 0.0)
    wp = pack_weight(w, idx)
    y = torch.empty(M, N, device=device, dtype=dtype)
    return dict(x=x, w=w, idx=idx, wp=wp, y=y)


def kernel_metrics(device, peaks) -> dict:
    """Mask (K1) and weight-packing (K2) achieved bandwidth on two weights.

    Kernel time per call from a CUDA graph of 30 calls (no host time), each
    call on the next of enough copies of the weight that their sum exceeds
    L2, so every call reads from HBM.
    """
    from ghostweight_triton_b200 import _native
    from ghostweight_triton_b200.kernels.gather import PACK_ALIGN

    calls = 30
    out = {}
    # Each weight with its own workload's dead pattern: the headline layer 50%
    # random columns (K' = 2048), the sharded MLP projection 70% of its
    # 128-column blocks (K' = 2560).
    for name, (N, K, dt, sp, pat) in {
            "headline_weight_4096x4096_fp16_random50": (4096, 4096, torch.float16, 0.5, "random"),
            "mlp_weight_28672x8192_bf16_block128_70": (28672, 8192, torch.bfloat16, MLP["sparsity"],
                                                       MLP["pattern"])}.items():
        w = torch.randn(N, K, device=device).to(dt)
        dead = torch.from_numpy(dead_columns(K, sp, 1, pat)).to(device)
        w[:, dead] = 0
        esz = w.element_size()
        copies = [w] + [w.clone() for _ in range(-(-L2_FLUSH_BYTES // (N * K * esz)))]
        mask = torch.empty(K, dtype=torch.int32, device=device)
        buf = torch.empty(K, dtype=torch.int64, device=device)
        cnt = torch.empty(1, dtype=torch.int32, device=device)
        _native.mask_compact(w, 0.0, mask, buf, cnt)
        kp = int(cnt.item())
        idx = buf[:kp].clone()
        ld = max(-(-kp // PACK_ALIGN) * PACK_ALIGN, PACK_ALIGN)
        wp = torch.empty(N, ld, dtype=dt, device=device)
        t_mask = graph_time(lambda: [_native.mask_compact(copies[i % len(copies)], 0.0, mask, buf, cnt)
                                     for i in range(calls)], 10, 1) / calls
        t_pack = graph_time(lambda: [_native.gather_columns(copies[i % len(copies)], idx, wp, pad_to=ld)
                                     for i in range(calls)], 10, 1) / calls
        assert int(cnt.item()) == kp
        mask_bytes = N * K * esz + K * 4 + kp * 8
        pack_bytes = 2 * N * kp * esz
        # What the pack has to move at DRAM granularity: every 32-byte sector
        # of a row that holds an alive column is read whole (50% random dead
        # columns leave almost none untouched), and ld columns are written.
        sectors = int(torch.unique(idx * esz // 32).numel())
        pack_sector_bytes = N * sectors * 32 + N * ld * esz
        out[name] = {"mask_us": round(t_mask * 1e6, 2),
                     "mask_GBps": round(mask_bytes / t_mask / 1e9, 1),
                     "mask_frac_hbm": round(mask_bytes / t_mask / 1e9 / peaks["hbm_gbs"], 3),
                     "pack_us": round(t_pack * 1e6, 2),
                     "pack_GBps": round(pack_bytes / t_pack / 1e9, 1),
                     "pack_frac_hbm": round(pack_bytes / t_pack / 1e9 / peaks["hbm_gbs"], 3),
                     "pack_touched_sector_bytes": pack_sector_bytes,
                     "pack_frac_hbm_touched_sectors": round(pack_sector_bytes / t_pack / 1e9 / peaks["hbm_gbs"], 3),
                     "K_alive": kp, "copies_rotated": len(copies),
                     "timing": f"CUDA graph of {calls} calls over the rotated copies, per call"}
        del w, copies, wp
    torch.cuda.empty_cache()
    return out


def sweep(device, peaks) -> list[dict]:
    """M in {4096, 1024, 128, 16} x sparsity x {random, block64}: ours vs dense cuBLAS."""
    import torch.nn.functional as F

    from ghostweight_triton_b200.kernels.matmul import ghost_linear, ghost_linear_pipelined

    rows = []
    K = N = 4096
    for M in (4096, 1024, 128, 16):
        for pattern in ("random", "block64"):
            for sp in (0.0, 0.25, 0.5, 0.75, 0.9):
                L = build_layer(M, N, K, sp, pattern, torch.float16, 100 + M, device)
                kp = L["idx"].numel()
                yd = torch.empty(M, N, dtype=torch.float16, device=device)
                ours = lambda: ghost_linear(L["x"], L["wp"], L["idx"], out=L["y"])
                dense = lambda: torch.mm(L["x"], L["w"].t(), out=yd)
                t = event_time(lambda i: ours(), iters=20)
                td = event_time(lambda i: F.linear(L["x"], L["w"]), iters=20)
                # The same calls replayed from CUDA graphs of 20 calls each:
                # kernel time without the per-call host overhead (which
                # dominates at M <= 128) or one graph launch per call.
                tg = graph_time(lambda: [ours() for _ in range(20)], 20, 1) / 20
                tdg = graph_time(lambda: [dense() for _ in range(20)], 20, 1) / 20
                useful = 2.0 * M * N * kp
                runs = {}
                if M > 4:
                    # The same 20 calls as independent batches through
                    # ghost_linear_pipelined (each gather under the previous
                    # GEMM), captured in one graph. At most 4 rows the decode
                    # kernel gathers x' itself and nothing is pipelined.
                    tpg = graph_time(lambda: ghost_linear_pipelined(
                        [(L["x"], L["wp"], L["idx"], L["y"])] * 20), 20, 1) / 20
                    runs.update({"graph_pipelined_us": round(tpg * 1e6, 2),
                                 "graph_pipelined_speedup_vs_dense": round(tdg / tpg, 3)})
                if pattern.startswith("block"):
                    # 64-column runs: the GEMM reads x in place (no gather launch).
                    direct = lambda: ghost_linear(L["x"], L["wp"], L["idx"], out=L["y"], strategy="runs")
                    tr = event_time(lambda i: direct(), iters=20)
                    trg = graph_time(lambda: [direct() for _ in range(20)], 20, 1) / 20
                    runs.update({"runs_us": round(tr * 1e6, 2), "graph_runs_us": round(trg * 1e6, 2),
                                 "graph_runs_speedup_vs_dense": round(tdg / trg, 3)})
                rows.append({"M": M, "pattern": pattern, "sparsity": sp, "K_alive": kp,
                             "us": round(t * 1e6, 2), "useful_tflops": round(useful / t / 1e12, 1),
                             "dense_equiv_tflops": round(2.0 * M * N * K / t / 1e12, 1),
                             "frac_tensor_peak": round(useful / t / 1e12 / peaks["bf16_tflops"], 3),
                             "cublas_dense_us": round(td * 1e6, 2),
                             "speedup_vs_dense": round(td / t, 3), "ideal": round(K / kp, 3),
                             "graph_us": round(tg * 1e6, 2), "graph_cublas_dense_us": round(tdg * 1e6, 2),
                             "graph_speedup_vs_dense": round(tdg / tg, 3), **runs})
                del L
    torch.cuda.empty_cache()
    return rows


def traffic_from_profiles() -> float | None:
    """DRAM bytes (read + write) per launch of the headline GEMM from the committed ncu summary."""
    p = REPO / "profiles" / "gemm_tc2_pair_4096x4096x2048_fp16.md"
    if p.exists():
        for line in p.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1])
    return None


def dynamic_decode_record(steps: int) -> dict:
    """The per-forward activation mask at decode size (16 rows, 50% of x's columns zero):
    the single launch (gw_dynamic_linear: mask, compaction and GEMM) against the four
    launches of the device-count path (mask, weight packing, gather, GEMM) and dense
    cuBLAS, on GPT-2's MLP shapes and 4096 x 4096; 16 layers per CUDA graph, replayed."""
    import torch.nn.functional as F

    from ghostweight_triton_b200 import _native
    from ghostweight_triton_b200.kernels.gather import pack_weight_dev
    from ghostweight_triton_b200.kernels.mask import dead_neuron_mask_compact
    from ghostweight_triton_b200.kernels.matmul import ghost_linear_dev

    dev = torch.device("cuda", torch.cuda.current_device())
    n_layers = 16
    out = []
    for M, N, K in ((16, 3072, 768), (16, 768, 3072), (16, 4096, 4096), (1, 4096, 4096)):
        g = torch.Generator(device=dev).manual_seed(M + N + K)
        ws = [(torch.randn(N, K, device=dev, generator=g) / K ** 0.5).half() for _ in range(n_layers)]
        xs = []
        for _ in range(n_layers):
            x = torch.randn(M, K, device=dev, generator=g).half()
            x[:, torch.randperm(K, device=dev, generator=g)[:K // 2]] = 0
            xs.append(x)
        ys = [torch.empty(M, N, device=dev, dtype=torch.float16) for _ in range(n_layers)]
        cnt = torch.empty(1, dtype=torch.int32, device=dev)

        def one(i):
            assert _native.dynamic_linear(xs[i], ws[i], 0.0, ys[i], count=cnt) == _native.GW_OK

        def four(i):
            _, buf, c = dead_neuron_mask_compact(xs[i], 0.0, want_mask=False)
            ghost_linear_dev(xs[i], pack_weight_dev(ws[i], buf, c), buf, c, out=ys[i])

        def dense(i):
            torch.mm(xs[i], ws[i].t(), out=ys[i])

        row = {"M": M, "N": N, "K": K}
        for name, f in (("single_launch_us", one), ("four_launches_us", four), ("cublas_dense_us", dense)):
            row[name] = round(graph_time(lambda: [f(i) for i in range(n_layers)], max(5, min(steps, 20)), 1)
                              / n_layers * 1e6, 2)
        one(0)
        ref = F.linear(xs[0].float(), ws[0].float())
        row["max_abs_err_vs_fp32"] = float((ys[0].float() - ref).abs().max())
        row["alive_count_ok"] = int(cnt.item()) == K - K // 2
        out.append(row)
        del ws, xs, ys
    torch.cuda.empty_cache()
    return {"what": "dynamic activation mask at decode size: one launch vs mask + pack + gather + GEMM "
                    "vs dense cuBLAS; graph replay of 16 layer calls", "rows": out,
            "note": "with a random dynamic mask every 16-byte vector of W holds alive columns, so any "
                    "sparse path reads all of W; dense cuBLAS reads it once at full speed"}


def run_ours(args, world, rank, local):
    from ghostweight_triton_b200 import GhostLinear

    device = torch.device("cuda", torch.cuda.current_device())
    peaks, peak_src = load_peaks()
    cfg = HEADLINE
    M, N, K = cfg["M"], cfg["N"], cfg["K"]
    layers = [build_layer(M, N, K, cfg["sparsity"], cfg["pattern"], torch.float16,
                          seed=1000 * rank + s, device=device) for s in range(N_SETS)]
    kp = layers[0]["idx"].numel()
    useful = 2.0 * M * N * kp

    from ghostweight_triton_b200 import _native

    # Product path (strategy "auto" with a workspace = "pregather"): the gather
    # launch writes x' = x[:, alive] to scratch, the tcgen05 GEMM launch streams
    # x' and W' by TMA (programmatic dependent launch overlaps its prologue with
    # the gather's tail). One scratch buffer serves every step in turn.
    ws = torch.empty(_native.gather_gemm_workspace_bytes(M, kp, torch.float16), dtype=torch.uint8,
                     device=device)
    ldp = (kp + 63) // 64 * 64
    xg = torch.empty(M, ldp, dtype=torch.float16, device=device)[:, :kp]   # x' for the kernels timed alone

    from ghostweight_triton_b200.kernels.matmul import ghost_linear_pipelined

    def step(i):
        # One step alone: the gather launch, then the PDL-chained GEMM launch
        # (or the single-launch overlap strategy).
        L = layers[i % N_SETS]
        _native.gather_gemm(L["x"], L["wp"], L["idx"], L["y"],
                            strategy="overlap" if args.strategy == "overlap" else "pregather", workspace=ws)

    def pipelined_steps(n):
        # n consecutive steps through ghost_linear_pipelined: step i+1's gather
        # runs on a low-priority stream under step i's GEMM.
        ghost_linear_pipelined([(L["x"], L["wp"], L["idx"], L["y"])
                                for L in (layers[i % N_SETS] for i in range(n))])

    def serial_steps(n):
        for i in range(n):
            step(i)

    # n consecutive steps, each a whole gather-GEMM of its own batch.
    run_steps = pipelined_steps if args.strategy == "pipelined" else serial_steps

    def step_overlap(i):
        L = layers[i % N_SETS]
        _native.gather_gemm(L["x"], L["wp"], L["idx"], L["y"], strategy="overlap", workspace=ws)

    def gemm_only(i):
        L = layers[i % N_SETS]
        _native.packed_gemm(xg, L["wp"], L["y"])

    def gather_only(i):
        L = layers[i % N_SETS]
        _native.gather_columns(L["x"], L["idx"], xg)

    # Warm-up, then a clock-sampled soak of ~1 s so the sampler sees the load,
    # then exactly `steps` timed steps (the sampler keeps running through them).
    run_steps(args.warmup)
    torch.cuda.synchronize()
    sampler = ClockSampler(physical_gpu_index(local)).start() if rank == 0 else None
    t_soak = time.perf_counter()
    n_soak = 0
    while not args.no_soak and time.perf_counter() - t_soak < 1.0:
        run_steps(200)
        n_soak += 200
        torch.cuda.synchronize()
    t = timed(lambda _: run_steps(args.steps), 1, world)
    clocks = sampler.stop() if sampler else None
    # The dominant kernel: the tcgen05 GEMM on the gathered operand, timed alone
    # (short windows, compared with the burst peak). For the breakdown also the
    # gather alone and the single-launch "overlap" variant (gather inside the
    # GEMM kernel).
    t_gemm = timed(gemm_only, args.steps, world) / args.steps
    t_gather = timed(gather_only, args.steps, world) / args.steps
    t_ovl = timed(step_overlap, args.steps, world) / args.steps
    # The same K steps one call at a time (gather launch + GEMM launch each)
    # against the pipelined steps under the same clocks: under the 1000 W cap
    # the SM clock follows the load within milliseconds, so each window of an
    # interleaved A/B follows a 0.3 s soak of its own kind, and the medians of
    # three rounds are reported.
    def soak_with(fn_n):
        t0 = time.perf_counter()
        while not args.no_soak and time.perf_counter() - t0 < 0.3:
            fn_n(50)
            torch.cuda.synchronize()

    ab = None
    if args.strategy in ("pipelined", "pregather"):
        ab_p, ab_s = [], []
        for _ in range(3):
            soak_with(pipelined_steps)
            ab_p.append(timed(lambda _: pipelined_steps(args.steps), 1, world) / args.steps)
            soak_with(serial_steps)
            ab_s.append(timed(step, args.steps, world) / args.steps)
        t_serial = sorted(ab_s)[1]
        ab = {"pipelined_us": round(sorted(ab_p)[1] * 1e6, 2), "one_call_at_a_time_us": round(t_serial * 1e6, 2),
              "pipelined_speedup": round(t_serial / sorted(ab_p)[1], 3), "rounds": 3,
              "soak_s_before_each_window": 0.0 if args.no_soak else 0.3,
              "note": ("at steady state under the 1000 W cap both modes do the same work for the "
                       "same energy; overlapping the gather with the GEMM adds contention for the "
                       "SMs, so one call at a time (the default) is as fast or faster there, while "
                       "pipelining gains in short bursts (graph-replayed sweeps, small batches)")}
    else:
        t_serial = timed(step, args.steps, world) / args.steps

    per_step = t / args.steps
    value = world * useful / per_step / 1e12

    achieved = useful / t_gemm / 1e12
    gather_bytes = M * K * 2 + M * kp * 2 + kp * 8       # full rows read (50% random touches every sector) + x' written
    # e2e through the public API: GhostLinear (frozen weight mask), pinned host x in, y out.
    e2e = None
    if not args.no_e2e:
        near = NearGpu(device.index).__enter__()
        gl = GhostLinear(K, N, bias=False, device=device, dtype=torch.float16)
        with torch.no_grad():
            gl.weight.copy_(layers[0]["w"])
        gl.freeze_weight_mask()
        hx = [L["x"].cpu().pin_memory() for L in layers]
        n_slots = 3
        hy = [torch.empty(M, N, dtype=torch.float16).pin_memory() for _ in range(n_slots)]
        layers_y0 = layers[0]["y"]
        # Three streams, three slots: the upload of step i+1 and the download of
        # step i-1 run while step i computes (PCIe carries both directions at
        # once). Events order each slot's reuse.
        comp = torch.cuda.current_stream()
        s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
        xd = [torch.empty(M, K, dtype=torch.float16, device=device) for _ in range(n_slots)]
        ev_in = [torch.cuda.Event() for _ in range(n_slots)]
        ev_comp = [torch.cuda.Event() for _ in range(n_slots)]
        ev_out = [torch.cuda.Event() for _ in range(n_slots)]
        for b in range(n_slots):
            ev_comp[b].record(comp)
            ev_out[b].record(comp)

        def e2e_step(i):
            b = i % n_slots
            # The host waits for slot b's previous download before queueing
            # this step: at most three steps are in flight, so the outputs that
            # wait for their downloads stay at three and the caching allocator
            # reaches its steady pool during warm-up (left unbounded, the host
            # runs many steps ahead and every step may need a new cudaMalloc).
            ev_out[b].synchronize()
            s_in.wait_event(ev_comp[b])                  # slot b's x no longer read
            with torch.cuda.stream(s_in):
                xd[b].copy_(hx[i % N_SETS], non_blocking=True)
                ev_in[b].record(s_in)
            comp.wait_event(ev_in[b])
            with torch.no_grad():
                yd = gl(xd[b])
            ev_comp[b].record(comp)
            s_out.wait_event(ev_comp[b])
            s_out.wait_event(ev_out[b])                  # slot b's host buffer downloaded before
            with torch.cuda.stream(s_out):
                hy[b].copy_(yd, non_blocking=True)
                yd.record_stream(s_out)
                ev_out[b].record(s_out)

        def e2e_timed(steps):
            barrier(world)
            torch.cuda.synchronize()
            st = torch.cuda.Event(enable_timing=True)
            en = torch.cuda.Event(enable_timing=True)
            st.record(comp)
            for i in range(steps):
                e2e_step(i)
            comp.wait_stream(s_out)
            en.record(comp)
            torch.cuda.synchronize()
            barrier(world)
            return max_over_ranks(st.elapsed_time(en) / 1e3, world)

        for i in range(max(8, args.warmup)):
            e2e_step(i)
        torch.cuda.synchronize()
        e_steps = max(1, min(args.steps, 200))
        te = e2e_timed(e_steps)
        # The link itself: one pinned 32 MiB upload and download, timed alone.
        t_h2d = event_time(lambda i: xd[0].copy_(hx[0], non_blocking=True), iters=10)
        t_d2h = event_time(lambda i: hy[0].copy_(layers_y0, non_blocking=True), iters=10)
        e2e = {"value": round(world * useful / (te / e_steps) / 1e12, 3), "unit": "TFLOP/s",
               "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2,
               "steps": e_steps, "ms_per_step": round(te / e_steps * 1e3, 4),
               "pcie_h2d_GBps": round(M * K * 2 / t_h2d / 1e9, 1),
               "pcie_d2h_GBps": round(M * N * 2 / t_d2h / 1e9, 1),
               "path": "GhostLinear.forward (frozen weight mask) with pinned-host x -> device -> pinned-host y; "
                       "upload, compute and download of consecutive steps overlap on three streams; "
                       "the host waits for a slot's previous download before reusing it (three slots, at most three steps in flight)",
               "host_cpus": near.describe()}
        near.__exit__()
        del hx, hy

    extra = {}
    cpu = None
    del layers
    torch.cuda.empty_cache()
    # The sharded MLP projection at this job's GPU count (every rank takes part).
    if not args.no_sharded:
        extra["sharded"] = sharded_record(args, world, rank, peaks, peak_src)
    if rank == 0 and world == 1:
        if not args.no_sweep:
            extra["sweep"] = sweep(device, peaks)
            extra["kernels"] = kernel_metrics(device, peaks)
        if not args.no_models:
            extra["models"] = {w: model_record(w, args.steps, args.warmup, world, rank, full=False)
                               for w in ("gpt2", "distilbert")}
            extra["dynamic_decode"] = dynamic_decode_record(args.steps)
        if not args.no_reference_triton:
            extra["reference_triton"] = reference_triton_record()
        if not args.no_cpu_baseline:
            r = cpu_reference_sample(M, N, K, cfg["sparsity"], cfg["pattern"], rows=256,
                                     budget_s=15.0, max_reps=50)
            cpu = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
            cpu["value"] = round(cpu["value"], 6)

    if rank == 0:
        peak = float(peaks["bf16_tflops"])
        traffic = traffic_from_profiles()
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step * 1e3, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic: x ~ N(0,1), W ~ N(0,1/sqrt(K)), 50% input columns zeroed (seeded uniform); random init",
            "config": {"workload": "gather-GEMM M=N=K=4096 fp16, 50% random dead input columns (K'=2048)",
                       "M": M, "N": N, "K": K, "K_alive": kp, "global_batch_rows": world * M,
                       "parallelism": f"independent batches per GPU x{world}",
                       "step": ("one gather + one GEMM launch per batch; consecutive batches through "
                                "ghost_linear_pipelined (batch i+1's gather under batch i's GEMM)"
                                if args.strategy == "pipelined" else "one gather_gemm call per batch"),
                       "l2": f"{N_SETS} rotating layer sets (x, W', y) = {N_SETS * 80} MB > 126 MB L2",
                       "soak_steps_before_timing": n_soak},
            "dense_equiv_tflops": round(world * 2.0 * M * N * K / per_step / 1e12, 3),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                         "peak_source": f"{peak_src} bf16_tflops burst (fp16 taken equal)",
                         "frac_of_sustained": (round(achieved / float(peaks["bf16_tflops_sustained"]), 4)
                                               if "bf16_tflops_sustained" in peaks else None),
                         "traffic": traffic,
                         "traffic_note": ("DRAM read + write of one launch from ncu; the window "
                                          "closes before y's write-back from L2 to DRAM, so it "
                                          "undercounts the algorithmic bytes and is not a "
                                          "traffic-efficiency figure"),
                         "kernel": "gemm_tc2_kernel<f16> (csrc/gw_gemm_tc2.cu: CTA pair, 256x256 tiles), timed alone"},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "clocks": clocks,
            "gpu_launches": (1 if args.strategy == "overlap" else 2) * args.steps,
            "step_kernels": {"step_us": round(per_step * 1e6, 2),
                             "gemm_on_gathered_operand_us": round(t_gemm * 1e6, 2),
                             "gemm_on_gathered_operand_tflops": round(useful / t_gemm / 1e12, 2),
                             "gather_alone_us": round(t_gather * 1e6, 2),
                             "gather_alone_GBps": round(gather_bytes / t_gather / 1e9, 1),
                             "gather_alone_frac_hbm": round(gather_bytes / t_gather / 1e9 / float(peaks["hbm_gbs"]), 3),
                             "single_launch_overlap_us": round(t_ovl * 1e6, 2),
                             "one_call_at_a_time_step_us": round(t_serial * 1e6, 2),
                             "one_call_at_a_time_tflops": round(world * useful / t_serial / 1e12, 2),
                             "pipelined_vs_one_call_at_a_time_same_clocks": ab},
            "strategy": {"pipelined": "pipelined (ghost_linear_pipelined: each step's gather launch on a "
                                      "low-priority stream under the previous step's GEMM launch, x' "
                                      "double-buffered; every step gathers and multiplies its own batch)",
                         "pregather": "pregather (gather launch + PDL-chained TMA tcgen05 GEMM launch)",
                         "overlap": "overlap (one launch: the pair GEMM's epilogue warps gather x' while "
                                    "its MMAs run)"}[args.strategy],
        }
        line.update(extra)
        print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- ours: sharded MLP
def sharded_parity(layer, x: torch.Tensor, y_full: torch.Tensor, rows: torch.Tensor, world: int) -> float:
    """How far sampled rows of a gathered [M, N] output are outside the output contract.

    Every rank computes the fp32 product of the sampled rows of x with its own
    weight rows, the blocks are all-gathered, and each rank compares the rows
    of its own full output with them: |y - r| <= 1e-2 + 1e-2 |r|, r the fp32
    product rounded to y's dtype. Returns the largest excess over all ranks
    (<= 0 passes).
    """
    n_real = layer.row_stop - layer.row_start
    ref_local = torch.zeros(rows.numel(), layer.n_local, dtype=torch.float32, device=x.device)
    ref_local[:, :n_real] = x[rows].float() @ layer.weight[:n_real].float().t()
    if layer.bias is not None:
        ref_local[:, :n_real] += layer.bias[:n_real].float()
    if world > 1:
        import torch.distributed as dist

        parts = torch.empty(world, rows.numel(), layer.n_local, dtype=torch.float32, device=x.device)
        dist.all_gather_into_tensor(parts, ref_local)
        ref = parts.permute(1, 0, 2).reshape(rows.numel(), world * layer.n_local)[:, :layer.out_features]
    else:
        ref = ref_local[:, :layer.out_features]
    r = ref.to(y_full.dtype).float()
    excess = ((y_full[rows].float() - r).abs() - (1e-2 + 1e-2 * r.abs())).max().item()
    return max_over_ranks(excess, world)


def sharded_record(args, world: int, rank: int, peaks: dict, peak_src: str) -> dict:
    """The sharded MLP projection, column-parallel over the job's GPUs.

    x [8192, 8192] bf16 ~ N(0, 1); W [28672, 8192] ~ N(0, 1/sqrt(K)) pre-sharded
    by output features (each rank draws only its rows) with 70% of the
    128-column blocks of input columns dead (seeded), K' = 2560. Times, max
    over ranks: the GEMM alone (this rank's columns), the full output on every
    rank through the GEMM whose epilogue stores each tile into all ranks'
    outputs over NVLink, and the same through NCCL all-gather + re-layout. The
    output of both full-output paths is checked in the run (sampled rows on
    every rank against the fp32 product, 1e-2 contract).
    """
    from ghostweight_triton_b200.sharded import ColumnParallelGhostLinear

    device = torch.device("cuda", torch.cuda.current_device())
    cfg = MLP
    M, N, K = cfg["M"], cfg["N"], cfg["K"]
    g = torch.Generator(device=device).manual_seed(5)          # the same x on every rank
    x = torch.randn(M, K, device=device, generator=g).to(torch.bfloat16)
    layer = ColumnParallelGhostLinear.from_full_weight_seed(
        N, K, seed=5, dead=dead_columns(K, cfg["sparsity"], 5, cfg["pattern"]),
        dtype=torch.bfloat16, device=device)
    kp = layer.k_alive
    useful = 2.0 * M * N * kp
    steps = max(1, args.steps)
    rows = torch.from_numpy(np.sort(np.random.default_rng(17).choice(M, 64, replace=False))).to(device)

    def step_gemm(i):
        layer.local_forward(x)

    def step_nccl(i):
        layer.gather_output = True
        return layer(x)

    def step_peers(i):
        layer.gather_output = "peers"
        return layer(x)

    for i in range(args.warmup):
        step_gemm(i)
        step_nccl(i)
        if world > 1:
            step_peers(i)
    t_gemm = timed(step_gemm, steps, world) / steps
    t_nccl = timed(step_nccl, steps, world) / steps
    t_peers = timed(step_peers, steps, world) / steps if world > 1 else None
    parity = {"rows_checked_per_rank": int(rows.numel()), "contract": "atol = rtol = 1e-2 vs fp32 rounded to bf16"}
    parity["nccl_max_excess"] = round(sharded_parity(layer, x, step_nccl(0), rows, world), 6)
    if world > 1:
        y = step_peers(0)
        parity["peers_max_excess"] = round(sharded_parity(layer, x, y, rows, world), 6)
    parity["ok"] = all(v <= 0.0 for k, v in parity.items() if k.endswith("_excess"))
    layer.close()
    strategy = layer.strategy
    del layer, x
    torch.cuda.empty_cache()

    t_full = min(t_nccl, t_peers) if t_peers is not None else t_nccl
    recv_bytes = (world - 1) / world * M * N * 2        # bytes of y each GPU receives
    t_flop = useful / world / (float(peaks["bf16_tflops"]) * 1e12)
    t_link = recv_bytes / 770e9
    bound = "nvlink" if t_link > t_flop else "tensor"
    return {
        "workload": "sharded MLP projection x[8192,8192] W[28672,8192] bf16, 70% dead 128-col blocks",
        "K_alive": kp, "n_gpus": world, "scaling": "strong", "strategy": strategy,
        "parallelism": f"column-parallel N over {world} GPU(s), full output on every rank",
        "gemm_only_ms": round(t_gemm * 1e3, 4),
        "gemm_only_tflops_per_gpu": round(useful / world / t_gemm / 1e12, 2),
        "gemm_only_frac_of_peak": round(useful / world / t_gemm / 1e12 / float(peaks["bf16_tflops"]), 4),
        "nccl_allgather_step_ms": round(t_nccl * 1e3, 4),
        "peer_fused_step_ms": round(t_peers * 1e3, 4) if t_peers is not None else None,
        "full_output_step_ms": round(t_full * 1e3, 4),
        "full_output_tflops": round(useful / t_full / 1e12, 2),
        "full_output_tflops_per_gpu": round(useful / world / t_full / 1e12, 2),
        "bytes_received_per_gpu": int(recv_bytes),
        "step_bound": bound,
        "frac_of_step_bound": round(max(t_link, t_flop) / t_full, 4),
        "link_bound_note": "slower of tensor work per GPU (measured bf16 peak) and (world-1)/world of y "
                           "received per GPU at the measured 770 GB/s peer copy",
        "gathered_by": ("GEMM epilogue peer stores over NVLink (CUDA IPC)"
                        if t_peers is not None and t_peers <= t_nccl else
                        ("NCCL all-gather + re-layout" if world > 1 else "nothing to gather (one GPU)")),
        "parity": parity, "peak_source": peak_src,
    }


def run_mlp_sharded(args, world, rank, local):
    peaks, peak_src = load_peaks()
    rec = sharded_record(args, world, rank, peaks, peak_src)
    if rank == 0:
        per = rec["full_output_step_ms"] * 1e-3
        line = {
            "metric": METRIC, "value": rec["full_output_tflops"], "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": rec["full_output_step_ms"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic, seeded",
            "config": {"workload": rec["workload"], "K_alive": rec["K_alive"],
                       "parallelism": rec["parallelism"], "strategy": rec["strategy"]},
            "sharded": rec,
            "roofline": {"bound": rec["step_bound"], "frac": rec["frac_of_step_bound"],
                         "achieved": rec["full_output_tflops_per_gpu"], "unit": "TFLOP/s per GPU",
                         "peak": float(peaks["bf16_tflops"]), "traffic": None,
                         "peak_source": f"{peak_src} bf16_tflops; link bound 770 GB/s"},
            "gpu_launches": (1 if rec["strategy"] == "runs" else 2) * args.steps,
            "ms_per_step_note": f"full output on every rank, {per * 1e3:.4f} ms",
        }
        print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- decoding (small M)
DECODE_LAYERS = 16
SMALL_BATCH_ROWS = (64, 128, 256, 512)


def run_decode(args, world, rank, local):
    """Decoding through a stack of 4096 x 4096 fp16 layers, a few rows at a time.

    16 layers, each W [4096, 4096] ~ N(0, 1/sqrt(K)) with 50% of its input
    columns zeroed (seeded uniform), K' = 2048, packed once (16 x 16.8 MB of
    packed weights > 126 MB L2, so every step streams its weight from HBM).
    Step = one layer's gather-GEMM on x [M, 4096] through the product path
    (ghost_linear, frozen alive list): for M = 16 the gather launch and the
    decode GEMM, for M = 1 the decode GEMM gathering x itself. The 16 layer
    calls are captured in one CUDA graph and replayed (launch-bound sizes).
    """
    import torch.nn.functional as F

    from ghostweight_triton_b200 import GhostLinear, _native
    from ghostweight_triton_b200.kernels.matmul import ghost_linear

    device = torch.device("cuda", torch.cuda.current_device())
    peaks, peak_src = load_peaks()
    K = N = 4096
    g = torch.Generator(device=device).manual_seed(11 + rank)
    layers = []
    for i in range(DECODE_LAYERS):
        dead = torch.from_numpy(dead_columns(K, 0.5, 100 + i, "random")).to(device)
        lin = GhostLinear(K, N, bias=False, threshold=0.0, device=device, dtype=torch.float16)
        with torch.no_grad():
            lin.weight.normal_(0.0, K ** -0.5, generator=g)
            lin.weight[:, dead] = 0
        lin.freeze_weight_mask()
        layers.append(lin)
    kp = int(layers[0]._frozen_indices.numel())
    packed = [lin._weight_packed(lin._frozen_indices, torch.float16) for lin in layers]

    def layer_time(M: int, fn_for):
        xs = [torch.randn(M, K, device=device, generator=g).half() for _ in range(DECODE_LAYERS)]
        ys = [torch.empty(M, N, device=device, dtype=torch.float16) for _ in range(DECODE_LAYERS)]
        fns = [fn_for(i, xs[i], ys[i]) for i in range(DECODE_LAYERS)]

        def all_layers():
            for f in fns:
                f()
        reps = max(10, min(args.steps, 50))
        return graph_time(all_layers, reps, world) / DECODE_LAYERS, xs, ys

    res = {}
    for M in (16, 1):
        t, xs, ys = layer_time(M, lambda i, x, y: (lambda: ghost_linear(
            x, packed[i], layers[i]._frozen_indices, out=y)))
        err = float((ys[0].float() - F.linear(xs[0].float(), layers[0].weight.detach().float())).abs().max().item())
        dense_w = [lin.weight.detach() for lin in layers]
        td, _, _ = layer_time(M, lambda i, x, y: (lambda: torch.mm(x, dense_w[i].t(), out=y)))
        res[M] = (t, td, err)
    # The decode GEMM alone on a pre-gathered x' (its roofline: W' from HBM).
    xg = [torch.randn(16, kp, device=device, generator=g).half() for _ in range(DECODE_LAYERS)]
    yg = [torch.empty(16, N, device=device, dtype=torch.float16) for _ in range(DECODE_LAYERS)]

    def gemm_all():
        for i in range(DECODE_LAYERS):
            _native.packed_gemm(xg[i], packed[i], yg[i])
    reps = max(10, min(args.steps, 50))
    t_gemm = graph_time(gemm_all, reps, world) / DECODE_LAYERS
    w_bytes = N * kp * 2
    alg_bytes = w_bytes + 16 * kp * 2 + 16 * N * 2
    # End to end through GhostLinear.forward: x from pinned host memory, y back.
    hx = [torch.randn(16, K).half().pin_memory() for _ in range(DECODE_LAYERS)]
    hy = torch.empty(16, N, dtype=torch.float16).pin_memory()

    def e2e_step(i):
        with torch.no_grad():
            hy.copy_(layers[i % DECODE_LAYERS](hx[i % DECODE_LAYERS].to(device, non_blocking=True)),
                     non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    te = timed(e2e_step, args.steps, world) / args.steps
    if rank == 0:
        t16, td16, err16 = res[16]
        t1, td1, err1 = res[1]
        cpu = cpu_decode_sample(kp)
        line = {
            "metric": "decode gather-GEMM time per layer (M=16 rows, 4096x4096 fp16, 50% dead)",
            "value": round(t16 * 1e6, 3), "unit": "us", "n_gpus": world, "steps": reps,
            "warmup": args.warmup, "ms_per_step": round(t16 * 1e3, 5), "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic: x ~ N(0,1), W ~ N(0,1/sqrt(K)), 50% input columns zeroed (seeded uniform)",
            "config": {"workload": "decode: 16 rotating 4096x4096 fp16 layers (K'=2048), M=16 rows per step",
                       "M": 16, "N": N, "K": K, "K_alive": kp,
                       "l2": "16 layers x 16.8 MB packed weights = 268 MB > 126 MB L2",
                       "timing": "CUDA graph of 16 layer calls, replayed"},
            "cublas_dense_us": round(td16 * 1e6, 3), "speedup_vs_dense": round(td16 / t16, 3),
            "ideal_speedup": round(K / kp, 3), "max_abs_err_vs_fp32": err16,
            "m1": {"us": round(t1 * 1e6, 3), "cublas_dense_us": round(td1 * 1e6, 3),
                   "speedup_vs_dense": round(td1 / t1, 3), "max_abs_err_vs_fp32": err1,
                   "path": "one launch: the decode GEMM gathers x[:, alive] itself"},
            "roofline": {"bound": "hbm", "achieved": round(alg_bytes / t_gemm / 1e9, 1),
                         "peak": float(peaks["hbm_gbs"]), "unit": "GB/s",
                         "frac": round(alg_bytes / t_gemm / 1e9 / float(peaks["hbm_gbs"]), 4),
                         "traffic": 16871424.0, "peak_source": f"{peak_src} hbm_gbs",
                         "kernel": "gemm_decode_kernel<16> on x' (csrc/gw_gemm_decode.cu), graph replay",
                         "us": round(t_gemm * 1e6, 3)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(te * 1e6, 3), "unit": "us", "h2d_bytes_per_step": 16 * K * 2,
                    "d2h_bytes_per_step": 16 * N * 2, "path": "GhostLinear.forward, pinned host x and y"},
            "gpu_launches": 2 * reps * DECODE_LAYERS,
        }
        print(json.dumps(line), flush=True)


def run_small_batch(args, world, rank, local):
    """Small batches (64 to 512 rows) through 4096 x 4096 fp16 layers at 50% dead.

    The range between the decode kernel (at most 32 rows) and the CTA-pair
    kernel, where the output has too few tiles for the SMs and the GEMM is the
    cluster split-K kernel. 8 layers, each W [4096, 4096] ~ N(0, 1/sqrt(K)) with
    50% of its input columns zeroed (seeded uniform), K' = 2048, packed once
    (8 x 16.8 MB of packed weights > 126 MB L2). Step = one layer's gather-GEMM
    through the product path (ghost_linear, frozen alive list: the gather launch
    and the GEMM launch) on the next layer; the 8 layer calls are captured in one
    CUDA graph and replayed. Headline: M = 256.
    """
    import torch.nn.functional as F

    from ghostweight_triton_b200 import GhostLinear, _native
    from ghostweight_triton_b200.kernels.matmul import ghost_linear, ghost_linear_pipelined

    device = torch.device("cuda", torch.cuda.current_device())
    peaks, peak_src = load_peaks()
    K = N = 4096
    n_layers = 8
    g = torch.Generator(device=device).manual_seed(13 + rank)
    layers = []
    for i in range(n_layers):
        dead = torch.from_numpy(dead_columns(K, 0.5, 200 + i, "random")).to(device)
        lin = GhostLinear(K, N, bias=False, threshold=0.0, device=device, dtype=torch.float16)
        with torch.no_grad():
            lin.weight.normal_(0.0, K ** -0.5, generator=g)
            lin.weight[:, dead] = 0
        lin.freeze_weight_mask()
        layers.append(lin)
    kp = int(layers[0]._frozen_indices.numel())
    packed = [lin._weight_packed(lin._frozen_indices, torch.float16) for lin in layers]
    dense_w = [lin.weight.detach() for lin in layers]
    reps = max(10, min(args.steps, 50))

    def per_layer(fn_for, xs, ys):
        fns = [fn_for(i, xs[i], ys[i]) for i in range(n_layers)]

        def all_layers():
            for f in fns:
                f()
        return graph_time(all_layers, reps, world) / n_layers

    ms = tuple(args.rows) if args.rows else SMALL_BATCH_ROWS
    rows = {}
    for M in ms:
        xs = [torch.randn(M, K, device=device, generator=g).half() for _ in range(n_layers)]
        ys = [torch.empty(M, N, device=device, dtype=torch.float16) for _ in range(n_layers)]
        t = per_layer(lambda i, x, y: (lambda: ghost_linear(x, packed[i], layers[i]._frozen_indices, out=y)),
                      xs, ys)
        err = float((ys[0].float() - F.linear(xs[0].float(), dense_w[0].float())).abs().max().item())
        xg = [torch.randn(M, kp, device=device, generator=g).half() for _ in range(n_layers)]
        tg = per_layer(lambda i, x, y: (lambda: _native.packed_gemm(x, packed[i], y)), xg, ys)
        td = per_layer(lambda i, x, y: (lambda: torch.mm(x, dense_w[i].t(), out=y)), xs, ys)
        # The 8 layer calls as independent batches: each gather runs under the
        # previous layer's GEMM (ghost_linear_pipelined), one graph.
        pcalls = [(xs[i], packed[i], layers[i]._frozen_indices, ys[i]) for i in range(n_layers)]
        tp = graph_time(lambda: ghost_linear_pipelined(pcalls), reps, world) / n_layers
        kernel, tile_n, split = _native.gemm_plan(M, N, kp)
        rows[M] = {"M": M, "us": round(t * 1e6, 3), "useful_tflops": round(2.0 * M * N * kp / t / 1e12, 2),
                   "gemm_us": round(tg * 1e6, 3), "cublas_dense_us": round(td * 1e6, 3),
                   "speedup_vs_dense": round(td / t, 3), "gemm_speedup_vs_dense": round(td / tg, 3),
                   "pipelined_us": round(tp * 1e6, 3), "pipelined_speedup_vs_dense": round(td / tp, 3),
                   "plan": {"kernel": kernel, "tile_n": tile_n, "split": split},
                   "max_abs_err_vs_fp32": err}
        del xs, ys, xg, pcalls
    M = 256 if 256 in rows else ms[0]
    hx = [torch.randn(M, K).half().pin_memory() for _ in range(n_layers)]
    hy = torch.empty(M, N, dtype=torch.float16).pin_memory()

    def e2e_step(i):
        with torch.no_grad():
            hy.copy_(layers[i % n_layers](hx[i % n_layers].to(device, non_blocking=True)), non_blocking=True)

    te = None
    if not args.no_e2e:
        for i in range(args.warmup):
            e2e_step(i)
        te = timed(e2e_step, args.steps, world) / args.steps
    if rank == 0:
        r = rows[M]
        t = r["us"] * 1e-6
        useful = 2.0 * M * N * kp
        tg = r["gemm_us"] * 1e-6
        line = {
            "metric": f"useful TFLOP/s of the gather-GEMM at {M} rows (2*M*N*K'), 4096x4096 fp16, 50% dead",
            "value": round(useful / t / 1e12, 3), "unit": "TFLOP/s", "n_gpus": world, "steps": reps,
            "warmup": args.warmup, "ms_per_step": round(t * 1e3, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic: x ~ N(0,1), W ~ N(0,1/sqrt(K)), 50% input columns zeroed (seeded uniform)",
            "config": {"workload": "small batches: 8 rotating 4096x4096 fp16 layers (K'=2048), M=64..512 rows",
                       "M": M, "N": N, "K": K, "K_alive": kp,
                       "l2": "8 layers x 16.8 MB packed weights = 134 MB > 126 MB L2",
                       "timing": "CUDA graph of 8 layer calls, replayed"},
            "rows": [rows[m] for m in ms],
            "roofline": {"bound": "tensor", "achieved": round(useful / tg / 1e12, 1),
                         "peak": float(peaks["bf16_tflops"]), "unit": "TFLOP/s",
                         "frac": round(useful / tg / 1e12 / float(peaks["bf16_tflops"]), 4), "traffic": None,
                         "peak_source": f"{peak_src} bf16_tflops", "us": r["gemm_us"],
                         "kernel": "gemm_splitk_kernel on x' (csrc/gw_gemm_splitk.cu), graph replay"},
            "cpu_baseline": None if args.no_cpu_baseline else cpu_decode_sample(kp, rows=64),
            "e2e": None if te is None else {
                "value": round(useful / te / 1e12, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": M * K * 2,
                "d2h_bytes_per_step": M * N * 2, "path": "GhostLinear.forward, pinned host x and y"},
            "gpu_launches": 2 * reps * n_layers,
        }
        print(json.dumps(line), flush=True)


def cpu_decode_sample(kp: int, rows: int = 16) -> dict:
    """The oracle's restatement of the reference path for one layer call of `rows` rows."""
    sys.path.insert(0, str(REPO))
    from oracle import gw_oracle as O

    rng = np.random.default_rng(5)
    K = N = 4096
    x = rng.standard_normal((rows, K)).astype(np.float16)
    w = (rng.standard_normal((K, N)) / 64).astype(np.float16)
    idx = np.sort(rng.permutation(K)[:kp]).astype(np.int64)
    O.ghostweight_matmul(x, w, idx)
    ts = []
    for _ in range(20):
        t0 = time.perf_counter()
        O.ghostweight_matmul(x, w, idx)
        ts.append(time.perf_counter() - t0)
    t = float(np.median(ts))
    if rows == 16:
        return {"value": round(t * 1e6, 1), "unit": "us", "cores": os.cpu_count(),
                "kind": "port", "sample": "one 16-row 4096x4096 layer call (K'=2048) through "
                                          "oracle.ghostweight_matmul, median of 20"}
    return {"value": round(2.0 * rows * N * kp / t / 1e12, 5), "unit": "TFLOP/s", "cores": os.cpu_count(),
            "kind": "port", "sample": f"one {rows}-row 4096x4096 layer call (K'={kp}) through "
                                      "oracle.ghostweight_matmul, median of 20"}


# ---------------------------------------------------------------------------- config 1: fp32 GhostLinear
def run_fp32_linear(args, world, rank, local):
    """Single GhostLinear fp32 through the reference's default (dynamic) path.

    X [8, 128, 768] ~ N(0,1), W [3072, 768] ~ N(0, 0.02), bias ~ N(0, 0.02); 384
    seeded-random input columns zeroed in W and in X, threshold 0, so the
    per-forward activation mask (mask kernel -> alive list) finds exactly the
    zeroed columns. Step = one GhostLinear.forward: mask + compaction + weight
    packing + exact-fp32 gather-GEMM + bias.
    """
    from ghostweight_triton_b200 import GhostLinear

    device = torch.device("cuda", torch.cuda.current_device())
    B, T, K, N = 8, 128, 768, 3072
    g = torch.Generator(device=device).manual_seed(1 + rank)
    dead = torch.from_numpy(dead_columns(K, 0.5, 1, "random")).to(device)
    layer = GhostLinear(K, N, bias=True, threshold=0.0, device=device, dtype=torch.float32)
    with torch.no_grad():
        layer.weight.normal_(0.0, 0.02, generator=g)
        layer.bias.normal_(0.0, 0.02, generator=g)
        layer.weight[:, dead] = 0
    xs = []
    for s in range(N_SETS):
        x = torch.randn(B, T, K, device=device, generator=g)
        x[..., dead] = 0
        xs.append(x)
    kp = K - dead.numel()
    useful = 2.0 * B * T * N * kp

    def step(i):
        with torch.no_grad():
            layer(xs[i % N_SETS])

    for i in range(args.warmup):
        step(i)
    t = timed(step, args.steps, world)
    per = t / args.steps
    with torch.no_grad():
        y = layer(xs[0])
        ref = torch.nn.functional.linear(xs[0].double(), layer.weight.double(), layer.bias.double())
        err = float((y.double() - ref).abs().max().item())
    # The same forward with the mask frozen (alive list and packed weight reused).
    layer.freeze_mask(xs[0])
    t_frozen = timed(step, args.steps, world) / args.steps
    hx = [x.cpu().pin_memory() for x in xs]
    hy = torch.empty(B, T, N).pin_memory()

    def e2e_step(i):
        with torch.no_grad():
            hy.copy_(layer(hx[i % N_SETS].to(device, non_blocking=True)), non_blocking=True)

    for i in range(3):
        e2e_step(i)
    te = timed(e2e_step, args.steps, world) / args.steps
    if rank == 0:
        cpu = cpu_linear_fp32(dead.cpu().numpy(), B * T, K, N)
        line = {
            "metric": "useful TFLOP/s of GhostLinear.forward fp32 (2*M*N*K')",
            "value": round(world * useful / per / 1e12, 4), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per * 1e3, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic: X ~ N(0,1), W, b ~ N(0,0.02), 384 of 768 input columns zeroed (seeded)",
            "config": {"workload": "single GhostLinear fp32, X [8,128,768], W [3072,768], 50% dead, dynamic mask",
                       "M": B * T, "N": N, "K": K, "K_alive": kp, "threshold": 0.0,
                       "l2": "inputs 3 MB: L2-resident"},
            "frozen_mask_ms_per_step": round(t_frozen * 1e3, 4),
            "frozen_mask_tflops": round(world * useful / t_frozen / 1e12, 4),
            "max_abs_err_vs_fp64": err,
            "cpu_baseline": cpu,
            "e2e": {"value": round(world * useful / te / 1e12, 4), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": B * T * K * 4, "d2h_bytes_per_step": B * T * N * 4,
                    "ms_per_step": round(te * 1e3, 4)},
            "gpu_launches": 5 * args.steps,
        }
        print(json.dumps(line), flush=True)


def cpu_linear_fp32(dead: np.ndarray, M: int, K: int, N: int) -> dict:
    """The reference's CPU path for config 1 (mask from |x|, x[:, alive] @ W[alive].T + b) on all cores."""
    from oracle import gw_oracle as O

    rng = np.random.default_rng(1)
    x = rng.standard_normal((M, K), dtype=np.float32)
    x[:, dead] = 0
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02)
    w[:, dead] = 0
    b = (rng.standard_normal(N, dtype=np.float32) * 0.02)
    idx = O.alive_indices(O.dead_neuron_mask(x, 0.0))
    times = []
    for _ in range(8):
        t0 = time.perf_counter()
        idx = O.alive_indices(O.dead_neuron_mask(x, 0.0))
        y = x[:, idx] @ w[:, idx].T + b
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": round(2.0 * M * N * len(idx) / t / 1e12, 6), "unit": "TFLOP/s",
            "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"the whole config ({M} rows): oracle mask + numpy fp32 gather-GEMM + bias, median of 8"}


# ---------------------------------------------------------------------------- configs 3, 4: models
MODELS = {
    "gpt2": dict(batch=8, seq=512, sparsity=0.5, vocab=50257,
                 desc="GPT-2 small random init (12 layers, d 768, 12 heads, MLP 3072), fp16 prefill "
                      "batch 8 x seq 512; all 48 Conv1D rewritten; 50% dead input columns per layer"),
    "distilbert": dict(batch=64, seq=128, sparsity=0.6, vocab=30522,
                       desc="DistilBERT-base random init (6 layers, d 768, 12 heads, FFN 3072), fp16 "
                            "encoder batch 64 x seq 128; all 36 linears rewritten; 60% dead input columns"),
}


def build_model(which: str, device, seed: int = 0):
    """Random-init model in fp16 on `device` with each projection's dead input columns zeroed."""
    import torch.nn as nn

    torch.manual_seed(seed)
    if which == "gpt2":
        from transformers import GPT2Config, GPT2Model
        model = GPT2Model(GPT2Config())
    else:
        from transformers import DistilBertConfig, DistilBertModel
        model = DistilBertModel(DistilBertConfig())
    from transformers.pytorch_utils import Conv1D

    sp = MODELS[which]["sparsity"]
    rng = np.random.default_rng(seed + 17)
    with torch.no_grad():
        for mod in model.modules():
            if isinstance(mod, nn.Linear) and mod.in_features >= 128:
                k = mod.in_features
                dead = torch.from_numpy(np.sort(rng.permutation(k)[:int(k * sp)]))
                mod.weight[:, dead] = 0
            elif isinstance(mod, Conv1D):
                k = mod.weight.shape[0]
                dead = torch.from_numpy(np.sort(rng.permutation(k)[:int(k * sp)]))
                mod.weight[dead, :] = 0
    return model.half().to(device).eval()


def model_record(which: str, steps: int, warmup: int, world: int, rank: int, full: bool = True) -> dict:
    """Tokens/s of the random-init model with every projection rewritten, next to the dense model.

    Drop-in (``replace_linears``, masks frozen from the weights), eager and
    replayed from a CUDA graph, and with the MLP blocks fused
    (``fuse_mlp_chains``), against the same dense fp16 model on the same GPU;
    relative error of the final hidden state against the dense model. With
    full=True also the end-to-end forward with token ids from pinned host
    memory and the hidden state copied back.
    """
    import copy

    from ghostweight_triton_b200 import replace_linears
    from ghostweight_triton_b200.fuse import fuse_mlp_chains

    device = torch.device("cuda", torch.cuda.current_device())
    cfg = MODELS[which]
    dense = build_model(which, device)
    ghost = copy.deepcopy(dense)
    replaced = replace_linears(ghost, threshold=0.0, include_conv1d=True, freeze_from_weight=True)
    tokens = cfg["batch"] * cfg["seq"]
    g = torch.Generator(device=device).manual_seed(3 + rank)
    ids = [torch.randint(0, cfg["vocab"], (cfg["batch"], cfg["seq"]), device=device, generator=g)
           for _ in range(2)]
    kwargs = {}
    if which == "distilbert":
        kwargs["attention_mask"] = torch.ones(cfg["batch"], cfg["seq"], dtype=torch.long, device=device)

    def fwd(model, i):
        with torch.no_grad():
            return model(input_ids=ids[i % 2], **kwargs).last_hidden_state

    for i in range(warmup):
        fwd(ghost, i)
        fwd(dense, i)
    steps = max(1, min(steps, 50))
    t = timed(lambda i: fwd(ghost, i), steps, world) / steps
    t_dense = timed(lambda i: fwd(dense, i), steps, world) / steps
    with torch.no_grad():
        ref = fwd(dense, 0).float()
        rel = float(((fwd(ghost, 0).float() - ref).norm() / ref.norm()).item())
    # The same forwards captured in CUDA graphs: no per-call host overhead.
    t_graph = graph_time(lambda: fwd(ghost, 0), steps, world)
    t_graph_dense = graph_time(lambda: fwd(dense, 0), steps, world)
    # MLP blocks fused (the first projection computes only the second's alive
    # features, written compacted; no gather before the second).
    fused = copy.deepcopy(ghost)
    n_fused = len(fuse_mlp_chains(fused))
    for i in range(warmup):
        fwd(fused, i)
    t_graph_fused = graph_time(lambda: fwd(fused, 0), steps, world)
    with torch.no_grad():
        rel_fused = float(((fwd(fused, 0).float() - ref).norm() / ref.norm()).item())
    del fused
    # Linear-layer FLOPs of one forward over the alive columns (what the kernels compute).
    useful = 0.0
    for mod in ghost.modules():
        if mod.__class__.__name__ == "GhostLinear" and mod.mask_frozen:
            useful += 2.0 * tokens * mod.out_features * mod._frozen_indices.numel()
    rec = {
        "metric": f"{which} {'prefill' if which == 'gpt2' else 'encoder'} tokens/s",
        "workload": cfg["desc"], "tokens_per_step": tokens, "layers_replaced": len(replaced),
        "tokens_per_s": round(world * tokens / t, 1), "ms_per_step": round(t * 1e3, 4),
        "dense_tokens_per_s": round(world * tokens / t_dense, 1),
        "speedup_vs_dense": round(t_dense / t, 3),
        "cuda_graph": {"tokens_per_s": round(world * tokens / t_graph, 1),
                       "dense_tokens_per_s": round(world * tokens / t_graph_dense, 1),
                       "speedup_vs_dense": round(t_graph_dense / t_graph, 3),
                       "ms_per_step": round(t_graph * 1e3, 4)},
        "mlp_chains_fused": {"blocks": n_fused, "tokens_per_s": round(world * tokens / t_graph_fused, 1),
                             "speedup_vs_dense": round(t_graph_dense / t_graph_fused, 3),
                             "ms_per_step": round(t_graph_fused * 1e3, 4),
                             "rel_err_vs_dense_model": rel_fused, "timing": "CUDA graph, as cuda_graph"},
        "linear_useful_tflops": round(useful / t / 1e12, 2),
        "rel_err_vs_dense_model": rel,
        "steps": steps,
        # Each frozen GhostLinear forward: the x' gather and the GEMM (or the GEMM alone).
        "gpu_launches_per_step_at_most": 2 * len(replaced),
    }
    if full:
        hids = [x.cpu().pin_memory() for x in ids]
        hout = torch.empty(cfg["batch"], cfg["seq"], 768, dtype=torch.float16).pin_memory()

        def e2e_step(i):
            with torch.no_grad():
                out = ghost(input_ids=hids[i % 2].to(device, non_blocking=True), **kwargs).last_hidden_state
            hout.copy_(out, non_blocking=True)

        for i in range(2):
            e2e_step(i)
        te = timed(e2e_step, steps, world) / steps
        rec["e2e"] = {"value": round(world * tokens / te, 1), "unit": "tokens/s",
                      "h2d_bytes_per_step": tokens * 8, "d2h_bytes_per_step": tokens * 768 * 2,
                      "ms_per_step": round(te * 1e3, 4)}
    del ghost, dense
    torch.cuda.empty_cache()
    return rec


def run_model(args, world, rank, local, which: str):
    rec = model_record(which, args.steps, args.warmup, world, rank, full=True)
    if rank == 0:
        cpu = cpu_model_sample(which)
        line = {
            "metric": rec["metric"], "value": rec["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
            "steps": rec["steps"], "warmup": args.warmup, "ms_per_step": rec["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic: random-init weights, token ids uniform in [0, vocab)",
            "config": {"workload": rec["workload"], "tokens_per_step": rec["tokens_per_step"],
                       "layers_replaced": rec["layers_replaced"], "parallelism": f"independent batches x{world}"},
            "cpu_baseline": cpu, "e2e": rec["e2e"],
            "gpu_launches": rec["gpu_launches_per_step_at_most"] * rec["steps"],
            **{k: v for k, v in rec.items() if k not in ("e2e", "metric", "workload", "steps")},
        }
        print(json.dumps(line), flush=True)


def graph_time(fn, steps: int, world: int) -> float:
    """Seconds per call of fn() replayed from a CUDA graph (CUDA events, max over ranks)."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    graph.replay()
    t = timed(lambda i: graph.replay(), steps, world) / steps
    del graph
    return t


def cpu_model_sample(which: str) -> dict:
    """The reference's CPU path for the model (dense PyTorch fp32; its kernels have no CPU path)."""
    cfg = MODELS[which]
    model = build_model(which, torch.device("cpu")).float()
    torch.set_num_threads(os.cpu_count() or 1)
    seq = cfg["seq"]
    ids = torch.randint(0, cfg["vocab"], (1, seq))
    kwargs = {"attention_mask": torch.ones(1, seq, dtype=torch.long)} if which == "distilbert" else {}
    with torch.no_grad():
        model(input_ids=ids, **kwargs)
        times = []
        for _ in range(3):
            t0 = time.perf_counter()
            model(input_ids=ids, **kwargs)
            times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": round(seq / t, 1), "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"one sequence of {seq} tokens through the dense fp32 model "
                                      f"(PyTorch CPU), median of 3"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["gemm", "mlp-sharded", "ghostlinear-fp32", "gpt2", "distilbert",
                                           "decode", "small-batch", "dynamic-decode"],
                    default="gemm")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--rows", type=int, nargs="+", default=None,
                    help="small-batch workload: the row counts to run (default 64 128 256 512)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-soak", action="store_true",
                    help="skip the 1 s clock-sampling soak (for short profiler runs)")
    ap.add_argument("--no-sharded", action="store_true", help="skip the sharded MLP sub-record")
    ap.add_argument("--no-models", action="store_true", help="skip the GPT-2 / DistilBERT sub-record")
    ap.add_argument("--no-reference-triton", action="store_true",
                    help="skip timing the reference's Triton kernels")
    ap.add_argument("--reference-triton-child", metavar="DIR", default=None, help=argparse.SUPPRESS)
    ap.add_argument("--strategy", choices=["pipelined", "pregather", "overlap"], default="pregather",
                    help="gemm workload: pregather / overlap = one gather_gemm call per step with "
                         "that strategy (pregather, the default, measured fastest at steady state); "
                         "pipelined = consecutive steps through ghost_linear_pipelined (each step's "
                         "gather under the previous step's GEMM)")
    args = ap.parse_args()
    if args.reference_triton_child:
        reference_triton_child(args.reference_triton_child)
        return
    args.warmup = max(3, args.warmup)
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.workload == "gemm":
            run_ours(args, world, rank, local)
        elif args.workload == "mlp-sharded":
            run_mlp_sharded(args, world, rank, local)
        elif args.workload == "ghostlinear-fp32":
            run_fp32_linear(args, world, rank, local)
        elif args.workload == "decode":
            run_decode(args, world, rank, local)
        elif args.workload == "small-batch":
            run_small_batch(args, world, rank, local)
        elif args.workload == "dynamic-decode":
            rec = dynamic_decode_record(args.steps)
            if rank == 0:
                r = rec["rows"][0]
                print(json.dumps({
                    "metric": "dynamic-mask layer call time (M=16, 768 -> 3072 fp16, 50% of x's columns zero)",
                    "value": r["single_launch_us"], "unit": "us", "n_gpus": world, "steps": args.steps,
                    "warmup": args.warmup, "ms_per_step": round(r["single_launch_us"] / 1e3, 5),
                    "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
                    "data": "synthetic, seeded", "config": {"workload": "dynamic decode, 16 rows per call"},
                    "dynamic_decode": rec, "gpu_launches": 16}), flush=True)
        else:
            run_model(args, world, rank, local, args.workload)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
