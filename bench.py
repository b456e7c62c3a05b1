#!/usr/bin/env python
"""Benchmark of the tree-ensemble batch predict on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

A step is one predict pass over one batch of the configuration's synthetic
rows (default c2: XGBoost-style binary GBDT, 500 complete depth-8 trees, 128
float64 features with 5% NaN, 1,000,000 rows; model seed 0, data seed 1).
Every rank predicts its own batch on its own GPU (weak scaling, no collective
on the data path); timing uses CUDA events on the launching stream between a
barrier + synchronize on both sides, max over ranks. Rank 0 prints one JSON
line:

  value      rows/s of all ranks, inputs resident in HBM (montlok_model_predict_device)
  e2e        rows/s through montlok_model_predict with pinned host buffers:
             host->device input, kernel, device->host output every step
  roofline   the predict kernel's HBM rate on its input bytes (rows x F x 8)
             against the measured copy bandwidth (MEASURED_PEAKS.json), with
             the DRAM traffic, issue and shared-memory utilisation of the
             committed ncu capture of the same kernel (profiles/)
  cpu_baseline  the reference runtime (oracle/_ref, compiled from its sources)
             on this host's cores, on a bounded sample of the same workload
  configs    (one GPU, default c2 run) the same figures for c1, c3 and c4 at
             their configured batches, and c5's per-call latency
  sharded    (rank 0) one host-buffer call of the same batch split over all N
             GPUs by the library itself (montlok_set_devices), strong scaling

``--impl reference`` times the reference's CPU implementation alone, with all
host threads, on the same workload (the full batch every step) and prints the
same line. It imports only the pure-Python model builders of the package and
the reference library: libmontlok.so is not loaded in that process.

``--config c5`` is the latency configuration: calls of 1, 8 and 64 rows
back to back through montlok_model_predict (host buffers; the library
replays a cached CUDA graph per call shape), timed per call inside the
library; the line reports p50/p99 microseconds per call size, the value being
the p50 of the 64-row calls, with the reference's own per-call latency on the
host cores beside it.
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
for _p in (ROOT / "montlok.cpp_b200" / "python", ROOT / "oracle"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import numpy as np  # noqa: E402

FALLBACK_HBM_GBS = 6650.0
METRIC = "rows/s (500-tree depth-8 GBDT, 1M rows)"  # BASELINE.json's metric, quoted on c2
LATENCY_SIZES = (1, 8, 64)


def metric_of(cfg) -> str:
    return METRIC if cfg.name == "c2" else f"rows/s ({cfg.name}: {cfg.describe})"


def peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def capture_of(config: str) -> dict:
    """The committed ncu capture summary of the config's kernel (empty when
    there is none)."""
    path = ROOT / "profiles" / f"{config}_dram_traffic.json"
    return json.loads(path.read_text()) if path.exists() else {}


class Clocks:
    """nvidia-smi samples of the SM clock and throttle reasons while running
    (written to a temporary file)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int) -> None:
        self.proc = None
        self.out = tempfile.TemporaryFile(mode="w+")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(device)], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        self.out.seek(0)
        rows = [line.split(", ") for line in self.out.read().splitlines() if line.count(",") >= 8]
        self.out.close()
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            for name, flag in zip(names, r[5:9]):
                if flag.strip() == "Active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": sorted(reasons),
                "samples": len(rows)}


def outputs_of(model: bytes) -> int:
    from montlok import export

    return int(export.read(model)[0]["outputs"]["size"])


# ---------------------------------------------------------------------------
# CPU side: the reference runtime (or the oracle port without it)
# ---------------------------------------------------------------------------


def cpu_reference_rate(model: bytes, x: np.ndarray, seconds: float, threads: int) -> dict:
    """rows/s of the reference CPU runtime (or the oracle port when the
    reference library is absent) on a bounded sample of `x`."""
    import oracle

    K = outputs_of(model)
    if oracle.available_reference():
        ref = oracle.Reference()
        ref.set_threads(threads)
        h = ref.open(model)
        try:
            probe = np.ascontiguousarray(x[:8192])
            out = np.empty((len(probe), K))
            t0 = time.perf_counter()
            ref.predict_handle(h, probe, out)
            rate = len(probe) / max(time.perf_counter() - t0, 1e-9)
            rows = int(min(len(x), max(8192, rate * seconds)))
            sample = np.ascontiguousarray(x[:rows])
            out = np.empty((rows, K))
            t0 = time.perf_counter()
            ref.predict_handle(h, sample, out)
            elapsed = time.perf_counter() - t0
        finally:
            ref.close(h)
        kind, what = "reference", f"{rows} rows of the same workload, one montlok_model_predict call"
    else:
        o = oracle.Oracle(model)
        probe = x[:2048]
        t0 = time.perf_counter()
        o.predict(probe, threads=threads)
        rate = len(probe) / max(time.perf_counter() - t0, 1e-9)
        rows = int(min(len(x), max(2048, rate * seconds)))
        t0 = time.perf_counter()
        o.predict(x[:rows], threads=threads)
        elapsed = time.perf_counter() - t0
        kind, what = "port", f"{rows} rows of the same workload through the C port"
    return {"value": rows / elapsed, "unit": "rows/s", "cores": threads, "kind": kind, "sample": what}


def reference_latency(calls: int, seconds: float, model: bytes, x: np.ndarray, threads: int,
                      latency_threads: int = 0) -> dict:
    """Per-call latency of the reference runtime ({} without it), with
    `latency_threads` of its spinning single-row workers."""
    import oracle

    if not oracle.available_reference():
        return {}
    ref = oracle.Reference()
    ref.set_threads(threads)
    ref.lib.montlok_set_latency_threads(int(latency_threads))
    h = ref.open(model)
    stats = {}
    try:
        for n in LATENCY_SIZES:
            rows = x[: len(x) // n * n].reshape(-1, n * x.shape[1])
            count = max(50, min(calls, int(seconds / len(LATENCY_SIZES) * 1e6 / (40.0 * n))))
            stats[str(n)] = latency_stats(ref.time_calls(h, rows, n, count, max(10, count // 10)))
    finally:
        ref.close(h)
        ref.lib.montlok_set_latency_threads(0)
    return stats


def latency_stats(samples_ns: np.ndarray) -> dict:
    return {"p50_us": float(np.percentile(samples_ns, 50)) / 1e3, "p99_us": float(np.percentile(samples_ns, 99)) / 1e3,
            "mean_us": float(np.mean(samples_ns)) / 1e3, "calls": int(len(samples_ns))}


def run_reference(args, cfg) -> None:
    """The reference CPU runtime alone on rank 0, each step the full batch."""
    import oracle
    from montlok import synth  # noqa: F401  (pure Python: the model builders)

    if int(os.environ.get("RANK", "0")) != 0:
        return
    threads = os.cpu_count() or 1
    model = cfg.model().to_bytes()
    if cfg.name == "c5":
        stats = reference_latency(args.calls, args.cpu_seconds, model, cfg.inputs(batch=64 * 256), threads)
        if not stats:
            print(json.dumps({"impl": "reference", "unavailable": "reference library not built"}), flush=True)
            return
        line = latency_line(args, cfg, stats)
        line["impl"] = "reference"
        line["cpu_baseline"] = {"value": stats["64"]["p50_us"], "unit": "us", "cores": threads, "kind": "reference",
                                "sample": "per-call latency, calls of 1, 8 and 64 rows"}
        line["e2e"] = {"value": stats["64"]["p50_us"], "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
        print(json.dumps(line), flush=True)
        return
    batch = args.rows or cfg.batch
    x = cfg.inputs(batch=batch)
    out = np.empty((batch, outputs_of(model)))
    kind = "reference" if oracle.available_reference() else "port"
    if kind == "reference":
        ref = oracle.Reference()
        ref.set_threads(threads)
        h = ref.open(model)
        step = lambda: ref.predict_handle(h, x, out)  # noqa: E731
    else:
        o = oracle.Oracle(model)
        step = lambda: o.predict(x, threads=threads)  # noqa: E731
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    elapsed = time.perf_counter() - t0
    value = batch * args.steps / elapsed
    line = {"metric": metric_of(cfg), "value": value, "unit": "rows/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic", "impl": "reference",
            "config": workload(cfg, args, batch),
            "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": kind,
                             "sample": f"the full {batch}-row batch per step, one montlok_model_predict call"},
            "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    loaded = [p for p in open("/proc/self/maps").read().split() if p.endswith("libmontlok.so")]
    line["libmontlok_loaded"] = bool(loaded)
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------


def workload(cfg, args, batch: int) -> dict:
    return {"workload": f"{cfg.name}: {cfg.describe}", "rows_per_rank": batch,
            "l2": "inputs larger than L2 (no flush needed)" if batch * 8 * 32 > 126e6 else
                  "inputs smaller than L2: a 256 MB buffer is written between timed steps",
            "parallelism": f"rows sharded, {args.gpus} GPU(s)"}


class Measure:
    """The device-resident and end-to-end timing of one configuration on this
    rank's GPU."""

    def __init__(self, torch, montlok, model_bytes: bytes, x: np.ndarray, stream) -> None:
        self.torch, self.montlok = torch, montlok
        self.model = montlok.load(model_bytes)
        self.x = x
        self.batch = len(x)
        self.K, self.F = self.model.outputs, self.model.features
        self.stream = stream
        self.x_dev = torch.from_numpy(x).cuda()
        self.out_dev = torch.empty((self.batch, self.K), dtype=torch.float64, device="cuda")
        self.small = self.batch * self.F * 8 < 256 << 20
        # Writing this buffer between steps evicts the inputs from L2 when they would fit it.
        self.flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda") if self.small else None
        self.kernel = self.model.kernel(self.batch)

    def step(self) -> None:
        self.model.predict_device(self.x_dev.data_ptr(), self.batch, self.out_dev.data_ptr(),
                                  self.montlok._core.FLOAT64, self.stream.cuda_stream)

    def device_ms(self, steps: int, warmup: int, barrier) -> float:
        torch = self.torch
        for _ in range(warmup):
            self.step()
        barrier()
        if not self.small:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(self.stream)
            for _ in range(steps):
                self.step()
            end.record(self.stream)
            barrier()
            return start.elapsed_time(end) / steps
        # Inputs that fit L2: flush it before each step, time each step alone.
        total = 0.0
        for _ in range(steps):
            with torch.cuda.stream(self.stream):
                self.flush.fill_(1)
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(self.stream)
            self.step()
            end.record(self.stream)
            end.synchronize()
            total += start.elapsed_time(end)
        barrier()
        return total / steps

    def e2e_ms(self, steps: int, barrier) -> tuple[float, np.ndarray]:
        torch = self.torch
        x_pin = torch.from_numpy(self.x).pin_memory()
        out_pin = torch.empty((self.batch, self.K), dtype=torch.float64).pin_memory()
        x_np, out_np = x_pin.numpy(), out_pin.numpy()
        self.model.predict(x_np, out=out_np)
        barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            self.model.predict(x_np, out=out_np)
        barrier()
        return (time.perf_counter() - t0) * 1e3 / steps, out_np.copy()

    def check(self, host: np.ndarray) -> None:
        y_dev = self.out_dev.cpu().numpy()
        if not np.array_equal(host.view(np.int64), y_dev.view(np.int64)):
            raise SystemExit("host-buffer and device-buffer predictions differ")

    def launches_per_step(self) -> int:
        K = self.K
        if self.kernel in ("generic", "generic-global-keys"):
            return (K + 7) // 8 + (1 if (K > 8 and self.model.spec["config"].get("link") == "softmax") else 0)
        return 1


def roofline(config: str, ms: float, batch: int, F: int) -> dict:
    peak, peak_kind = peaks()
    bytes_per_launch = batch * F * 8
    achieved = bytes_per_launch / (ms / 1e3) / 1e9
    capture = capture_of(config)
    per_row = capture.get("dram_bytes_per_row")
    return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "peak_source": f"{peak_kind} hbm_gbs", "traffic": float(per_row) * batch if per_row else None,
            "algorithmic_bytes_per_launch": bytes_per_launch,
            "ncu_capture": {k: capture.get(k) for k in ("kernel", "captured_rows", "issue_active_pct",
                                                         "smem_pipe_pct", "warp_inst_per_warp_tree") if k in capture}}


def config_figures(torch, montlok, cfg, args, barrier, batch: int, cpu: bool) -> dict:
    """Device rows/s, e2e rows/s, roofline and CPU baseline of one config on this GPU."""
    model_bytes = cfg.model().to_bytes()
    x = cfg.inputs(batch=batch)
    m = Measure(torch, montlok, model_bytes, x, torch.cuda.Stream())
    ms = m.device_ms(args.steps, args.warmup, barrier)
    e2e_ms, host = m.e2e_ms(args.e2e_steps, barrier)
    m.check(host)
    fig = {"metric": metric_of(cfg), "kernel": m.kernel, "rows": batch, "value": batch / (ms / 1e3),
           "unit": "rows/s", "ms_per_step": ms,
           "e2e": {"value": batch / (e2e_ms / 1e3), "unit": "rows/s", "ms_per_step": e2e_ms,
                   "h2d_bytes_per_step": batch * m.F * 8, "d2h_bytes_per_step": batch * m.K * 8},
           "roofline": roofline(cfg.name, ms, batch, m.F), "gpu_launches": args.steps * m.launches_per_step()}
    if cpu:
        fig["cpu_baseline"] = cpu_reference_rate(model_bytes, x, args.cpu_seconds, os.cpu_count() or 1)
    del m
    torch.cuda.empty_cache()
    return fig


def latency_line(args, cfg, stats: dict) -> dict:
    p50 = stats["64"]["p50_us"]
    return {"metric": f"p50 us per 64-row call ({cfg.name}: {cfg.describe})", "value": p50, "unit": "us",
            "n_gpus": args.gpus, "steps": args.calls, "warmup": args.warmup, "ms_per_step": p50 / 1e3,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": f"{cfg.name}: {cfg.describe}", "call_rows": list(LATENCY_SIZES),
                       "timing": "per call, inside the library, host buffers in and out"},
            "latency": stats}


def latency_figures(torch, montlok, cfg, args, cpu: bool) -> dict:
    """c5: per-call latency of 1, 8 and 64-row host-buffer calls, the device
    time of a 64-row launch, and the reference's per-call latency."""
    model_bytes = cfg.model().to_bytes()
    model = montlok.load(model_bytes)
    x = cfg.inputs(batch=64 * 256)
    stats = {}
    for n in LATENCY_SIZES:
        rows = x[: len(x) // n * n].reshape(-1, n * model.features)
        samples, _ = montlok._core.bench(model, rows, batch=n, iterations=args.calls)
        stats[str(n)] = latency_stats(samples)
    xd = torch.from_numpy(np.ascontiguousarray(x[:64])).cuda()
    od = torch.empty((64, model.outputs), dtype=torch.float64, device="cuda")
    stream = torch.cuda.Stream()
    for _ in range(max(args.warmup, 3)):
        model.predict_device(xd.data_ptr(), 64, od.data_ptr(), montlok._core.FLOAT64, stream.cuda_stream)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(100):
        model.predict_device(xd.data_ptr(), 64, od.data_ptr(), montlok._core.FLOAT64, stream.cuda_stream)
    end.record(stream)
    torch.cuda.synchronize()
    # With latency threads on, calls of at most 8 rows go to the resident
    # latency engine instead of a graph launch.
    montlok.set_latency_threads(1)
    engine = {}
    try:
        for n in (1, 8):
            rows = x[: len(x) // n * n].reshape(-1, n * model.features)
            samples, _ = montlok._core.bench(model, rows, batch=n, iterations=args.calls)
            engine[str(n)] = latency_stats(samples)
    finally:
        montlok.set_latency_threads(0)
    fig = {"latency": stats, "latency_engine": engine, "kernel": {str(n): model.kernel(n) for n in LATENCY_SIZES},
           "device_us_per_64_rows": start.elapsed_time(end) * 10.0,
           "gpu_launches": args.calls * len(LATENCY_SIZES)}
    if cpu:
        threads = os.cpu_count() or 1
        ref = reference_latency(args.calls, args.cpu_seconds, model_bytes, x, threads)
        if ref:
            spin = min(7, max(1, threads - 1))
            fig["cpu_baseline"] = {"value": ref["64"]["p50_us"], "unit": "us", "cores": threads, "kind": "reference",
                                   "sample": "per-call latency, calls of 1, 8 and 64 rows", "latency": ref,
                                   f"latency_with_{spin}_latency_threads":
                                       reference_latency(args.calls, args.cpu_seconds, model_bytes, x, threads, spin)}
    return fig


def run_latency(args, cfg) -> None:
    """The small-batch configuration on rank 0's GPU (other ranks idle)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    import torch

    import montlok

    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    clocks = Clocks(int(os.environ.get("LOCAL_RANK", "0")))
    fig = latency_figures(torch, montlok, cfg, args, cpu=not args.no_cpu)
    line = latency_line(args, cfg, fig["latency"])
    line["device_us_per_64_rows"] = fig["device_us_per_64_rows"]
    line["latency_engine"] = fig["latency_engine"]
    line["kernel"] = fig["kernel"]
    line["e2e"] = {"value": fig["latency"]["64"]["p50_us"], "unit": "us", "h2d_bytes_per_step": 64 * 200 * 8,
                   "d2h_bytes_per_step": 64 * 8}
    line["roofline"] = None
    line["gpu_launches"] = fig["gpu_launches"]
    line["clocks"] = clocks.stop()
    if "cpu_baseline" in fig:
        line["cpu_baseline"] = fig["cpu_baseline"]
    print(json.dumps(line), flush=True)


def sharded_call(torch, montlok, cfg, world: int, batch: int, steps: int) -> dict:
    """One host-buffer call of `batch` pinned rows that the library splits
    over devices 0..world-1 itself (montlok_set_devices), timed on the host
    around the blocking call: strong scaling of a single call."""
    model = montlok.load(cfg.model().to_bytes())
    x_pin = torch.from_numpy(cfg.inputs(batch=batch)).pin_memory()
    out_pin = torch.empty((batch, model.outputs), dtype=torch.float64).pin_memory()
    x_np, out_np = x_pin.numpy(), out_pin.numpy()
    montlok.set_devices(world)
    try:
        model.predict(x_np, out=out_np)  # uploads to every device, first-touch of the workers
        t0 = time.perf_counter()
        for _ in range(steps):
            model.predict(x_np, out=out_np)
        ms = (time.perf_counter() - t0) * 1e3 / steps
    finally:
        montlok.set_devices(0)
    return {"devices": world, "rows": batch, "value": batch / (ms / 1e3), "unit": "rows/s", "ms_per_call": ms,
            "h2d_bytes_per_call": batch * model.features * 8, "timing": "host clock around one blocking call"}


def h2d_rate(torch, barrier, gib: int = 1) -> float:
    """Seconds of one pinned host -> device copy of `gib` GiB on this rank's
    GPU, every rank copying at the same time (the ceiling the e2e figures run
    against: each GPU's link and the host memory the ranks share)."""
    src = torch.empty(gib << 30, dtype=torch.uint8).pin_memory()
    dst = torch.empty(gib << 30, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dst.copy_(src, non_blocking=True)
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(3):
            dst.copy_(src, non_blocking=True)
    end.record(stream)
    barrier()
    seconds = start.elapsed_time(end) / 3e3
    del src, dst
    return seconds


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=10)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--config", default="c2")
    parser.add_argument("--rows", type=int, default=0, help="rows per rank (default: the config's batch)")
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--e2e-steps", type=int, default=3)
    parser.add_argument("--cpu-seconds", type=float, default=8.0)
    parser.add_argument("--no-cpu", action="store_true")
    parser.add_argument("--configs", default="c1,c3,c4,c5",
                        help="other configurations measured on one GPU beside the default c2 line ('' for none)")
    parser.add_argument("--calls", type=int, default=20000, help="timed calls per size (latency configuration)")
    args = parser.parse_args()
    args.warmup = max(args.warmup, 3)

    from montlok import synth

    cfg = synth.CONFIGS[args.config]
    if args.impl == "reference":
        run_reference(args, cfg)
        return
    if args.config == "c5":
        run_latency(args, cfg)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    batch = args.rows or cfg.batch

    import torch
    import torch.distributed as dist

    import montlok

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    model_bytes = cfg.model().to_bytes()
    x = cfg.inputs(batch=batch)
    m = Measure(torch, montlok, model_bytes, x, torch.cuda.Stream())
    clocks = Clocks(local)
    ms = m.device_ms(args.steps, args.warmup, barrier)
    e2e_ms, host = m.e2e_ms(args.e2e_steps, barrier)
    clock = clocks.stop()
    m.check(host)

    h2d_s = h2d_rate(torch, barrier)

    from montlok.distributed import max_over_ranks

    ms, e2e_ms, h2d_s = max_over_ranks([ms, e2e_ms, h2d_s], device="cuda")

    line = None
    if rank == 0:
        line = {
            "metric": metric_of(cfg), "value": world * batch / (ms / 1e3), "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": workload(cfg, args, batch), "kernel": m.kernel,
            "e2e": {"value": world * batch / (e2e_ms / 1e3), "unit": "rows/s", "h2d_bytes_per_step": batch * m.F * 8,
                    "d2h_bytes_per_step": batch * m.K * 8, "ms_per_step": e2e_ms,
                    "timing": "host clock around the blocking montlok_model_predict call, max over ranks"},
            "roofline": roofline(args.config, ms, batch, m.F),
            "gpu_launches": args.steps * m.launches_per_step(),
            "clocks": clock,
            "h2d_ceiling": {"per_gpu_gbs": (1 << 30) / h2d_s / 1e9, "all_gpus_gbs": world * (1 << 30) / h2d_s / 1e9,
                            "e2e_input_gbs": world * batch * m.F * 8 / (e2e_ms / 1e3) / 1e9,
                            "how": "3 pinned 1 GiB host->device copies per rank, all ranks at once, slowest rank"},
        }
    del m, x
    torch.cuda.empty_cache()
    # Strong scaling of one call split by the library over every rank's GPU:
    # rank 0 alone, while the other ranks wait at the barrier.
    if world > 1 or args.gpus > 1:
        if rank == 0:
            line["sharded"] = sharded_call(torch, montlok, cfg, max(world, args.gpus), batch, args.e2e_steps)
        if world > 1:
            dist.barrier()
    if rank == 0:
        if world == 1 and not args.no_cpu:
            line["cpu_baseline"] = cpu_reference_rate(model_bytes, cfg.inputs(batch=batch), args.cpu_seconds,
                                                      os.cpu_count() or 1)
        if world == 1 and args.config == "c2" and args.configs:
            configs = {}
            for name in [n for n in args.configs.split(",") if n]:
                other = synth.CONFIGS[name]
                if name == "c5":
                    configs[name] = latency_figures(torch, montlok, other, args, cpu=not args.no_cpu)
                else:
                    configs[name] = config_figures(torch, montlok, other, args, barrier, other.batch,
                                                   cpu=not args.no_cpu)
            line["configs"] = configs
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
