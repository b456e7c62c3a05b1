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
             against the measured copy bandwidth (MEASURED_PEAKS.json)
  cpu_baseline  the reference runtime (oracle/_ref, compiled from its sources)
             on this host's cores, on a bounded sample of the same workload

``--impl reference`` times the reference's CPU implementation alone, with all
host threads, on the same workload and prints the same line.

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
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT / "montlok.cpp_b200" / "python", ROOT / "oracle"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import numpy as np  # noqa: E402

FALLBACK_HBM_GBS = 6650.0
METRIC = "rows/s (500-tree depth-8 GBDT, 1M rows)"  # BASELINE.json's metric, quoted on c2


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


def traffic_per_launch(config: str, rows: int) -> float | None:
    """DRAM bytes of one launch over `rows` rows, from the committed ncu
    capture of the same kernel (bytes per row times rows)."""
    capture = capture_of(config)
    return float(capture["dram_bytes_per_row"]) * rows if "dram_bytes_per_row" in capture else None


class Clocks:
    """nvidia-smi samples of the SM clock and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int) -> None:
        self.proc = None
        self.path = ROOT / "gpurun_out" / f"clocks_rank{device}.csv"
        try:
            self.path.parent.mkdir(exist_ok=True)
            self.out = open(self.path, "w")
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
        self.out.close()
        rows = [line.split(", ") for line in self.path.read_text().splitlines() if line.count(",") >= 8]
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


def cpu_reference_rate(model: bytes, x: np.ndarray, seconds: float, threads: int) -> tuple[float, str, str]:
    """rows/s of the reference CPU runtime (or the oracle port when the
    reference library is absent) on a bounded sample of `x`."""
    import oracle

    K = outputs_of(model)
    if oracle.available_reference():
        ref = oracle.Reference()
        ref.set_threads(threads)
        h = ref.open(model)
        try:
            probe = x[:8192]
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
        return rows / elapsed, "reference", f"{rows} rows of the same workload, one montlok_model_predict call"
    o = oracle.Oracle(model)
    probe = x[:2048]
    t0 = time.perf_counter()
    o.predict(probe, threads=threads)
    rate = len(probe) / max(time.perf_counter() - t0, 1e-9)
    rows = int(min(len(x), max(2048, rate * seconds)))
    t0 = time.perf_counter()
    o.predict(x[:rows], threads=threads)
    return rows / (time.perf_counter() - t0), "port", f"{rows} rows of the same workload through the C port"


def run_reference(args, cfg, model: bytes, x: np.ndarray) -> dict:
    """The reference CPU runtime alone, each step a bounded sample of the workload."""
    import oracle

    threads = os.cpu_count() or 1
    rows = min(len(x), args.reference_rows)
    sample = np.ascontiguousarray(x[:rows])
    out = np.empty((rows, outputs_of(model)))
    kind = "reference" if oracle.available_reference() else "port"
    if kind == "reference":
        ref = oracle.Reference()
        ref.set_threads(threads)
        h = ref.open(model)
        step = lambda: ref.predict_handle(h, sample, out)  # noqa: E731
    else:
        o = oracle.Oracle(model)
        step = lambda: o.predict(sample, threads=threads)  # noqa: E731
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    elapsed = time.perf_counter() - t0
    value = rows * args.steps / elapsed
    return {"metric": metric_of(cfg), "value": value, "unit": "rows/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic", "impl": "reference",
            "config": workload(cfg, args),
            "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": kind,
                             "sample": f"{rows} rows of the workload per step"},
            "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


LATENCY_SIZES = (1, 8, 64)


def latency_stats(samples_ns: np.ndarray) -> dict:
    return {"p50_us": float(np.percentile(samples_ns, 50)) / 1e3, "p99_us": float(np.percentile(samples_ns, 99)) / 1e3,
            "mean_us": float(np.mean(samples_ns)) / 1e3, "calls": int(len(samples_ns))}


def latency_line(args, cfg, stats: dict, impl: str | None) -> dict:
    p50 = stats["64"]["p50_us"]
    line = {"metric": f"p50 us per 64-row call ({cfg.name}: {cfg.describe})", "value": p50, "unit": "us",
            "n_gpus": args.gpus, "steps": args.calls, "warmup": args.warmup, "ms_per_step": p50 / 1e3,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": f"{cfg.name}: {cfg.describe}", "call_rows": list(LATENCY_SIZES),
                       "timing": "per call, inside the library, host buffers in and out"},
            "latency": stats}
    if impl:
        line["impl"] = impl
    return line


def reference_latency(args, model: bytes, x: np.ndarray, threads: int) -> tuple[dict, str]:
    """Per-call latency of the reference runtime (or None without it)."""
    import oracle

    if not oracle.available_reference():
        return {}, "unavailable"
    ref = oracle.Reference()
    ref.set_threads(threads)
    h = ref.open(model)
    stats = {}
    try:
        for n in LATENCY_SIZES:
            rows = x[: len(x) // n * n].reshape(-1, n * x.shape[1])
            calls = max(50, min(args.calls, int(args.cpu_seconds / len(LATENCY_SIZES) * 1e6 / (40.0 * n))))
            stats[str(n)] = latency_stats(ref.time_calls(h, rows, n, calls, max(10, calls // 10)))
    finally:
        ref.close(h)
    return stats, "reference"


def run_latency(args, cfg) -> None:
    """The small-batch configuration on rank 0's GPU (other ranks idle)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    model_bytes = cfg.model().to_bytes()
    x = cfg.inputs(batch=64 * 256)
    threads = os.cpu_count() or 1
    if args.impl == "reference":
        stats, kind = reference_latency(args, model_bytes, x, threads)
        if not stats:
            print(json.dumps({"impl": "reference", "unavailable": "reference library not built"}), flush=True)
            return
        line = latency_line(args, cfg, stats, "reference")
        line["cpu_baseline"] = {"value": stats["64"]["p50_us"], "unit": "us", "cores": threads, "kind": kind,
                                "sample": "per-call latency, calls of 1, 8 and 64 rows"}
        line["e2e"] = {"value": stats["64"]["p50_us"], "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
        print(json.dumps(line), flush=True)
        return
    import torch

    import montlok

    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    model = montlok.load(model_bytes)
    clocks = Clocks(int(os.environ.get("LOCAL_RANK", "0")))
    stats = {}
    for n in LATENCY_SIZES:
        rows = x[: len(x) // n * n].reshape(-1, n * model.features)
        samples, _ = montlok._core.bench(model, rows, batch=n, iterations=args.calls)
        stats[str(n)] = latency_stats(samples)
    # Device time of one 64-row predict (inputs resident), CUDA events.
    xd = torch.from_numpy(np.ascontiguousarray(x[:64])).cuda()
    od = torch.empty((64, model.outputs), dtype=torch.float64, device="cuda")
    stream = torch.cuda.Stream()
    for _ in range(args.warmup):
        model.predict_device(xd.data_ptr(), 64, od.data_ptr(), montlok._core.FLOAT64, stream.cuda_stream)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(100):
        model.predict_device(xd.data_ptr(), 64, od.data_ptr(), montlok._core.FLOAT64, stream.cuda_stream)
    end.record(stream)
    torch.cuda.synchronize()
    line = latency_line(args, cfg, stats, None)
    line["device_us_per_64_rows"] = start.elapsed_time(end) * 10.0
    line["e2e"] = {"value": stats["64"]["p50_us"], "unit": "us", "h2d_bytes_per_step": 64 * model.features * 8,
                   "d2h_bytes_per_step": 64 * model.outputs * 8}
    line["roofline"] = None
    line["gpu_launches"] = args.calls * len(LATENCY_SIZES)
    line["clocks"] = clocks.stop()
    if not args.no_cpu:
        ref_stats, kind = reference_latency(args, model_bytes, x, threads)
        if ref_stats:
            line["cpu_baseline"] = {"value": ref_stats["64"]["p50_us"], "unit": "us", "cores": threads, "kind": kind,
                                    "sample": "per-call latency, calls of 1, 8 and 64 rows", "latency": ref_stats}
    print(json.dumps(line), flush=True)


def workload(cfg, args) -> dict:
    return {"workload": f"{cfg.name}: {cfg.describe}", "rows_per_rank": args.rows or cfg.batch,
            "l2": "inputs larger than L2 (no flush needed)", "parallelism": f"rows sharded, {args.gpus} GPU(s)"}


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
    parser.add_argument("--reference-rows", type=int, default=65536)
    parser.add_argument("--no-cpu", action="store_true")
    parser.add_argument("--calls", type=int, default=20000, help="timed calls per size (latency configuration)")
    args = parser.parse_args()
    args.warmup = max(args.warmup, 3)

    from montlok import synth

    cfg = synth.CONFIGS[args.config]
    if args.config == "c5":
        run_latency(args, cfg)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    batch = args.rows or cfg.batch

    if args.impl == "reference":
        if rank != 0:
            return
        model = cfg.model().to_bytes()
        x = cfg.inputs(batch=min(batch, max(args.reference_rows, 8192)))
        print(json.dumps(run_reference(args, cfg, model, x)), flush=True)
        return

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
    model = montlok.load(model_bytes)
    x = cfg.inputs(batch=batch)
    K, F = model.outputs, model.features
    x_dev = torch.from_numpy(x).cuda()
    out_dev = torch.empty((batch, K), dtype=torch.float64, device="cuda")
    stream = torch.cuda.Stream()
    launches_per_step = (K + 7) // 8 + (1 if (K > 8 and model.spec["config"].get("link") == "softmax") else 0)

    def step():
        model.predict_device(x_dev.data_ptr(), batch, out_dev.data_ptr(), montlok._core.FLOAT64, stream.cuda_stream)

    clocks = Clocks(local)
    for _ in range(args.warmup):
        step()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        step()
    end.record(stream)
    barrier()
    ms = start.elapsed_time(end) / args.steps
    y_dev = out_dev.cpu().numpy()

    # End to end through the reference-facing call: pinned host buffers, copies inside.
    x_pin = torch.from_numpy(x).pin_memory()
    out_pin = torch.empty((batch, K), dtype=torch.float64).pin_memory()
    out_np = out_pin.numpy()
    x_np = x_pin.numpy()
    model.predict(x_np, out=out_np)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        model.predict(x_np, out=out_np)
    barrier()
    e2e_ms = (time.perf_counter() - t0) * 1e3 / args.e2e_steps
    clock = clocks.stop()
    if not np.array_equal(out_np.view(np.int64), y_dev.view(np.int64)):
        raise SystemExit("host-buffer and device-buffer predictions differ")

    from montlok.distributed import max_over_ranks

    ms, e2e_ms = max_over_ranks([ms, e2e_ms], device="cuda")

    if rank == 0:
        peak, peak_kind = peaks()
        bytes_per_launch = batch * F * 8
        achieved = bytes_per_launch / (ms / 1e3) / 1e9
        traffic = traffic_per_launch(args.config, batch)
        line = {
            "metric": metric_of(cfg), "value": world * batch / (ms / 1e3), "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": workload(cfg, args),
            "e2e": {"value": world * batch / (e2e_ms / 1e3), "unit": "rows/s", "h2d_bytes_per_step": batch * F * 8,
                    "d2h_bytes_per_step": batch * K * 8, "ms_per_step": e2e_ms,
                    "timing": "host clock around the blocking montlok_model_predict call, max over ranks"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"{peak_kind} hbm_gbs", "traffic": traffic,
                         "algorithmic_bytes_per_launch": bytes_per_launch,
                         "issue_active_pct_ncu": capture_of(args.config).get("issue_active_pct")},
            "gpu_launches": args.steps * launches_per_step,
            "clocks": clock,
        }
        if world == 1 and not args.no_cpu:
            rate, kind, sample = cpu_reference_rate(model_bytes, x, args.cpu_seconds, os.cpu_count() or 1)
            line["cpu_baseline"] = {"value": rate, "unit": "rows/s", "cores": os.cpu_count() or 1, "kind": kind,
                                    "sample": sample}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
