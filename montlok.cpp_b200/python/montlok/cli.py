"""``montlok`` command line for the GPU predict path (``python -m montlok``).

    montlok predict MODEL INPUT [-o OUTPUT] [--memory host|pinned|device] [--devices N]
    montlok bench MODEL [--batch B] [--iterations K] [--rows R] [--memory ...] [--devices N] [--json]

``predict`` reads rows from a .npy/.npz array or a CSV table (an optional
first line of column names is matched against the model's feature names),
predicts them and writes a .npy array or CSV (stdout when no ``-o``).
``bench`` times calls of ``--batch`` random N(0, 1) rows and reports the
per-call p50/p99 latency and rows/s. Both can hand the library host memory
(pageable or pinned) or device memory, and split host batches over GPUs
(``--devices``, montlok_set_devices). These are the two verbs of the
reference's CLI that sit on the predict path (its python/montlok/cli.py);
its converter, info and environment verbs are not part of this build.
"""

from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path
from typing import Sequence

import numpy as np

MEMORY = ("host", "pinned", "device")


def _table(path: Path) -> tuple[np.ndarray, list[str] | None]:
    """The rows of a .npy/.npz/.csv file, and the CSV's column names if it has them."""
    if path.suffix == ".npy":
        return np.load(path), None
    if path.suffix == ".npz":
        with np.load(path) as archive:
            return archive[archive.files[0]], None
    lines = path.read_text().splitlines()
    if not lines:
        return np.zeros((0, 0)), None
    first = [cell.strip() for cell in lines[0].split(",")]
    try:
        [float(cell) for cell in first if cell]
        names, body = None, lines
    except ValueError:
        names, body = first, lines[1:]
    rows = [[float(cell) if cell.strip() else np.nan for cell in line.split(",")] for line in body if line.strip()]
    return np.asarray(rows, dtype=np.float64).reshape(len(rows), -1), names


def _arrange(model, table: np.ndarray, names: list[str] | None) -> np.ndarray:
    """The table's columns in the model's feature order (by name when both have names)."""
    table = np.atleast_2d(table)
    known = model.spec.get("inputs", {}).get("names")
    if names and known:
        missing = [n for n in known if n not in names]
        if missing:
            raise SystemExit(f"montlok: input lacks feature column(s) {', '.join(missing[:5])}")
        table = table[:, [names.index(n) for n in known]]
    if table.shape[1] != model.features:
        raise SystemExit(f"montlok: the input has {table.shape[1]} columns, the model {model.features} features")
    return np.ascontiguousarray(table, dtype=np.float32 if table.dtype == np.float32 else np.float64)


class Buffers:
    """Inputs and outputs of one call shape in host, pinned or device memory."""

    def __init__(self, model, x: np.ndarray, memory: str) -> None:
        self.model, self.memory = model, memory
        rows = len(x)
        if memory == "host":
            self.x, self.out = x, np.empty((rows, model.outputs))
            return
        import torch

        if memory == "pinned":
            self._x = torch.from_numpy(x).pin_memory()
            self._out = torch.empty((rows, model.outputs), dtype=torch.float64).pin_memory()
            self.x, self.out = self._x.numpy(), self._out.numpy()
        else:
            self.x = torch.from_numpy(x).cuda()
            self.out = torch.empty((rows, model.outputs), dtype=torch.float64, device="cuda")
        self.torch = torch

    def run(self) -> None:
        self.model.predict(self.x, out=self.out)
        if self.memory == "device":
            self.torch.cuda.current_stream().synchronize()

    def result(self) -> np.ndarray:
        return self.out.cpu().numpy() if self.memory == "device" else np.array(self.out)


def predict(args: argparse.Namespace) -> int:
    import montlok

    montlok.set_threads(args.threads)
    montlok.set_devices(args.devices)
    model = montlok.load(args.model)
    table, names = _table(Path(args.input))
    x = _arrange(model, table, names)
    buffers = Buffers(model, x, args.memory)
    buffers.run()
    y = buffers.result()
    if args.output and args.output.endswith(".npy"):
        np.save(args.output, y)
        return 0
    columns = model.spec.get("outputs", {}).get("names") or [f"output_{k}" for k in range(model.outputs)]
    text = ",".join(columns) + "\n" + "\n".join(",".join(repr(float(v)) for v in row) for row in y) + "\n"
    if args.output:
        Path(args.output).write_text(text)
    else:
        sys.stdout.write(text)
    return 0


def bench(args: argparse.Namespace) -> int:
    import montlok

    montlok.set_threads(args.threads)
    montlok.set_devices(args.devices)
    model = montlok.load(args.model)
    rng = np.random.default_rng(0)
    inputs = [Buffers(model, rng.standard_normal((args.batch, model.features)), args.memory)
              for _ in range(max(1, min(args.rows, 64)))]
    for i in range(max(100, args.iterations // 10)):
        inputs[i % len(inputs)].run()
    samples = np.empty(args.iterations)
    for i in range(args.iterations):
        start = time.perf_counter_ns()
        inputs[i % len(inputs)].run()
        samples[i] = time.perf_counter_ns() - start
    p50, p99 = (float(np.percentile(samples, q)) / 1e3 for q in (50, 99))
    rate = args.batch / (float(np.mean(samples)) / 1e9)
    report = {"model": str(args.model), "memory": args.memory, "devices": args.devices, "batch": args.batch,
              "calls": args.iterations, "p50_us": p50, "p99_us": p99, "rows_per_s": rate,
              "kernel": model.kernel(args.batch)}
    if args.json:
        print(json.dumps(report))
    else:
        print(f"{args.batch}-row calls, {args.memory} memory, {report['kernel']} kernel: "
              f"p50 {p50:.2f} us  p99 {p99:.2f} us  {rate:,.0f} rows/s over {args.iterations} calls")
    return 0


def parser() -> argparse.ArgumentParser:
    from . import __version__

    top = argparse.ArgumentParser(prog="montlok", description="tree-ensemble predict on the GPU")
    top.add_argument("--version", action="version", version=f"montlok {__version__}")
    verbs = top.add_subparsers(dest="verb", required=True)

    p = verbs.add_parser("predict", help="predict the rows of a .npy/.npz/.csv file")
    p.add_argument("model")
    p.add_argument("input")
    p.add_argument("-o", "--output", help=".npy or .csv path (default: CSV on stdout)")
    p.add_argument("--memory", choices=MEMORY, default="host", help="where the rows are handed to the library")
    p.add_argument("--devices", type=int, default=0, help="GPUs a host batch is split over (0: the current one)")
    p.add_argument("--threads", type=int, default=0, help="host staging threads (0: one per hardware thread)")
    p.set_defaults(run=predict)

    p = verbs.add_parser("bench", help="per-call latency and throughput of one model")
    p.add_argument("model")
    p.add_argument("--batch", type=int, default=1, help="rows per call")
    p.add_argument("--iterations", type=int, default=20000, help="timed calls")
    p.add_argument("--rows", type=int, default=16, help="distinct inputs cycled through (at most 64)")
    p.add_argument("--memory", choices=MEMORY, default="host", help="where the rows are handed to the library")
    p.add_argument("--devices", type=int, default=0, help="GPUs a host batch is split over (0: the current one)")
    p.add_argument("--threads", type=int, default=0, help="host staging threads (0: one per hardware thread)")
    p.add_argument("--json", action="store_true", help="print one JSON object")
    p.set_defaults(run=bench)
    return top


def main(argv: Sequence[str] | None = None) -> int:
    args = parser().parse_args(argv)
    if getattr(args, "batch", 1) <= 0 or getattr(args, "iterations", 1) <= 0:
        raise SystemExit("montlok: --batch and --iterations must be positive")
    return args.run(args)


if __name__ == "__main__":
    raise SystemExit(main())
