"""The `montlok` command for tree-ensemble models on the GPU.

    montlok info MODEL                  what a model file holds
    montlok convert SOURCE -o MODEL     scikit-learn trees, LightGBM / XGBoost dumps -> .montlok
    montlok predict MODEL INPUT         predictions for a CSV / .npy / .npz file
    montlok bench MODEL                 in-process latency and rows/s of one model
    montlok env                         versions, GPUs, settings

Same commands, options and output formats as the reference's CLI for these
verbs (python/montlok/cli.py:102-245, 343-396 in montlok.cpp); `python -m
montlok` runs the same command.
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import sys
from pathlib import Path
from typing import Any, Sequence

import numpy as np

import montlok
from montlok import export


def read_table(path: str | Path) -> tuple[Any, list[str] | None]:
    """A .npy array, the arrays of a .npz, or a CSV and its header (None when
    the first row is numeric)."""
    path = Path(path)
    if path.suffix == ".npy":
        return np.load(path), None
    if path.suffix == ".npz":
        with np.load(path) as data:
            return {name: data[name] for name in data.files}, None
    with path.open() as stream:
        first = stream.readline()
    header: list[str] | None = [token.strip() for token in first.split(",")]
    try:
        [float(token) for token in header]
        header = None
    except ValueError:
        pass
    return np.loadtxt(path, delimiter=",", ndmin=2, skiprows=1 if header else 0), header


def write_table(values: np.ndarray, names: Sequence[str], path: str | None) -> None:
    if path and path.endswith(".npy"):
        np.save(path, values)
        return
    stream = open(path, "w", newline="") if path and path != "-" else sys.stdout
    try:
        np.savetxt(stream, np.atleast_2d(values), delimiter=",", header=",".join(names), comments="", fmt="%.17g")
    finally:
        if stream is not sys.stdout:
            stream.close()


def model_inputs(model: montlok.Model, table: np.ndarray, header: list[str] | None) -> np.ndarray:
    """Rows of `table` as the model's input; a header selects the model's named features in order."""
    names = model.spec["inputs"].get("names")
    if header and names:
        missing = [name for name in names if name not in header]
        if missing:
            raise SystemExit(f"input lacks feature columns: {', '.join(missing[:5])}")
        table = table[:, [header.index(name) for name in names]]
    return table


def output_names(model: montlok.Model) -> list[str]:
    return ["y"] if model.outputs == 1 else [f"y{k}" for k in range(model.outputs)]


def _size(path: Path) -> str:
    size = float(path.stat().st_size)
    for unit in ("B", "KiB", "MiB", "GiB"):
        if size < 1024 or unit == "GiB":
            return f"{size:.0f} {unit}" if unit == "B" else f"{size:.1f} {unit}"
        size /= 1024
    return ""


def cmd_info(args: argparse.Namespace) -> int:
    model = montlok.load(args.model)
    spec = model.spec
    if args.json:
        print(json.dumps(spec, indent=2))
        return 0
    _, tensors = export.read(args.model)
    config = spec.get("config", {})
    prefix = config.get("tensors", "trees")
    rows = [("model", f"{args.model} ({_size(Path(args.model))})"), ("family", model.family),
            ("inputs", f"{model.features} features"), ("outputs", str(model.outputs)),
            ("trees", f"{len(tensors[prefix + '.root'])} ({len(tensors[prefix + '.feature'])} nodes)"),
            ("splits", f"{'<=' if config.get('decision', 'le') == 'le' else '<'} on "
                       f"{'float32' if config.get('feature_cast') == 'f32' else 'float64'} features"),
            ("link", f"{config.get('link', 'identity')}, {config.get('aggregate', 'sum')} of trees")]
    pre = spec.get("preprocess")
    if pre:
        parts = (["standardize"] if pre.get("mean") else []) + ([f"clip {pre['clip']}"] if pre.get("clip") else [])
        rows.insert(4, ("preprocess", ", ".join(parts)))
    meta = spec.get("metadata", {})
    if meta:
        rows.append(("exported", ", ".join(f"{k}={v}" for k, v in meta.items() if isinstance(v, (str, int, float)))))
    width = max(len(name) for name, _ in rows)
    for name, value in rows:
        print(f"{name:<{width}}  {value}")
    return 0


def cmd_convert(args: argparse.Namespace) -> int:
    path = Path(args.source)
    names = args.feature_names.split(",") if args.feature_names else None
    if path.suffix == ".json":
        data = json.loads(path.read_text())
        if isinstance(data, dict) and "tree_info" in data:
            exported = export.from_lightgbm(data, feature_names=names)
        else:
            raise SystemExit(f"{path}: expected a LightGBM dump_model() JSON file")
    elif path.suffix in (".joblib", ".pkl", ".pickle"):
        import pickle

        with path.open("rb") as stream:
            exported = export.from_sklearn(pickle.load(stream), feature_names=names)
    else:
        raise SystemExit(f"{path}: use a LightGBM dump_model() .json or a pickled scikit-learn tree model")
    exported.save(args.output)
    model = montlok.load(args.output)
    print(f"{args.output}: {model.family}, {model.features} features -> {model.outputs} output(s)")
    return 0


def cmd_predict(args: argparse.Namespace) -> int:
    montlok.set_threads(args.threads)
    montlok.set_devices(args.devices)
    model = montlok.load(args.model)
    table, header = read_table(args.input)
    if isinstance(table, dict):
        table = table["x"] if "x" in table else next(iter(table.values()))
    y = model.predict(model_inputs(model, table, header))
    write_table(y.reshape(len(y), -1) if y.ndim > 1 else y.reshape(1, -1), output_names(model), args.output)
    return 0


def _ns(value: float) -> str:
    return f"{value:.0f} ns" if value < 1000 else f"{value / 1000:.2f} µs" if value < 1e6 else f"{value / 1e6:.2f} ms"


def bench_device(model, rows: np.ndarray, batch: int, iterations: int) -> tuple[np.ndarray, float]:
    """Per-call latency of montlok_model_predict_device with inputs and outputs
    resident on the GPU (CUDA events around each call), and the mean of
    back-to-back calls."""
    import torch

    x = torch.from_numpy(np.ascontiguousarray(rows.reshape(-1, model.features))).cuda()
    out = torch.empty((len(rows) * batch, model.outputs), dtype=torch.float64, device="cuda")
    stream = torch.cuda.Stream()
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iterations)]

    def call(i: int) -> None:
        j = (i % len(rows)) * batch
        model.predict_device(x[j].data_ptr(), batch, out[j].data_ptr(), montlok._core.FLOAT64, stream.cuda_stream)

    for i in range(max(100, iterations // 10)):
        call(i)
    for i, (a, b) in enumerate(events):
        a.record(stream)
        call(i)
        b.record(stream)
    stream.synchronize()
    samples = np.array([a.elapsed_time(b) * 1e6 for a, b in events])
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(iterations):
        call(i)
    end.record(stream)
    stream.synchronize()
    return samples, start.elapsed_time(end) * 1e6 / iterations


def cmd_bench(args: argparse.Namespace) -> int:
    montlok.set_threads(args.threads)
    montlok.set_latency_threads(args.latency_threads)
    montlok.set_devices(args.devices)
    try:
        model = montlok.load(args.model)
        rows = np.random.default_rng(7).standard_normal((args.rows, args.batch * model.features))
        if args.memory == "device":
            samples, mean = bench_device(model, rows, args.batch, args.iterations)
        else:
            if args.memory == "pinned":
                import torch

                rows = torch.from_numpy(rows).pin_memory().numpy()
            samples, mean = montlok._core.bench(model, rows, args.batch, args.iterations, args.stream)
    finally:
        montlok.set_latency_threads(0)
    p50, p90, p99, p999 = np.percentile(samples, [50, 90, 99, 99.9])
    call = "stream step" if args.stream else "predict"
    print(f"{args.model}: {call}, batch {args.batch}, {args.memory} memory, {args.threads} thread(s), "
          f"{args.latency_threads} latency thread(s), {args.iterations} calls")
    print(f"p50 {_ns(p50)}  p90 {_ns(p90)}  p99 {_ns(p99)}  p99.9 {_ns(p999)}  mean {_ns(mean)}")
    print(f"{1e9 / mean:,.0f} calls/s, {args.batch * 1e9 / mean:,.0f} rows/s")
    return 0


def cmd_env(args: argparse.Namespace) -> int:
    info = montlok.build_info()
    rows = [("montlok", f"{info['version']} (C ABI {info['abi']})"),
            ("python", f"{info['python']} ({info['machine']})"), ("cpu", f"{os.cpu_count()} hardware threads"),
            ("families", ", ".join(info["families"])), ("gpus", f"{info['device_count']} visible, "
                                                                f"{info['devices'] or 'current'} used"),
            ("threads", f"{info['threads']} staging, {info['latency_threads']} latency")]
    width = max(len(name) for name, _ in rows)
    for name, value in rows:
        print(f"{name:<{width}}  {value}")
    return 0


def parser() -> argparse.ArgumentParser:
    root = argparse.ArgumentParser(prog="montlok", description="Tree-ensemble models on NVIDIA B200 GPUs.")
    root.add_argument("--version", action="version", version=f"montlok {montlok.__version__}")
    commands = root.add_subparsers(dest="command", required=True, metavar="COMMAND")
    p = commands.add_parser("info", help="what a model file holds")
    p.add_argument("model")
    p.add_argument("--json", action="store_true", help="print the full spec")
    p.set_defaults(run=cmd_info)
    p = commands.add_parser("convert", help="scikit-learn trees or a LightGBM dump -> .montlok")
    p.add_argument("source")
    p.add_argument("-o", "--output", required=True)
    p.add_argument("--feature-names", help="comma-separated names stored in the model")
    p.set_defaults(run=cmd_convert)
    p = commands.add_parser("predict", help="predictions for a CSV/NPY file")
    p.add_argument("model")
    p.add_argument("input", help="CSV (header optional), .npy or .npz")
    p.add_argument("-o", "--output", help="CSV or .npy (default: CSV on stdout)")
    p.add_argument("--threads", type=int, default=0, help="host staging threads (default: one per hardware thread)")
    p.add_argument("--devices", type=int, default=0, help="GPUs the rows are split over (default: the current one)")
    p.set_defaults(run=cmd_predict)
    p = commands.add_parser("bench", help="in-process latency of one model")
    p.add_argument("model")
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--iterations", type=int, default=20000)
    p.add_argument("--rows", type=int, default=1024, help="distinct random inputs used in turn")
    p.add_argument("--threads", type=int, default=1)
    p.add_argument("--latency-threads", type=int, default=0)
    p.add_argument("--stream", action="store_true", help="time stream steps (stateless for trees)")
    p.add_argument("--memory", choices=("host", "pinned", "device"), default="host",
                   help="where inputs and outputs live: pageable host, pinned host, or GPU (predict_device)")
    p.add_argument("--devices", type=int, default=0, help="GPUs host batches are split over (default: the current one)")
    p.set_defaults(run=cmd_bench)
    p = commands.add_parser("env", help="versions, GPUs and settings")
    p.set_defaults(run=cmd_env)
    return root


def main(argv: Sequence[str] | None = None) -> int:
    args = parser().parse_args(argv)
    return args.run(args)


if __name__ == "__main__":
    sys.exit(main())
