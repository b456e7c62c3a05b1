"""The `montlok` command line (python -m montlok): the argument surface and
table reading on CPU; predict and bench (host, pinned and device memory) on
a GPU."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from forests import random_model, same_bits
import montlok
from montlok import cli, export

ROOT = Path(__file__).resolve().parents[1]


def run(*argv: str) -> subprocess.CompletedProcess:
    env = {"PYTHONPATH": str(ROOT / "montlok.cpp_b200" / "python"), "PATH": "/usr/bin:/bin"}
    return subprocess.run([sys.executable, "-m", "montlok", *argv], capture_output=True, text=True, env=env,
                          timeout=300)


def test_version_without_a_gpu():
    r = run("--version")
    assert r.returncode == 0 and "montlok" in r.stdout


def test_csv_tables_match_columns_by_name(tmp_path):
    """A CSV header is matched against the model's feature names."""
    model = montlok.load(export.tree_ensemble(_nodes(), [0], [0], features=3,
                                              feature_names=["a", "b", "c"]).to_bytes())
    path = tmp_path / "x.csv"
    path.write_text("c,a,b\n3,1,2\n6,4,\n")
    table, names = cli._table(path)
    assert names == ["c", "a", "b"]
    x = cli._arrange(model, table, names)
    np.testing.assert_array_equal(x[0], [1.0, 2.0, 3.0])
    assert np.isnan(x[1, 1]) and x[1, 0] == 4.0 and x[1, 2] == 6.0


def _nodes():
    nodes = export.Nodes()
    root = nodes.add(feature=0, threshold=0.5, flags=1 | (1 << 1))
    nodes.left[root] = nodes.add(value=1.0)
    nodes.right[root] = nodes.add(value=2.0)
    return nodes


def test_bench_and_predict_options_parse():
    args = cli.parser().parse_args(["bench", "m.montlok", "--memory", "device", "--devices", "2", "--batch", "64"])
    assert (args.memory, args.devices, args.batch) == ("device", 2, 64)
    args = cli.parser().parse_args(["predict", "m.montlok", "x.npy", "--devices", "4"])
    assert args.devices == 4
    with pytest.raises(SystemExit):
        cli.parser().parse_args(["bench", "m.montlok", "--memory", "disk"])


@pytest.mark.gpu
def test_predict_matches_the_oracle(gpu, tmp_path):
    from oracle import Oracle

    rng = np.random.default_rng(3)
    model = random_model(rng, features=4, trees=50, outputs=3, link="softmax")
    (tmp_path / "m.montlok").write_bytes(model)
    x = rng.normal(size=(77, 4))
    np.save(tmp_path / "x.npy", x)
    r = run("predict", str(tmp_path / "m.montlok"), str(tmp_path / "x.npy"), "-o", str(tmp_path / "y.npy"))
    assert r.returncode == 0, r.stderr
    assert same_bits(np.load(tmp_path / "y.npy").reshape(77, 3), Oracle(model).predict(x))


@pytest.mark.gpu
@pytest.mark.parametrize("memory", ["host", "pinned", "device"])
def test_bench_memory_modes(gpu, tmp_path, memory):
    rng = np.random.default_rng(4)
    (tmp_path / "m.montlok").write_bytes(random_model(rng, features=6, trees=80))
    r = run("bench", str(tmp_path / "m.montlok"), "--batch", "8", "--iterations", "300", "--rows", "16", "--memory",
            memory)
    assert r.returncode == 0, r.stderr
    assert f"{memory} memory" in r.stdout and "p50" in r.stdout
    r = run("bench", str(tmp_path / "m.montlok"), "--batch", "8", "--iterations", "100", "--memory", memory, "--json")
    assert r.returncode == 0, r.stderr
    report = json.loads(r.stdout)
    assert report["memory"] == memory and report["p50_us"] > 0 and report["kernel"]
