"""The `montlok` command line (python -m montlok): info, convert, env and the
argument surface on CPU; predict and bench (host, pinned and device memory)
on a GPU."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from forests import random_model, same_bits
from golden.make_golden import lightgbm_dump
from montlok import cli, export

ROOT = Path(__file__).resolve().parents[1]


def run(*argv: str) -> subprocess.CompletedProcess:
    env = {"PYTHONPATH": str(ROOT / "montlok.cpp_b200" / "python"), "PATH": "/usr/bin:/bin"}
    return subprocess.run([sys.executable, "-m", "montlok", *argv], capture_output=True, text=True, env=env,
                          timeout=300)


def test_info_and_convert(tmp_path):
    dump = tmp_path / "model.json"
    dump.write_text(json.dumps(lightgbm_dump("multiclass num_class:3", 3, 12, 5, seed=4)))
    out = tmp_path / "model.montlok"
    r = run("convert", str(dump), "-o", str(out))
    assert r.returncode == 0, r.stderr
    assert out.exists() and "tree_ensemble" in r.stdout
    r = run("info", str(out))
    assert r.returncode == 0, r.stderr
    assert "features" in r.stdout
    r = run("info", str(out), "--json")
    assert json.loads(r.stdout)["family"] == "tree_ensemble"


def test_env_runs_without_a_gpu():
    r = run("env")
    assert r.returncode == 0 and "montlok" in r.stdout and "gpus" in r.stdout


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
