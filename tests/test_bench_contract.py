"""The benchmark's JSON line on the CPU: ``bench.py --impl reference`` (the
reference arm: the oracle's restatement of the packed forward around the
reference's own C kernels) on the tiny configuration prints one line whose keys,
units and metric string are the ones the GPU arm prints for the same config,
so the two arms' values can be compared."""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def _bench_module():
    spec = importlib.util.spec_from_file_location("bench_contract_mod", REPO / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_reference_arm_line_matches_the_contract():
    out = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--config", "tiny",
                          "--steps", "2", "--warmup", "3"],
                         cwd=REPO, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["unit"] == "tok/s" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["steps"] == 2 and d["warmup"] >= 3
    assert isinstance(d["config"], dict) and "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert cb["unit"] == d["unit"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    # the GPU arm's metric string for the same configuration
    bench = _bench_module()
    assert d["metric"] == bench.metric_name(argparse.Namespace(config="tiny", policy="sg8"))


def test_reference_arm_under_torchrun_prints_one_line_from_rank_zero():
    """The driver launches the reference arm at N > 1 through torchrun as well:
    rank 0 alone times the CPU implementation and prints the line (n_gpus = N,
    all host threads), the other ranks exit 0 without work."""
    out = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                          "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(REPO / "bench.py"),
                          "--impl", "reference", "--gpus", "2", "--config", "tiny", "--steps", "2", "--warmup", "3"],
                         cwd=REPO, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
    # torchrun exports OMP_NUM_THREADS=1 to every rank; the arm must still use the host's threads
    assert d["cpu_baseline"]["cores"] >= 1
    if len(os.sched_getaffinity(0)) > 1:
        assert d["cpu_baseline"]["cores"] > 1


def _free_port() -> int:
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]
