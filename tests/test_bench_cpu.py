"""CPU tests of bench.py's reference arm: the JSON line keeps the contract the driver reads
(one line, the metric keys, `impl`, `cpu_baseline`, `e2e`) for every workload, and the
non-zero ranks of a torchrun launch print nothing and exit 0."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"}


def _run(args, env=None):
    out = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", *args], cwd=REPO,
                         capture_output=True, text=True, timeout=600, env=env)
    assert out.returncode == 0, out.stderr[-2000:]
    return out.stdout.strip().splitlines()


@pytest.mark.parametrize("workload", ["gemv", "gemm", "attn", "head", "ple"])
def test_reference_line_contract(workload):
    lines = _run(["--workload", workload, "--steps", "1", "--warmup", "3"])
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert KEYS <= set(d), KEYS - set(d)
    assert d["impl"] == "reference" and d["value"] > 0 and d["warmup"] >= 3
    cb = d["cpu_baseline"]
    assert {"value", "unit", "cores", "kind", "sample"} <= set(cb) and cb["kind"] in ("port", "reference")
    assert cb["value"] == d["value"] and d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


def test_serve_reference_line_is_the_gpu_arms_config():
    """The config-5 reference arm times the whole 256-sequence batch and reports the GPU
    arm's own metric and config object (like-for-like)."""
    sys.path.insert(0, str(REPO))
    import bench
    lines = _run(["--workload", "serve", "--steps", "1", "--warmup", "3"])
    d = json.loads(lines[0])
    assert KEYS <= set(d)
    assert d["metric"] == bench.SERVE_METRIC and d["config"] == bench.serve_config(1)
    assert d["unit"] == "tok/s" and d["value"] > 0 and "256 sequences" in d["cpu_baseline"]["sample"]


def test_reference_arm_other_ranks_are_silent():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    assert _run(["--workload", "gemv", "--steps", "1", "--warmup", "3"], env=env) == []
