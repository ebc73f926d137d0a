"""bench.py's reference arm, which runs on the host cores: the one-line JSON
contract a benchmark harness reads (one line on stdout, its keys, the
reference-arm fields), without a GPU.

The reference arm times the numpy oracle (the CPU restatement of the
reference's path) on a bounded sample of the C2 workload.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args: str) -> dict:
    res = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *args],
                         capture_output=True, text=True, timeout=600, cwd=REPO)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, res.stdout
    return json.loads(lines[0])


@pytest.mark.parametrize("op", ["attention", "topk", "indexer", "cache_write"])
def test_reference_arm_prints_one_contract_line(op):
    d = _run("--impl", "reference", "--op", op, "--steps", "3", "--warmup", "3", "--cpu-seconds", "1")
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in d, key
    assert d["n_gpus"] == 1 and d["steps"] == 3 and d["warmup"] == 3
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["higher_is_better"] is True
    # a step is one batch of the op's units (query tokens, rows or cache tokens)
    per_step = d["value"] * d["ms_per_step"] / 1e3
    assert per_step == pytest.approx(round(per_step), rel=1e-3) and round(per_step) >= 1
    assert "workload" in d["config"]
    cpu = d["cpu_baseline"]
    assert cpu["value"] == d["value"] and cpu["unit"] == d["unit"]
    assert cpu["kind"] in ("port", "reference") and cpu["cores"] >= 1 and cpu["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


_MAPPED = r"""
import runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "2", "--warmup", "3"]
runpy.run_path("bench.py", run_name="__main__")
maps = open("/proc/self/maps").read()
libs = sorted({ln.split()[-1] for ln in maps.splitlines() if "glm53" in ln})
print("MAPPED " + ";".join(libs) + " PKG " + str("glm53_sparse_mla" in sys.modules))
"""


def test_reference_arm_maps_no_repo_library_and_keeps_the_config():
    """The attention reference arm times the CPU restatement only: it maps no
    shared library of this repository (the package import would load the CUDA
    extension), and its config carries the keys the repository's arm prints
    for the same arguments."""
    res = subprocess.run([sys.executable, "-c", _MAPPED], capture_output=True, text=True,
                         timeout=600, cwd=REPO)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.strip()]
    line = json.loads(lines[0])
    tail = lines[-1]
    assert tail.startswith("MAPPED "), tail
    libs, pkg = tail[len("MAPPED "):].split(" PKG ")
    assert libs == "", libs
    assert pkg == "False"
    cfg = line["config"]
    for key in ("workload", "parallelism", "l2", "timing", "splits", "allgather"):
        assert key in cfg, key
    assert cfg["parallelism"] == "dp1" and cfg["splits"] == "auto" and cfg["allgather"] is False
