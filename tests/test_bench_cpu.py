"""The bench's reference arm, as the round-end driver launches it, on the CPU.

`bench.py --impl reference` times the CPU oracle on a bounded sample of the headline workload
(no GPU involved) and must print ONE JSON line with the same metric, unit and `config` as the
native arm, plus `impl`, `cpu_baseline` and an `e2e` object with no host-device traffic. Under
torchrun only rank 0 runs it; the other ranks exit 0 without work.
"""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys

import pytest

from conftest import ROOT

CONTRACT_KEYS = {
    "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
    "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e",
}


def _json_lines(stdout: str) -> list[dict]:
    return [json.loads(s) for s in stdout.splitlines() if s.startswith("{")]


def _check_reference_line(line: dict, n_gpus: int) -> None:
    import bench
    from rtgs_b200.image2gs.synthetic import WORKLOADS

    assert CONTRACT_KEYS <= set(line), CONTRACT_KEYS - set(line)
    assert line["impl"] == "reference"
    assert line["metric"] == "2D-gaussian image fits/sec" and line["unit"] == "fits/s"
    assert line["higher_is_better"] is True and line["n_gpus"] == n_gpus
    assert line["value"] > 0 and line["ms_per_step"] > 0
    # The same config object as the native arm's line for this workload.
    wl = WORKLOADS["single_large"]
    assert line["config"] == bench.workload_config("single_large", dict(wl), 1, n_gpus)
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def _cpu_env() -> dict:
    env = dict(os.environ)
    env["CUDA_VISIBLE_DEVICES"] = ""
    return env


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                       cwd=ROOT, env=_cpu_env(), capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1, r.stdout[-2000:]
    _check_reference_line(lines[0], n_gpus=1)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(900)
def test_reference_arm_under_torchrun_prints_once_from_rank_0():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0"]
    r = subprocess.run(cmd, cwd=ROOT, env=_cpu_env(), capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1, r.stdout[-2000:]
    _check_reference_line(lines[0], n_gpus=2)
