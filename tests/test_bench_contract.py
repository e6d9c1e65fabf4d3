"""bench.py's command-line contract on the host (no GPU): the reference arm prints one JSON line with the keys
the driver reads, on rank 0 only, on the same workload string as this repo's own arm; this repo's arm fails
loudly without a GPU instead of timing a fallback."""
import json
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
             "vs_baseline", "dtype", "data", "config"}


def _bench(args, env_extra=None, timeout=300):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=timeout)


def test_reference_arm_prints_one_contract_line():
    r = _bench(["--impl", "reference", "--steps", "1", "--warmup", "1"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert BASE_KEYS <= set(line)
    assert line["impl"] == "reference" and line["n_gpus"] == 1 and line["steps"] == 1
    assert line["higher_is_better"] is True and line["value"] > 0
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["unit"] == line["unit"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    # the driver compares the two arms on the same workload, metric and unit
    sys.path.insert(0, ROOT)
    import bench as B
    assert line["metric"] == B.METRIC
    assert line["config"]["workload"] == B.stack_workload(B.SHAPE["E"], 1)


def test_reference_arm_is_silent_on_other_ranks():
    r = _bench(["--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1"],
               env_extra={"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


@pytest.mark.skipif(torch.cuda.is_available(), reason="this host has a GPU: the arm would run for real")
def test_own_arm_fails_loudly_without_a_gpu():
    r = _bench(["--steps", "1", "--warmup", "3"])
    assert r.returncode != 0
    assert not any(l.startswith("{") for l in r.stdout.splitlines())
