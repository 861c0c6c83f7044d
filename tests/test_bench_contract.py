"""bench.py's reference arm (the oracle's restatement of the forward, timed
on the host cores) prints the one JSON line the benchmark contract asks for,
with the same metric, unit and config as the GPU arm; under torchrun only
rank 0 runs it. No GPU needed: these run in the CPU suite."""
import json
import os
import subprocess
import sys

from conftest import ROOT


def _run(extra_env):
    env = dict(os.environ)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        env.pop(k, None)
    env.update(extra_env)
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]


def test_reference_arm_line():
    sys.path.insert(0, ROOT)
    import bench
    lines = _run({})
    assert len(lines) == 1
    d = lines[0]
    assert d["impl"] == "reference"
    assert (d["metric"], d["unit"], d["higher_is_better"]) == (bench.METRIC, bench.UNIT, True)
    assert d["config"] == bench.config(1)
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 0
    assert d["value"] > 0 and d["ms_per_step"] > 0
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert cb["unit"] == d["unit"] and cb["sample"]
    e = d["e2e"]
    assert e == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_silent():
    """A rank other than 0 exits 0 without work or output."""
    assert _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}) == []


def test_reference_arm_config_follows_world():
    """Rank 0 of an N-process launch reports the config of the N-GPU line."""
    sys.path.insert(0, ROOT)
    import bench
    d = _run({"RANK": "0", "WORLD_SIZE": "2", "LOCAL_RANK": "0"})[0]
    assert d["config"] == bench.config(2) and d["n_gpus"] == 2
