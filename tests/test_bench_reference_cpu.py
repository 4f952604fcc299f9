"""``bench.py --impl reference`` on CPU: the reference arm times the oracle
(the reference's CPU algorithm, restated) and prints one JSON line with the
same metric, unit and workload as the GPU arm.  Under torchrun only rank 0
works; the other ranks exit 0 without output.
"""

import json
import os
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                          cwd=REPO, env=env, capture_output=True, text=True, timeout=300)


def test_reference_arm_line():
    res = _run({"RANK": "0", "WORLD_SIZE": "1"})
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "tok/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["steps"] == 1 and line["warmup"] == 3
    assert line["config"]["workload"] == "mixtral8x7b_moe_layer_decode" and line["config"]["tokens"] == 64
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    res = _run({"RANK": "1", "WORLD_SIZE": "2"})
    assert res.returncode == 0, res.stderr[-2000:]
    assert res.stdout.strip() == ""


def test_reference_arm_expert_parallel_config():
    """Under --gpus N > 1 the GPU arm measures config 4 (GLM-4.5-Air layer,
    32 sequences per GPU), and so does the reference arm."""
    env = dict(os.environ, RANK="0", WORLD_SIZE="2")
    res = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1",
                          "--warmup", "3", "--ref-budget", "1"], cwd=REPO, env=env, capture_output=True, text=True,
                         timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["n_gpus"] == 2 and line["value"] > 0
    assert line["config"]["workload"] == "glm45air_moe_layer_decode_ep" and line["config"]["experts"] == 128
    assert line["cpu_baseline"]["value"] == line["value"] and "touched experts" in line["cpu_baseline"]["sample"]
