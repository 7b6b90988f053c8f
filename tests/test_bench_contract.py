"""bench.py's reference arm on CPU: one JSON line with the contract's keys,
the cpu_baseline block and an e2e block, for the default config and for the
other MLP configs (`--config`).  The GPU arm is exercised on a B200."""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
        "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
        "cpu_baseline", "e2e"}


@pytest.mark.parametrize("config", ["c0", "c2"])
def test_reference_arm_prints_one_contract_line(config):
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "0", "--config", config],
                         capture_output=True, text=True, timeout=600, cwd=REPO,
                         env=dict(os.environ, WORLD_SIZE="1", RANK="0"))
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert KEYS <= set(d)
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "samples/s"
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
    assert f"configs[{config[1:]}]" in d["config"]["workload"]
    if config == "c2":
        assert d["metric"].startswith("train samples/s, MLP 784-8192-8192-10")


def test_reference_arm_non_zero_rank_exits_quietly():
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "0"], capture_output=True, text=True,
                         timeout=300, cwd=REPO, env=dict(os.environ, WORLD_SIZE="2", RANK="1"))
    assert out.returncode == 0 and not out.stdout.strip()


def test_reference_arm_at_two_gpus_times_the_socket_exchange():
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "0", "--gpus", "2", "--config", "c0"],
                         capture_output=True, text=True, timeout=600, cwd=REPO,
                         env=dict(os.environ, WORLD_SIZE="2", RANK="0"))
    assert out.returncode == 0, out.stderr[-2000:]
    d = json.loads([ln for ln in out.stdout.splitlines() if ln.startswith("{")][0])
    ddp = d["cpu_baseline"]["socket_ddp"]
    assert ddp["world"] == 2 and ddp["kind"] == "port"
    assert ddp["sample_s"] > 0 and ddp["per_step_s"] > ddp["sample_s"] * 0.5
