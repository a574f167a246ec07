"""CPU checks of bench.py's reference arm (`--impl reference`), which times the
oracle's restatement of the reference algorithm on the host cores: one JSON
line with the contract's keys, its numbers consistent with each other, and
no work on ranks other than 0.  Runs on a small seeded workload in seconds."""
import json
import os
import subprocess
import sys

from conftest import REPO


def _run(args, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *args], cwd=REPO, env=env,
                          capture_output=True, text=True, timeout=300)


def test_reference_arm_prints_one_consistent_line():
    steps, warmup = 2, 1
    r = _run(["--impl", "reference", "--workload", "small_T64", "--steps", str(steps), "--warmup", str(warmup),
              "--cpu-budget", "0.5"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, lines
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["steps"] == steps and d["warmup"] == warmup and d["n_gpus"] == 1
    assert d["higher_is_better"] is True and d["value"] > 0
    assert d["config"]["workload"] == "small_T64"
    cb = d["cpu_baseline"]
    assert set(cb) >= {"value", "unit", "cores", "kind", "sample"}
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == d["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0
    s = d["sample"]
    assert s["steps_timed"] == steps
    assert abs(d["ms_per_step"] - 1e3 * s["seconds_per_step"]) < 1e-6
    # value = tokens x sampled rows / routed rows per second of the timed sample
    tokens = d["config"]["tokens_per_gpu"]
    expect = tokens * (s["sample_rows"] / s["routed_rows"]) / s["seconds_per_step"]
    assert abs(d["value"] - expect) <= 1e-6 * expect


def test_reference_arm_other_ranks_exit_without_work():
    r = _run(["--impl", "reference", "--workload", "small_T64", "--steps", "1", "--warmup", "0"],
             {"WORLD_SIZE": "2", "RANK": "1", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
