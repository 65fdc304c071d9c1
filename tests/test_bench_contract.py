"""bench.py's reference arm on the host (no GPU): the JSON line it prints
carries the keys the benchmark contract asks for, and under a multi-rank
launch only rank 0 works and prints.  Run on a 4-view layer so that the
oracle finishes in seconds."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--frames", "4",
                           "--steps", "1", "--warmup", "0"], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=240)


def test_reference_arm_line():
    p = _run({})
    assert p.returncode == 0, p.stderr[-2000:]
    line = json.loads(p.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "views/s"
    assert line["n_gpus"] == 1 and line["steps"] == 1 and line["warmup"] == 0
    assert line["higher_is_better"] is True and line["data"] == "synthetic"
    assert "workload" in line["config"]
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["unit"] == line["unit"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_exit_quietly():
    p = _run({"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert p.returncode == 0, p.stderr[-2000:]
    assert p.stdout.strip() == ""


def test_clock_sampler_covers_a_short_region(tmp_path, monkeypatch):
    """The clock sampler waits for nvidia-smi's first sample before the timed
    region starts, so that a region of a few tens of milliseconds (a short
    multi-GPU step) still holds samples; samples outside the region do not
    count.  A stand-in nvidia-smi that starts slowly and prints a line every
    10 ms."""
    fake = tmp_path / "nvidia-smi"
    fake.write_text("#!/bin/bash\nsleep 0.3\nwhile true; do echo \"0, 1800, 1965, 500.0, 0x4, Not Active, "
                    "Not Active, Not Active, Active\"; sleep 0.01; done\n")
    fake.chmod(0o755)
    monkeypatch.setenv("PATH", f"{tmp_path}:{os.environ['PATH']}")
    sys.path.insert(0, ROOT)
    import time
    import bench

    with bench.Clocks(0) as c:
        time.sleep(0.03)
    s = c.summary()
    assert 1 <= s["samples"] <= 8, s
    assert s["sm_mhz"] == 1800.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]
