"""`bench.py --impl reference` on CPU: the reference arm times the CPU reference of the path (the oracle port) and
prints one JSON line with our arm's metric, unit, direction and config-5 workload, a cpu_baseline describing its
bounded sample and an e2e figure with no host<->device bytes; under torchrun only rank 0 runs and prints. The arm
loads the oracle's library and nothing of the product (no liblrmcuda.so)."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CMD = [sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1", "--context", "64"]


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run(CMD, cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)


def test_reference_arm_line():
    sys.path.insert(0, ROOT)
    import bench

    r = _run({"RANK": "0", "WORLD_SIZE": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "tok/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["steps"] == 1 and line["warmup"] == 1
    assert line["config"] == bench.decode_config(64, 64, 1, 28)
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_reference_arm_loads_no_product_library():
    # Run the arm in a process that then lists the shared objects it mapped.
    code = ("import runpy, sys; sys.argv = " + repr(["bench.py"] + CMD[2:]) + "; "
            "runpy.run_path('bench.py', run_name='__main__'); "
            "print('MAPS:' + '|'.join(sorted({l.split()[-1] for l in open('/proc/self/maps') "
            "if l.rstrip().endswith('.so')})))")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=dict(os.environ, RANK="0", WORLD_SIZE="1"),
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    maps = [ln for ln in r.stdout.splitlines() if ln.startswith("MAPS:")][0][5:].split("|")
    ours = [m for m in maps if m.startswith(ROOT)]
    assert any(m.endswith("oracle/_build/liblrm_oracle.so") for m in ours), ours
    assert not any("rosylnalive_b200" in m for m in ours), ours
