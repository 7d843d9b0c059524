"""bench.py on CPU: the streamed workload refuses configurations it does not
run with one JSON line (the driver's arms are exercised on the GPU box)."""
import json
import os
import subprocess
import sys

from tests.conftest import ROOT


def _run(*args, timeout=600):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT,
                         env=env, capture_output=True, text=True, timeout=timeout)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def test_streamed_workload_is_one_gpu_only():
    d = _run("--workload", "streamed", "--gpus", "2")
    assert d["workload"] == "streamed" and "unavailable" in d


def test_slots_workload_is_one_gpu_only():
    d = _run("--workload", "slots", "--gpus", "4")
    assert d["workload"] == "slots" and "unavailable" in d
