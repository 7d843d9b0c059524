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


def test_reference_arm_times_every_layer_of_every_step():
    """--impl reference: the CPU restatement over whole steps (all layers),
    one JSON line with the contract's keys; the time it claims fits in the
    wall time it took."""
    import time
    t0 = time.time()
    d = _run("--impl", "reference", "--layers", "2", "--steps", "2", "--warmup", "1",
             "--tokens", "8")
    wall = time.time() - t0
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["value"] > 0
    assert d["config"]["n_layer"] == 2 and d["config"]["tokens"] == 8
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert "every step whole: 2 layers" in d["cpu_baseline"]["sample"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0
    assert d["steps"] * d["ms_per_step"] / 1e3 < wall


def test_prefill_workload_is_one_gpu_only():
    d = _run("--workload", "prefill", "--gpus", "2")
    assert d["workload"] == "prefill" and "unavailable" in d


def test_single_op_workload_is_one_gpu_only():
    d = _run("--workload", "single-op", "--gpus", "2")
    assert d["workload"] == "single-op" and "unavailable" in d
