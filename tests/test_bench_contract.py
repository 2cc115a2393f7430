"""What bench.py must do without a GPU: refuse more than one GPU with exit code 2 and one line, and answer for the
reference arm with one JSON line that says why the reference cannot run here."""

import json
import os
import subprocess
import sys

from conftest import ROOT


def run(*args):
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                          cwd=ROOT)


def test_more_than_one_gpu_is_refused_with_one_line_and_exit_code_2():
    proc = run("--gpus", "2", "--steps", "2", "--warmup", "1")
    assert proc.returncode == 2
    lines = [l for l in proc.stdout.split("\n") if l.strip()]
    assert len(lines) == 1 and "one GPU" in lines[0] and "--gpus 2" in lines[0]


def test_the_reference_arm_says_why_it_is_unavailable():
    proc = run("--impl", "reference", "--gpus", "1", "--steps", "2", "--warmup", "1")
    assert proc.returncode == 0, proc.stderr[-1000:]
    lines = [l for l in proc.stdout.split("\n") if l.strip()]
    assert len(lines) == 1
    record = json.loads(lines[0])
    assert record["impl"] == "reference" and isinstance(record["unavailable"], str) and record["unavailable"]
    assert "\n" not in record["unavailable"]
