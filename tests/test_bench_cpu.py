"""The benchmark's reference arm on the CPU (no GPU): one JSON line with the
keys the bench contract names, the same `config` as the CUDA arm would print,
and no native library in the process but the oracle's -- the reference arm
times the oracle and must not map the CUDA library."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_RUN = """
import runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0", "--prompt-len", "8",
            "--new-tokens", "4", "--cpu-seconds", "0.5"]
runpy.run_path("bench.py", run_name="__main__")
maps = open("/proc/self/maps").read()
print("MAPS", int("libkrikil_cuda" in maps), int("liboracle" in maps))
"""


def test_reference_arm_line_and_loaded_libraries():
    env = dict(os.environ, OMP_NUM_THREADS="2")
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    out = subprocess.run([sys.executable, "-c", _RUN], cwd=ROOT, env=env, capture_output=True, text=True,
                         timeout=300, check=True).stdout.strip().splitlines()
    line = json.loads(out[-2])
    assert out[-1] == "MAPS 0 1"  # the oracle only, never the CUDA library
    assert line["impl"] == "reference" and line["unit"] == "tokens/s" and line["value"] > 0
    assert line["higher_is_better"] is True and line["n_gpus"] == 1 and line["steps"] == 1
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["value"] == line["value"] and cb["cores"] >= 1 and cb["sample"]
    cfg = line["config"]
    assert cfg["seqs_total"] == 1024 and cfg["seqs_per_gpu"] == 1024 and cfg["prompt_len"] == 8
    assert cfg["new_tokens"] == 4 and cfg["parallelism"] == "replicas x1 (no collectives)"


def test_reference_arm_other_ranks_exit_without_work():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2")
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1",
                        "--warmup", "3"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == ""
