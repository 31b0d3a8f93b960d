"""The C++ mirror of the reference's Rust API (include/krikil.hpp), compiled
with g++ and driven like the reference's own tests (tests/cpp/test_api.cpp).
On a machine without a GPU the loader checks run and the program reports 77;
on a GPU its prefill/step logits and generated streams are checked against the
oracle."""
import os
import shutil
import subprocess

import numpy as np
import pytest

import oracle as O
from krikil_rs_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "krikil_rs_b200", "lib")


@pytest.fixture(scope="module")
def binary(tmp_path_factory):
    if not shutil.which("g++"):
        pytest.skip("no g++")
    exe = str(tmp_path_factory.mktemp("cpp") / "test_api")
    subprocess.run(["g++", "-std=c++17", "-O2", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "cpp", "test_api.cpp"), "-L", LIBDIR, "-lkrikil_cuda",
                    f"-Wl,-rpath,{LIBDIR}", "-o", exe], check=True)
    return exe


def _run(binary, tmp_path):
    out = str(tmp_path / "out.bin")
    tok = os.path.join(ROOT, "tests", "golden", "tokenizer_small.json")
    p = subprocess.run([binary, synth.weights_file(0), out, tok], capture_output=True, text=True, timeout=600)
    return p, out


def test_cpp_api_compiles_and_loader_errors(binary, tmp_path):
    p, _ = _run(binary, tmp_path)
    assert p.returncode in (0, 77), p.stdout + p.stderr


@pytest.mark.gpu
def test_cpp_api_matches_oracle(binary, tmp_path):
    p, out = _run(binary, tmp_path)
    assert p.returncode == 0, p.stdout + p.stderr
    buf = np.fromfile(out, np.uint8)
    f = buf[:2 * 2048 * 4].view(np.float32)
    rest = buf[2 * 2048 * 4:].view(np.uint32)
    ng = int(rest[0])
    greedy = rest[1:1 + ng].tolist()
    ns = int(rest[1 + ng])
    sampled = rest[2 + ng:2 + ng + ns].tolist()
    prompt = [(i * 397 + 11) % 2048 for i in range(12)]
    orc = O.OracleModel(synth.load_safetensors(synth.weights_file(0)))
    st = O.OracleState(64)
    np.testing.assert_allclose(f[:2048], O.forward_prefill(orc, st, prompt), atol=1e-4, rtol=1e-5)
    np.testing.assert_allclose(f[2048:], O.forward_step(orc, st, 199), atol=1e-4, rtol=1e-5)
    ref, _ = O.generate_greedy(orc, O.OracleState(64), prompt, 10, repetition_penalty=1.2, eos=0)
    assert greedy == ref
    assert sampled == O.generate_sample(orc, O.OracleState(64), prompt, 10, 0.7, 0.95, 50, 1.2, 42, eos=0)
