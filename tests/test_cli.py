"""The krikil command line (src/main.rs on the GPU library): option parsing,
error reports and exit codes on the CPU; on a GPU, the streamed text of a
greedy and a seeded sampling run against the oracle's token streams decoded
with the tokenizer."""
import os
import subprocess

import pytest

from krikil_rs_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "krikil_rs_b200", "bin", "krikil")
SMALL_TOK = os.path.join(ROOT, "tests", "golden", "tokenizer_small.json")


def run(*args, cwd=None):
    if not os.path.exists(EXE):
        pytest.fail(f"{EXE} is missing: build it with make -C krikil_rs_b200")
    return subprocess.run([EXE, *args], capture_output=True, text=True, timeout=600, cwd=cwd)


def test_help_version_and_usage_errors():
    p = run("--help")
    assert p.returncode == 0 and "--repetition-penalty" in p.stdout and "[default: 0.7]" in p.stdout
    assert run("-V").stdout.strip() == "krikil 0.1.0"
    p = run()
    assert p.returncode == 2 and "<PROMPT>" in p.stderr
    p = run("--top-k", "x", "hi")
    assert p.returncode == 2 and "invalid value 'x' for '--top-k'" in p.stderr
    p = run("--bogus", "hi")
    assert p.returncode == 2 and "unexpected argument '--bogus'" in p.stderr
    p = run("a", "b")
    assert p.returncode == 2


def test_front_end_errors(tmp_path):
    # tokenizer resolution (src/tokenizer.rs:54-79) happens before the model loads
    p = run("-m", str(tmp_path / "model.safetensors"), "hi", cwd=str(tmp_path))
    assert p.returncode == 1
    assert p.stderr.startswith("Error: Could not find tokenizer.json. Looked at ")
    p = run("--tokenizer", str(tmp_path / "t.json"), "hi")
    assert p.returncode == 1 and f"Explicit tokenizer path not found: {tmp_path}/t.json" in p.stderr
    bad = tmp_path / "tokenizer.json"
    bad.write_text("{")
    p = run("-m", str(tmp_path / "model.safetensors"), "hi")
    assert p.returncode == 1 and p.stderr.startswith(f"Error: Failed to load tokenizer from {bad}\n\nCaused by:")
    p = run("-m", str(tmp_path / "model.safetensors"), "--tokenizer", SMALL_TOK, "hi")
    assert p.returncode == 1 and p.stderr.startswith(f"Error: Failed to load model from {tmp_path}/model.safetensors")
    assert "Failed to open model file" in p.stderr
    p = run("--template", str(tmp_path / "none.jinja"), "--tokenizer", SMALL_TOK, "hi")
    assert p.returncode == 1 and "Failed to read chat template from" in p.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["greedy", "sample"])
def test_cli_generates_the_oracle_stream(mode, tmp_path):
    import oracle as O
    from krikil_rs_b200.text import ChatTemplateEngine, PebbleTokenizer

    weights = synth.weights_file(0)
    tok = PebbleTokenizer.from_file(SMALL_TOK)
    prompt = "What is the capital of France?"
    ids = tok.encode(ChatTemplateEngine.default_template().render_user_prompt(prompt))
    orc = O.OracleModel(synth.load_safetensors(weights))
    if mode == "greedy":
        args = ["--temp", "0"]
        ref, _ = O.generate_greedy(orc, O.OracleState(256), ids, 24, repetition_penalty=1.2, eos=0)
    else:
        args = ["--seed", "7"]  # temperature 0.7, top-p 0.95, top-k 50 (the defaults)
        ref = O.generate_sample(orc, O.OracleState(256), ids, 24, 0.7, 0.95, 50, 1.2, 7, eos=0)
    p = run("-m", weights, "--tokenizer", SMALL_TOK, "--context", "256", "--max-tokens", "24", *args, prompt)
    assert p.returncode == 0, p.stderr
    assert p.stdout == "".join(tok.decode_token(t) for t in ref) + "\n"
    assert f"[Prompt: {len(ids)} tokens, Generated: {len(ref)} tokens" in p.stderr
    q = run("-m", weights, "--tokenizer", SMALL_TOK, "--context", "256", "--max-tokens", "24", "--quiet", *args,
            prompt)
    assert q.returncode == 0 and q.stdout == p.stdout and "[Prompt" not in q.stderr
