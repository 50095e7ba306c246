"""`python -m b200ds` commands on the CPU."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args):
    env = dict(os.environ, PYTHONPATH=ROOT)
    return subprocess.run([sys.executable, "-m", "b200ds", *args], capture_output=True, text=True, env=env,
                          cwd=ROOT, timeout=300)


def test_presets_and_switches():
    p = _run("presets")
    assert p.returncode == 0 and "deepseek-v4.1-flash" in p.stdout and "tiny-v4" in p.stdout
    s = _run("switches")
    assert s.returncode == 0 and "B200_MOE_PULL" in s.stdout


def test_generate_tiny_cpu():
    p = _run("generate", "--model", "tiny", "--device", "cpu", "--no-cuda-graphs", "--ids", "5,6,7",
             "--max-tokens", "3")
    assert p.returncode == 0, p.stderr
    out = json.loads(p.stdout.strip().splitlines()[-1])
    assert len(out["token_ids"]) == 3 and out["finish_reason"] == "length"


def test_generate_guided_with_logprobs():
    p = _run("generate", "--model", "tiny", "--device", "cpu", "--no-cuda-graphs", "--prompt", "pick",
             "--max-tokens", "8", "--guided-choice", "red,green", "--logprobs", "0")
    assert p.returncode == 0, p.stderr
    out = json.loads(p.stdout.strip().splitlines()[-1])
    assert out["text"] in ("red", "green") and len(out["logprobs"]) == len(out["token_ids"])
