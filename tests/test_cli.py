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


def test_serve_cli_starts_and_answers():
    """`python -m b200ds serve` with the engine flags: the server comes up,
    answers /health and a completion, and stops on SIGTERM."""
    import signal
    import socket
    import time
    import urllib.request
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    env = dict(os.environ, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="")
    p = subprocess.Popen([sys.executable, "-m", "b200ds", "serve", "--model", "tiny", "--port", str(port),
                          "--no-cuda-graphs", "--page-size", "8", "--max-prefill-tokens", "64",
                          "--schedule-policy", "lpm", "--host-kv-pages", "16", "--watchdog-timeout", "60",
                          "--max-num-seqs", "8"], cwd=ROOT, env=env, stdout=subprocess.PIPE,
                         stderr=subprocess.STDOUT)
    try:
        url = f"http://127.0.0.1:{port}"
        deadline = time.time() + 120
        while time.time() < deadline:
            try:
                if urllib.request.urlopen(url + "/health", timeout=2).status == 200:
                    break
            except OSError:
                time.sleep(0.5)
        req = urllib.request.Request(url + "/v1/completions", data=json.dumps(
            {"prompt": [5, 6, 7], "max_tokens": 3, "temperature": 0}).encode(),
            headers={"Content-Type": "application/json"})
        out = json.loads(urllib.request.urlopen(req, timeout=60).read())
        assert len(out["choices"][0]["token_ids"]) == 3
    finally:
        p.send_signal(signal.SIGTERM)
        try:
            p.wait(30)
        except subprocess.TimeoutExpired:
            p.kill()
            p.wait(10)
