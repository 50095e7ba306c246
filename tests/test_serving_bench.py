"""Client-side serving benchmark against a live HTTP server (tiny CPU
engine behind uvicorn on a free local port): every streamed request
completes with its full output length and the report carries TTFT / TPOT
percentiles and throughput."""
import asyncio
import os
import socket
import sys
import threading
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_serving_benchmark_against_live_server():
    import uvicorn
    from b200ds import EngineConfig, load_engine
    from b200ds.engine.tokenizer import ByteTokenizer
    from b200ds.server.openai import EngineWorker, create_app
    sys.path.insert(0, os.path.join(ROOT, "benchmarks"))
    import serving
    eng = load_engine("tiny", ecfg=EngineConfig(page_size=8, cuda_graphs=False), device="cpu")
    eng.tokenizer = ByteTokenizer()
    worker = EngineWorker(eng, eng.tokenizer).start()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    server = uvicorn.Server(uvicorn.Config(create_app(worker, "tiny"), host="127.0.0.1", port=port,
                                           log_level="warning"))
    t = threading.Thread(target=server.run, daemon=True)
    t.start()
    try:
        deadline = time.time() + 30
        while not server.started and time.time() < deadline:
            time.sleep(0.05)
        out = asyncio.run(serving.run(f"http://127.0.0.1:{port}", num_prompts=6, concurrency=3, input_len=8,
                                      output_len=5, vocab=1024))
        assert out["completed"] == 6 and out["failed"] == 0 and out["output_tokens"] == 30, out
        assert out["output_tok_s"] > 0 and out["ttft_ms"]["p50"] > 0 and out["tpot_ms"]["p50"] > 0
    finally:
        server.should_exit = True
        t.join(10)
        worker.stop()
