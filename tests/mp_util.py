"""Run a function on N CPU ranks (gloo) and collect per-rank results."""
import os
import socket
import tempfile
import traceback

import torch
import torch.multiprocessing as mp


def free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, fn, args, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        res = fn(rank, world, *args)
        torch.save({"ok": True, "res": res}, os.path.join(outdir, f"r{rank}.pt"))
    except BaseException as e:  # report, never hang the parent
        torch.save({"ok": False, "err": traceback.format_exc()}, os.path.join(outdir, f"r{rank}.pt"))
    finally:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()


def run_ranks(fn, world: int, *args, timeout: float = 300.0):
    port = free_port()
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_worker, args=(r, world, port, fn, args, d)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout)
        for p in procs:
            if p.is_alive():
                p.kill()
                raise TimeoutError("rank did not finish")
        out, errs = [], []
        for r in range(world):
            f = os.path.join(d, f"r{r}.pt")
            if not os.path.exists(f):
                errs.append(f"rank {r} produced no result (exit {procs[r].exitcode})")
                continue
            o = torch.load(f, weights_only=False)
            if not o["ok"]:
                errs.append(f"rank {r} failed:\n{o['err']}")
                continue
            out.append(o["res"])
        if errs:
            raise RuntimeError("\n".join(errs))
        return out
