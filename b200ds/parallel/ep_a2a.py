"""Expert-parallel all-to-all exchange for large DP-attention steps.

Under DP attention each rank routes its own rows; the routed experts are
split over the ranks (rank r owns experts [r * E_local, (r + 1) * E_local)).
For steps too large for the symmetric dispatch buffers (long prefill chunks)
the rows travel with host-launched collectives.  Here each row goes only to
the ranks that own at least one of its experts (once per such rank, with its
full expert list and weights: the receiver's routing layout skips experts it
does not own), every rank runs its experts over the rows it received, and the
per-rank partial sums come back the same way and are added into the source
rows.  Against an all-gather of every row to every rank plus a reduce-scatter
of W x T partial rows, a row crosses NVLink only towards its experts' owners
(about 5.3 of 8 ranks for top-8 of 256 experts over 8 ranks), and the
experts never see rows of other ranks' experts.

The exchange is a generator that yields right after issuing each bulk
collective (asynchronous while two micro-batches interleave), like the other
DP exchanges.  The per-destination row counts go first, in place: the sizes
of the bulk transfers are read on the host, so the path never runs inside a
CUDA graph capture.

Reference parity: the stock expert-parallel dispatcher the reference routes
through (`get_moe_a2a_backend`, the dispatcher's combine hooks,
moe_fwd.py:355-382).
"""
from __future__ import annotations

import os
from typing import Callable

import torch
import torch.distributed as dist


def a2a_ok(x: torch.Tensor, rows_per_rank: int) -> bool:
    """Whether a DP step of `rows_per_rank` agreed rows takes the
    all-to-all exchange (switch dp_moe_a2a): large steps only, and never
    while a CUDA graph is being captured (the transfer sizes are read on the
    host).  Every rank decides the same way (agreed rows, same switches)."""
    from ..utils import levers
    if not levers.on("dp_moe_a2a"):
        return False
    if rows_per_rank < int(os.environ.get("B200_DP_A2A_MIN_ROWS", "64")):
        return False
    return not (x.is_cuda and torch.cuda.is_current_stream_capturing())


def send_plan(ids: torch.Tensor, e_local: int, world: int):
    """Rows to send, grouped by destination rank: (destination-sorted row
    indices, rows per destination [W]).  A row goes to every rank that owns
    one of its experts (ids < 0 = no expert)."""
    T, K = ids.shape
    dev = ids.device
    owner = torch.div(ids.long(), e_local, rounding_mode="floor")
    valid = ids >= 0
    hit = torch.zeros(world, T, dtype=torch.bool, device=dev)
    rows = torch.arange(T, device=dev).unsqueeze(1).expand(T, K)
    hit[owner[valid], rows[valid]] = True
    dst, row = hit.nonzero(as_tuple=True)          # sorted by destination, then row
    return row, hit.sum(1)


def a2a_moe_steps(x: torch.Tensor, w: torch.Tensor, ids: torch.Tensor, ps, e_local: int,
                  run_experts: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor],
                  overlap: bool = False):
    """Generator: this rank's rows x [T, H] with routing weights w [T, K]
    and global expert ids [T, K] through every rank's experts; returns the
    fp32 sum [T, H] over the routed experts.  run_experts(rows, weights,
    ids) returns this rank's experts' partial sums [n, H] (fp32) of the rows
    it received."""
    W, grp = ps.ep_size, ps.ep_group
    T, H = x.shape
    row, send = send_plan(ids, e_local, W)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=grp)
    sc, rc = send.tolist(), recv.tolist()
    nr = sum(rc)
    xs, ws, is_ = x[row].contiguous(), w[row].float().contiguous(), ids[row].to(torch.int32).contiguous()
    xr = x.new_empty(nr, H)
    wr = ws.new_empty(nr, ws.shape[1])
    ir = is_.new_empty(nr, is_.shape[1])
    works = [dist.all_to_all_single(dst, src, rc, sc, group=grp, async_op=overlap)
             for dst, src in ((xr, xs), (wr, ws), (ir, is_))]
    yield
    if overlap:
        for wk in works:
            wk.wait()
    part = run_experts(xr, wr, ir) if nr else torch.zeros(0, H, dtype=torch.float32, device=x.device)
    back = part.new_empty(int(row.shape[0]), H)
    work = dist.all_to_all_single(back, part.contiguous(), sc, rc, group=grp, async_op=overlap)
    yield
    if overlap:
        work.wait()
    return torch.zeros(T, H, dtype=torch.float32, device=x.device).index_add_(0, row, back)
