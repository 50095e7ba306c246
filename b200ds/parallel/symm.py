"""Symmetric (peer-mapped) workspaces for the fused NVLink collectives.

`FusedAllReduce` owns one torch symmetric-memory buffer per tensor-parallel
group: arrival counters plus two parities of per-source receive slots
[world][max_tokens][hidden] bf16.  Its `allreduce_add_rmsnorm` pushes the
local partial into every rank's slot (P2P stores over NVLink) and then runs
the reduce + residual + RMSNorm + MXFP8 kernel; steps with more tokens than
`max_tokens` (long prefill chunks) use NCCL instead.

Reference parity: symmetric-memory rendezvous of the EPA / LGP buffers
(epa.py:994-1010, lgp.py:272-291).
"""
from __future__ import annotations


import torch
import torch.distributed as dist


class FusedAllReduce:
    def __init__(self, ps, hidden: int, max_tokens: int = 256, push_ctas: int = 296, group: str = "tp"):
        import torch.distributed._symmetric_memory as symm_mem
        from .. import _C
        self.ps = ps
        self.hidden = hidden
        self.max_tokens = max_tokens
        self.push_ctas = push_ctas
        if group == "ep":       # expert-parallel reduce-scatter under DP attention
            self.world, self.rank, group = ps.ep_size, ps.ep_rank, ps.ep_group
        else:
            self.world, self.rank, group = ps.tp_size, ps.tp_rank, ps.tp_group
        dev = ps.device
        name = group.group_name
        if hasattr(symm_mem, "enable_symm_mem_for_group") and not symm_mem.is_symm_mem_enabled_for_group(name):
            symm_mem.enable_symm_mem_for_group(name)
        nbytes = int(_C.ar_buffer_size(self.world, max_tokens, hidden))
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=dev)
        self.buf.zero_()
        self.hdl = symm_mem.rendezvous(self.buf, name)
        self.bases = [int(p) for p in self.hdl.buffer_ptrs]
        self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ticket = torch.zeros(1, dtype=torch.int32, device=dev)        # reduce-side ticket
        self.push_ticket = torch.zeros(1, dtype=torch.int32, device=dev)   # push-side ticket
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)

    def supports(self, T: int) -> bool:
        return 0 < T <= self.max_tokens

    def allreduce_add_rmsnorm(self, a: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                              quantize: bool, keep_bf16: bool = True):
        """residual += all_reduce(a); returns (normalized act, residual)."""
        from .. import _C
        from ..ops.cuda import alloc_qact
        T, H = a.shape
        x = a if (a.dtype == torch.bfloat16 and a.is_contiguous()) else a.to(torch.bfloat16).contiguous()
        _C.ar_push(x, self.bases, self.rank, self.max_tokens, self.epoch, self.push_ticket, self.push_ctas)
        y = torch.empty(T, H, dtype=torch.bfloat16, device=a.device) if (keep_bf16 or not quantize) else None
        qa = alloc_qact(T, H, a.device) if quantize else None
        _C.ar_reduce_norm(T, H, self.bases, self.rank, self.max_tokens, self.epoch, self.ticket, 1,
                          residual, w, eps, y, qa.q if qa else None, qa.sf if qa else None, self.err)
        if qa is not None:
            qa.hf = y
            return qa, residual
        return y, residual

    def _outs(self, T, H, dev, quantize, keep_bf16=True):
        from ..ops.cuda import alloc_qact
        y = torch.empty(T, H, dtype=torch.bfloat16, device=dev) if (keep_bf16 or not quantize) else None
        qa = alloc_qact(T, H, dev) if quantize else None
        return y, qa

    def _reduce(self, T, H, push_ctas, residual, w, eps, y, qa):
        from .. import _C
        _C.ar_reduce_norm(T, H, self.bases, self.rank, self.max_tokens, self.epoch, self.ticket, push_ctas,
                          residual, w, eps, y, qa.q if qa else None, qa.sf if qa else None, self.err)
        if qa is not None:
            qa.hf = y
            return qa, residual
        return y, residual

    def gemm_allreduce_add_rmsnorm(self, x, wq, residual, ln_w, eps, quantize):
        """o_proj / down_proj GEMM whose split-K cluster epilogue pushes the
        output tiles into every rank's slot, then reduce + residual + norm."""
        from .. import _C
        from ..ops import QAct
        from ..ops.cuda import choose_splits, quant
        a = x if isinstance(x, QAct) else quant(x)
        T, K = a.q.shape
        N = wq.data.shape[0]
        splits = choose_splits(T, N, K, max_ctas=148 + 74)
        if splits < 2 or T > 128:
            from ..ops.cuda import gemm
            return self.allreduce_add_rmsnorm(gemm(a, wq), residual, ln_w, eps, quantize)
        n = _C.gemm_push(wq.data, wq.sf, a.q, a.sf, N, T, K, splits, self.bases, self.rank, self.max_tokens,
                         self.epoch, self.push_ticket)
        y, qa = self._outs(T, N, a.q.device, quantize)
        return self._reduce(T, N, int(n), residual, ln_w, eps, y, qa)

    def moe_allreduce_add_rmsnorm(self, part, residual, ln_w, eps, quantize):
        """MoE combine (local experts + shared partial) pushed straight into
        every rank's slot, then reduce + residual + norm."""
        from .. import _C
        T = part.pair_row.shape[0]
        H = part.y.shape[1]
        add = part.add.to(torch.bfloat16).contiguous() if part.add is not None else None
        _C.moe_combine_push(part.y, part.pair_row, add, self.bases, self.rank, self.max_tokens, self.epoch,
                            self.push_ticket, self.push_ctas)
        y, qa = self._outs(T, H, part.y.device, quantize)
        return self._reduce(T, H, 1, residual, ln_w, eps, y, qa)

    def ep_rs_add_rmsnorm(self, part, residual, ln_w, eps, quantize):
        """Expert-parallel combine: each received token's partial goes to its
        owner's slot (reduce-scatter), then this rank's reduce + residual +
        norm over its own T_r tokens."""
        from .. import _C
        H = part.y.shape[1]
        add = part.add.to(torch.bfloat16).contiguous() if part.add is not None else None
        _C.ep_combine_rs(part.y, part.pair_row, part.T_step, part.T_r, add, self.bases, self.rank, self.max_tokens,
                         self.epoch, self.push_ticket, self.push_ctas)
        y, qa = self._outs(part.T_r, H, part.y.device, quantize)
        return self._reduce(part.T_r, H, 1, residual, ln_w, eps, y, qa)

    def check(self) -> None:
        """Raise if a bounded wait inside the kernels timed out."""
        e = int(self.err.item())
        if e:
            raise RuntimeError(f"fused all-reduce: peer wait timed out (code {e})")


class EPDispatch:
    """Symmetric dispatch buffer of the expert-parallel MoE (DP attention):
    two parities of [world * max_tokens] received MXFP8 token rows plus their
    routing rows, arrival counters, and the device epoch / tickets of the
    dispatch -> align -> gather protocol (csrc/comm/ep.cu)."""

    def __init__(self, ps, hidden: int, topk: int, max_tokens: int):
        import torch.distributed._symmetric_memory as symm_mem
        from .. import _C
        self.world = ps.ep_size
        self.rank = ps.ep_rank
        self.max_t = max_tokens
        self.hidden = hidden
        dev = ps.device
        group = ps.ep_group
        name = group.group_name
        if hasattr(symm_mem, "enable_symm_mem_for_group") and not symm_mem.is_symm_mem_enabled_for_group(name):
            symm_mem.enable_symm_mem_for_group(name)
        nbytes = int(_C.ep_buffer_size(self.world, max_tokens, hidden, topk))
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=dev)
        self.buf.zero_()
        self.hdl = symm_mem.rendezvous(self.buf, name)
        self.bases = [int(p) for p in self.hdl.buffer_ptrs]
        self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
        self.push_ticket = torch.zeros(1, dtype=torch.int32, device=dev)
        self.gather_ticket = torch.zeros(1, dtype=torch.int32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        # this rank's received rows, read in place by the fused expert kernel:
        # (q, scales, global scales) addresses of parity 0 and the parity stride
        off, self.par_bytes, off_sf, off_g = (int(v) for v in _C.ep_region_layout(self.world, max_tokens, hidden, topk))
        mine = self.bases[self.rank] + off
        self.recv_q, self.recv_sf, self.recv_g = mine, mine + off_sf, mine + off_g
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)

    def supports(self, T_step: int) -> bool:
        return 0 < T_step <= self.max_t

    def check(self) -> None:
        e = int(self.err.item())
        if e:
            raise RuntimeError(f"expert-parallel dispatch: peer wait timed out (code {e})")
