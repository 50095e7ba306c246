"""Symmetric (peer-mapped) workspaces for the fused NVLink collectives.

`FusedAllReduce` owns one torch symmetric-memory buffer per tensor-parallel
group: arrival counters plus two parities of per-source receive slots
[world][max_tokens][hidden] bf16.  Its `allreduce_add_rmsnorm` pushes the
local partial into every rank's slot (P2P stores over NVLink) and then runs
the reduce + residual + RMSNorm + MXFP8 kernel; steps with more tokens than
`max_tokens` (long prefill chunks) use NCCL instead.

NVLS mode (`nvls` switch, groups of at least `B200_NVLS_MIN_WORLD` ranks whose
GPUs support multicast): a second symmetric buffer is bound to an NVLink
multicast object.  Producers store their partial only into their own input
slot; the reduction kernel sums each rank's share of the rows in the switch
(multimem.ld_reduce), broadcasts it (multimem.st) and runs the same
residual + RMSNorm + quant epilogue.  Per rank, one read and one write of
1/world of the rows cross NVLink instead of world - 1 full copies.

Reference parity: symmetric-memory rendezvous of the EPA / LGP buffers
(epa.py:994-1010, lgp.py:272-291).
"""
from __future__ import annotations


import torch
import torch.distributed as dist


class FusedAllReduce:
    def __init__(self, ps, hidden: int, max_tokens: int = 256, push_ctas: int = 296, group: str = "tp",
                 allow_nvls: bool = True, topk: int = 0):
        import torch.distributed._symmetric_memory as symm_mem
        from .. import _C
        self.ps = ps
        self.hidden = hidden
        self.max_tokens = max_tokens
        self.push_ctas = push_ctas
        is_tp = group != "ep"
        if group == "ep":       # expert-parallel reduce-scatter under DP attention
            self.world, self.rank, group = ps.ep_size, ps.ep_rank, ps.ep_group
        else:
            self.world, self.rank, group = ps.tp_size, ps.tp_rank, ps.tp_group
        dev = ps.device
        name = group.group_name
        if hasattr(symm_mem, "enable_symm_mem_for_group") and not symm_mem.is_symm_mem_enabled_for_group(name):
            symm_mem.enable_symm_mem_for_group(name)
        # expert-parallel workspaces also hold the combine region the experts'
        # FC2 epilogues write into ([2][max_tokens][topk][hidden] bf16)
        self.topk = topk
        nbytes = int(_C.ep_ar_buffer_size(self.world, max_tokens, hidden, topk) if topk > 0
                     else _C.ar_buffer_size(self.world, max_tokens, hidden))
        self.comb_off = int(_C.ep_combine_offset(self.world, max_tokens, hidden)) if topk > 0 else 0
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=dev)
        self.buf.zero_()
        self.hdl = symm_mem.rendezvous(self.buf, name)
        self.bases = [int(p) for p in self.hdl.buffer_ptrs]
        self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ticket = torch.zeros(1, dtype=torch.int32, device=dev)        # reduce-side ticket
        self.push_ticket = torch.zeros(1, dtype=torch.int32, device=dev)   # push-side ticket
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        # NVLS only for the tensor-parallel all-reduce (the expert-parallel
        # reduce-scatter keeps the push protocol)
        self.nvls = (_Nvls.create(ps, name, group, self.world, self.rank, max_tokens, hidden, dev)
                     if self.world > 1 and is_tp and allow_nvls else None)
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)

    def supports(self, T: int) -> bool:
        return 0 < T <= self.max_tokens

    def _push_target(self):
        """(bases, epoch, push ticket, multicast address) the producers of an
        all-reduce write to: the NVLS buffer's own slot, or every rank's
        push slot."""
        n = self.nvls
        if n is not None:
            return n.bases, n.epoch, n.push_ticket, n.mc
        return self.bases, self.epoch, self.push_ticket, 0

    def allreduce_add_rmsnorm(self, a: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                              quantize: bool, keep_bf16: bool = True):
        """residual += all_reduce(a); returns (normalized act, residual)."""
        from .. import _C
        from ..ops.cuda import alloc_qact
        T, H = a.shape
        x = a if (a.dtype == torch.bfloat16 and a.is_contiguous()) else a.to(torch.bfloat16).contiguous()
        y = torch.empty(T, H, dtype=torch.bfloat16, device=a.device) if (keep_bf16 or not quantize) else None
        qa = alloc_qact(T, H, a.device) if quantize else None
        if self._one_kernel(T):
            self._fused(x, None, None, T, residual, w, eps, y, qa)
            return self._done(y, qa, residual)
        bases, epoch, ticket, mc = self._push_target()
        _C.ar_push(x, bases, self.rank, self.max_tokens, epoch, ticket, self.push_ctas, mc=mc)
        return self._reduce(T, H, 1, residual, w, eps, y, qa)

    def _one_kernel(self, rows: int) -> bool:
        """Push, per-CTA arrivals and reduce + norm in one launch: the push
        protocol (switch `ar_one_kernel`) or, on NVLS groups, the variant
        whose rows are summed through the switch by one rank per CTA (switch
        `nvls_one_kernel`; otherwise NVLS keeps push + reduce kernels)."""
        from ..utils import levers
        if self.nvls is not None:
            return levers.on("nvls_one_kernel")
        # measured (benchmarks/collectives.py, one B200 box): one kernel wins
        # while the pushed rows are few (2 ranks x 64 rows: 23.2 vs 25.8 us;
        # 8 ranks x 1 row: 29.9 vs 38.6 us); at 8 ranks x 64 rows the push
        # kernel's 296 CTAs store faster than one CTA per row (48.0 vs 55.7 us)
        import os
        limit = int(os.environ.get("B200_AR_ONE_KERNEL_ROWS", "256"))
        return levers.on("ar_one_kernel") and self.world * rows <= limit

    def _fused(self, x, pair_row, add, T, residual, w, eps, y, qa):
        from .. import _C
        n = self.nvls
        bases, epoch, ticket, mc = (n.bases, n.epoch, n.ticket, n.mc) if n is not None else \
            (self.bases, self.epoch, self.ticket, 0)
        import os
        # push mode: CTAs per row owner that share the NVLink stores (B200_AR_CHUNKS, default 1)
        chunks = 1 if n is not None else max(1, min(8, int(os.environ.get("B200_AR_CHUNKS", "1"))))
        _C.ar_fused_norm(x, pair_row, add, T, bases, self.rank, self.max_tokens, epoch, ticket, residual, w, eps, y,
                         qa.q if qa else None, qa.sf if qa else None, self.err, mc=mc, chunks=chunks)

    @staticmethod
    def _done(y, qa, residual):
        if qa is not None:
            qa.hf = y
            return qa, residual
        return y, residual

    def _outs(self, T, H, dev, quantize, keep_bf16=True):
        from ..ops.cuda import alloc_qact
        y = torch.empty(T, H, dtype=torch.bfloat16, device=dev) if (keep_bf16 or not quantize) else None
        qa = alloc_qact(T, H, dev) if quantize else None
        return y, qa

    def _reduce(self, T, H, push_ctas, residual, w, eps, y, qa, nvls: bool = True):
        from .. import _C
        n = self.nvls if nvls else None
        if n is not None:
            _C.nvls_ar_norm(T, H, n.bases, self.rank, self.max_tokens, n.mc, n.epoch, n.ticket, push_ctas,
                            residual, w, eps, y, qa.q if qa else None, qa.sf if qa else None, self.err)
        else:
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
        bases, epoch, ticket, mc = self._push_target()
        n = _C.gemm_push(wq.data, wq.sf, a.q, a.sf, N, T, K, splits, bases, self.rank, self.max_tokens,
                         epoch, ticket, mc=mc)
        y, qa = self._outs(T, N, a.q.device, quantize)
        return self._reduce(T, N, int(n), residual, ln_w, eps, y, qa)

    def moe_allreduce_add_rmsnorm(self, part, residual, ln_w, eps, quantize):
        """MoE combine (local experts + shared partial) pushed straight into
        every rank's slot, then reduce + residual + norm."""
        from .. import _C
        T = part.pair_row.shape[0]
        H = part.y.shape[1]
        add = part.add.to(torch.bfloat16).contiguous() if part.add is not None else None
        if self._one_kernel(T):
            y, qa = self._outs(T, H, part.y.device, quantize)
            self._fused(part.y, part.pair_row, add, T, residual, ln_w, eps, y, qa)
            return self._done(y, qa, residual)
        bases, epoch, ticket, mc = self._push_target()
        _C.moe_combine_push(part.y, part.pair_row, add, bases, self.rank, self.max_tokens, epoch, ticket,
                            self.push_ctas, mc=mc)
        y, qa = self._outs(T, H, part.y.device, quantize)
        return self._reduce(T, H, 1, residual, ln_w, eps, y, qa)

    def ep_comb_add_rmsnorm(self, part, residual, ln_w, eps, quantize):
        """Expert-parallel combine whose pair rows the experts' FC2 epilogues
        already stored into this rank's combine slots: one kernel sums each
        own token's K rows + its shared-expert row + the residual, RMSNorm,
        quant."""
        from .. import _C
        H = self.hidden
        add = part.add.to(torch.bfloat16).contiguous() if part.add is not None else None
        y, qa = self._outs(part.T_r, H, residual.device, quantize)
        _C.ep_comb_reduce_norm(part.T_r, H, part.ids.shape[1], part.ids, add, self.bases, self.rank, self.max_tokens,
                               self.epoch, self.ticket, residual, ln_w, eps, y, qa.q if qa else None,
                               qa.sf if qa else None, self.err)
        if qa is not None:
            qa.hf = y
            return qa, residual
        return y, residual

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
        return self._reduce(part.T_r, H, 1, residual, ln_w, eps, y, qa, nvls=False)

    def allreduce_hc_post(self, y: torch.Tensor, X: torch.Tensor, post: torch.Tensor, comb: torch.Tensor):
        """DeepSeek-V4 sublayer boundary: y (this rank's partial [T, D]) is
        pushed into every rank's slot, then one kernel sums the partials and
        applies the hyper-connection post to X in place; returns the row sum
        of squares of the new streams."""
        from .. import _C
        T, D = y.shape
        x = y if (y.dtype == torch.bfloat16 and y.is_contiguous()) else y.to(torch.bfloat16).contiguous()
        _C.ar_push(x, self.bases, self.rank, self.max_tokens, self.epoch, self.push_ticket, self.push_ctas)
        ss = torch.empty(T, dtype=torch.float32, device=y.device)
        _C.ar_hc_post(T, D, self.bases, self.rank, self.max_tokens, self.epoch, self.ticket, 1, X, post, comb, ss,
                      self.err)
        return ss

    def check(self) -> None:
        """Raise if a bounded wait inside the kernels timed out."""
        e = int(self.err.item())
        if e:
            raise RuntimeError(f"fused all-reduce: peer wait timed out (code {e})")


class _Nvls:
    """The multicast-bound all-reduce buffer of one group (see the module
    docstring): symmetric allocation, its multicast address, and the device
    epoch / tickets of the NVLS protocol (csrc/comm/allreduce.cu)."""

    @staticmethod
    def create(ps, name, group, world, rank, max_tokens, hidden, dev):
        """An _Nvls when the `nvls` switch is on, the group is large enough
        and every rank got a multicast mapping (agreed with MIN over the CPU
        group, so all ranks take the same path); else None."""
        import os
        from ..utils import levers
        # off at <= 8 ranks unless asked for: measured on 8 B200s at decode
        # sizes the NVLS all-reduce (77 us at 64 rows) loses to the push
        # protocol (48 us) and to NCCL (34 us), and NCCL wins large messages
        want = levers.on("nvls") and world >= int(os.environ.get("B200_NVLS_MIN_WORLD", "16"))
        if not want:
            return None
        obj, ok = None, 0
        try:
            obj = _Nvls(name, world, rank, max_tokens, hidden, dev)
            ok = 1 if obj.mc else 0
        except Exception as e:   # no multicast on this box: the push protocol stays
            levers.announce("nvls-off", f"NVLS all-reduce unavailable ({type(e).__name__}: {e})")
        if not levers.agree_min([ok], getattr(ps, "cpu_group", None))[0]:
            return None
        levers.announce("nvls-on", f"NVLS all-reduce on ({world} ranks)")
        return obj

    def __init__(self, name, world, rank, max_tokens, hidden, dev):
        import torch.distributed._symmetric_memory as symm_mem
        from .. import _C
        if not symm_mem._SymmetricMemory.has_multicast_support(symm_mem.DeviceType.CUDA, torch.device(dev).index):
            raise RuntimeError("the device has no multicast support")
        nbytes = int(_C.nvls_buffer_size(max_tokens, hidden))
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=dev)
        self.buf.zero_()
        self.hdl = symm_mem.rendezvous(self.buf, name)
        if int(getattr(self.hdl, "offset", 0) or 0) != 0:
            raise RuntimeError("symmetric buffer at a nonzero offset of its allocation")
        self.mc = int(self.hdl.multicast_ptr or 0)
        self.bases = [int(p) for p in self.hdl.buffer_ptrs]
        self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ticket = torch.zeros(1, dtype=torch.int32, device=dev)
        self.push_ticket = torch.zeros(1, dtype=torch.int32, device=dev)


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
        # every rank's region (peer pull: each rank's own rows stay there and
        # the owners' expert kernels read them over NVLink)
        self.src_q = [b + off for b in self.bases]
        self.src_sf = [b + off + off_sf for b in self.bases]
        self.src_g = [b + off + off_g for b in self.bases]
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)

    def supports(self, T_step: int) -> bool:
        return 0 < T_step <= self.max_t

    def check(self) -> None:
        e = int(self.err.item())
        if e:
            raise RuntimeError(f"expert-parallel dispatch: peer wait timed out (code {e})")
