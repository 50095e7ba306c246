"""Tensor/expert parallel forward on 2 GPUs (NCCL) against a 1-GPU run of the
same model: logits must agree to bf16/fp8 tolerance."""
import os

import pytest
import torch

from mp_util import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _needs(n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def _batch(cfg, dev, T=12):
    from b200ds.models.batch import build_batch
    g = torch.Generator().manual_seed(3)
    toks = torch.randint(0, cfg.vocab_size, (T,), generator=g).tolist()
    seqs = [{"tokens": toks[:5], "start": 0, "pages": [1]}, {"tokens": toks[5:], "start": 0, "pages": [2]}]
    return build_batch(seqs, 64, device=dev)


def _rank(rank, world, comm_impl, kind):
    import torch
    from b200ds import ops
    from b200ds.config import EngineConfig, small_gpu_config
    from b200ds.models.loader import build_model
    from b200ds.models.reference import init_weights
    from b200ds.parallel.state import ParallelState, init_parallel
    nvls = comm_impl == "nvls"
    if nvls:      # the NVLS all-reduce (multicast) already at 2 ranks
        os.environ["B200_NVLS_MIN_WORLD"] = "2"
        comm_impl = "fused"
    if comm_impl == "fused4":     # one-kernel all-reduce, 4 CTAs per row owner sharing the stores
        os.environ["B200_AR_CHUNKS"] = "4"
        comm_impl = "fused"
    ps = init_parallel(backend="nccl", timeout_s=60)
    ops.set_impl("native")
    # 32 heads: 16 per rank keeps both runs on the same tcgen05 MLA kernel
    cfg = small_gpu_config(num_attention_heads=32)
    if kind == "dense":
        # one dense layer: a single fp8 quantization stage between the runs,
        # while any sharding error would still show as an O(1) difference
        cfg = small_gpu_config(num_attention_heads=32, n_routed_experts=0, first_k_dense_replace=1,
                               num_hidden_layers=1)
    sd = init_weights(cfg, 0)
    ecfg = EngineConfig(tp_size=world, ep_size=world, comm_impl=comm_impl)
    m = build_model(cfg, ecfg, ps, sd, device=ps.device)
    m.allocate_kv(8)
    fb = _batch(cfg, ps.device)
    try:
        out = m.forward(fb).float().cpu()
        # device sampling without gathering the logits (candidates exchanged over
        # the fused slots or NCCL): greedy rows must pick this run's argmax
        z = torch.zeros(2, device=ps.device)
        toks = m.forward_tokens(_batch(cfg, ps.device), z, z + 1, z.int(), z).cpu()
    finally:
        # both ranks finish their device work before either can leave (a rank
        # must not exit while peers may still read its multicast-bound memory)
        torch.cuda.synchronize()
        import torch.distributed as dist
        dist.barrier(group=ps.cpu_group)
    if nvls:
        assert ps.fused_ar is not None and ps.fused_ar.nvls is not None, "NVLS buffer not set up"
    assert toks.tolist() == out.argmax(-1).tolist(), (toks, out.argmax(-1))
    ref = None
    if rank == 0:
        single = ParallelState(device=ps.device)
        m1 = build_model(cfg, EngineConfig(), single, sd, device=ps.device)
        m1.allocate_kv(8)
        ref = m1.forward(fb).float().cpu()
    torch.cuda.synchronize()
    if ps.fused_ar is not None:
        ps.fused_ar.check()
    return out, ref


def _oracle_logits(kind):
    """fp32 CPU oracle logits at the last token of each test sequence."""
    from b200ds.config import small_gpu_config
    from b200ds.models.reference import ReferenceModel, init_weights
    cfg = small_gpu_config(num_attention_heads=32)
    if kind == "dense":
        cfg = small_gpu_config(num_attention_heads=32, n_routed_experts=0, first_k_dense_replace=1,
                               num_hidden_layers=1)
    m = ReferenceModel(cfg, init_weights(cfg, 0), max_len=64)
    g = torch.Generator().manual_seed(3)
    toks = torch.randint(0, cfg.vocab_size, (12,), generator=g)
    outs = []
    for seq in (toks[:5], toks[5:]):
        m.reset(1)
        outs.append(m.forward(seq.view(1, -1), 0)[0, -1])
    return torch.stack(outs)


def _rel(a, b):
    return ((a - b).norm() / b.norm()).item()


def _has_multicast():
    try:
        import torch.distributed._symmetric_memory as sm
        return bool(sm._SymmetricMemory.has_multicast_support(sm.DeviceType.CUDA, 0))
    except Exception:
        return False


@pytest.mark.parametrize("comm_impl", ["nccl", "fused", "fused4", "nvls"])
@pytest.mark.parametrize("kind,tol", [("dense", 2e-2), ("moe", 1e-1)])
def test_tp2_ep2_matches_single_gpu(comm_impl, kind, tol):
    """TP2/EP2 vs one GPU.  The runs differ only in how partial sums are
    rounded (bf16 partials, then summed), but every later MXFP8 quantization
    can turn such a difference into a flipped e4m3 code or UE8M0 block scale,
    so the error compounds with depth: the 1-layer dense model is held
    tightly, the 4-layer MoE model loosely.  Both ranks must agree exactly.
    "nvls": the all-reduces run through NVLink multicast (multimem) on 2 ranks."""
    _needs(2)
    if comm_impl == "nvls" and not _has_multicast():
        pytest.skip("no NVLink multicast on this box")
    res = run_ranks(_rank, 2, comm_impl, kind, timeout=600)
    out0, ref = res[0]
    out1, _ = res[1]
    assert torch.equal(out0, out1)
    oracle = _oracle_logits(kind)
    e_tp2, e_tp1 = _rel(out0, oracle), _rel(ref, oracle)
    # TP2 is as accurate as one GPU against the fp32 oracle ...
    assert e_tp2 <= 1.3 * e_tp1 + 0.01, (e_tp2, e_tp1)
    # ... and the two GPU runs differ by fp8 requantization noise only
    assert _rel(out0, ref) < 2.5 * tol, _rel(out0, ref)


def _dp_batch(rank, cfg, dev):
    from b200ds.models.batch import build_batch
    g = torch.Generator().manual_seed(11 + rank)
    if rank == 0:
        toks = torch.randint(0, cfg.vocab_size, (12,), generator=g).tolist()
        seqs = [{"tokens": toks[:5], "start": 0, "pages": [1]}, {"tokens": toks[5:], "start": 0, "pages": [2]}]
    else:
        toks = torch.randint(0, cfg.vocab_size, (9,), generator=g).tolist()
        seqs = [{"tokens": toks, "start": 0, "pages": [3]}]
    return build_batch(seqs, 64, device=dev)


def _dp_rank(rank, world, comm_impl, fmt="mxfp8"):
    import torch
    from b200ds import ops
    from b200ds.config import EngineConfig, small_gpu_config
    from b200ds.models.loader import build_model
    from b200ds.models.reference import init_weights
    from b200ds.parallel.state import ParallelState, init_parallel
    from b200ds.utils import levers
    if comm_impl == "peer":       # the expert kernels read the routed rows from their source ranks over NVLink
        levers.set_switch("ep_peer_pull", True)
        comm_impl = "fused"
    if comm_impl == "a2a":        # NCCL all-to-all exchange: rows only to their experts' owners
        os.environ["B200_DP_A2A_MIN_ROWS"] = "1"
        comm_impl = "nccl"
    ps = init_parallel(backend="nccl", dp_attention=True, timeout_s=60)
    ops.set_impl("native")
    cfg = small_gpu_config(num_attention_heads=16, expert_format=fmt)
    sd = init_weights(cfg, 0)
    ecfg = EngineConfig(tp_size=1, ep_size=world, dp_attention=True, comm_impl=comm_impl)
    m = build_model(cfg, ecfg, ps, sd, device=ps.device)
    m.allocate_kv(8)
    fb = _dp_batch(rank, cfg, ps.device)
    fb.dp_tmax = 12                      # the larger rank's token rows
    out = m.forward(fb).float().cpu()
    single = build_model(cfg, EngineConfig(), ParallelState(device=ps.device), sd, device=ps.device)
    single.allocate_kv(8)
    ref = single.forward(_dp_batch(rank, cfg, ps.device)).float().cpu()
    torch.cuda.synchronize()
    for obj in (ps.fused_ar, ps.fused_ep):
        if obj is not None:
            obj.check()
    return rank, out, ref


@pytest.mark.parametrize("comm_impl,fmt", [("nccl", "mxfp8"), ("fused", "mxfp8"), ("fused", "nvfp4"),
                                           ("peer", "mxfp8"), ("peer", "nvfp4"), ("a2a", "mxfp8")])
def test_dp2_ep2_matches_single_gpu(comm_impl, fmt):
    """DP attention + EP MoE on 2 GPUs, ranks with different token counts:
    each rank's logits follow a 1-GPU run of its own batch (fp8 noise only).
    The fused path exercises ep_dispatch / ep_align, the expert kernel
    reading the received rows in place from the dispatch buffer (alternating
    parities over the layers) and the combine stored by the FC2 epilogue into
    the owners' slots; "peer" leaves the rows on their source ranks and the
    expert kernel reads them over NVLink."""
    _needs(2)
    res = run_ranks(_dp_rank, 2, comm_impl, fmt, timeout=600)
    for rank, out, ref in res:
        assert _rel(out, ref) < 0.15, (rank, _rel(out, ref))


def _v4_rank(rank, world):
    import torch
    import torch.distributed as dist
    from b200ds import ops
    from b200ds.config import EngineConfig, small_v4_gpu_config
    from b200ds import build_model_from
    from b200ds.models.batch import build_batch
    from b200ds.models.reference_v4 import init_weights_v4
    from b200ds.parallel.state import init_parallel
    ps = init_parallel(backend="nccl", timeout_s=60)
    ops.set_impl("native")
    cfg = small_v4_gpu_config()
    sd = init_weights_v4(cfg, 0)
    m = build_model_from(cfg, EngineConfig(tp_size=world, ep_size=world, comm_impl="fused"), sd, device=ps.device,
                         ps=ps)
    m.allocate_kv(8)
    g = torch.Generator().manual_seed(5)
    toks = torch.randint(0, cfg.vocab_size, (40,), generator=g).tolist()
    seqs = [{"tokens": toks[:17], "start": 0, "pages": [1]}, {"tokens": toks[17:], "start": 0, "pages": [2]}]
    try:
        out = m.forward(build_batch(seqs, 64, device=ps.device)).float().cpu()
    finally:
        torch.cuda.synchronize()
        dist.barrier(group=ps.cpu_group)
    assert ps.fused_ar is not None and ps.fused_ar.nvls is None
    ps.fused_ar.check()
    return out


def test_v4_tp2_fused_boundary_matches_oracle():
    """DeepSeek-V4-family model at TP2: every sublayer's all-reduce runs fused
    with the hyper-connection post (ar_push / GEMM push + ar_hc_post); both
    ranks agree exactly and follow the fp32 oracle like one GPU does."""
    _needs(2)
    from b200ds.config import small_v4_gpu_config
    from b200ds.models.reference_v4 import ReferenceV4Model, init_weights_v4
    res = run_ranks(_v4_rank, 2, timeout=600)
    assert torch.equal(res[0], res[1])
    cfg = small_v4_gpu_config()
    oracle = ReferenceV4Model(cfg, init_weights_v4(cfg, 0), 128)
    g = torch.Generator().manual_seed(5)
    toks = torch.randint(0, cfg.vocab_size, (40,), generator=g)
    want = []
    for seq in (toks[:17], toks[17:]):
        oracle.reset(1)
        want.append(oracle.forward(seq.view(1, -1), 0, decode=False)[0, -1])
    want = torch.stack(want)
    assert _rel(res[0], want) < 0.15, _rel(res[0], want)


def _cp_rank(rank, world):
    import torch
    import torch.distributed as dist
    from b200ds import ops
    from b200ds.config import EngineConfig, small_gpu_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.loader import build_model
    from b200ds.models.reference import init_weights
    from b200ds.parallel.state import ParallelState, init_parallel
    ps = init_parallel(backend="nccl", dp_attention=True, timeout_s=60)
    ops.set_impl("native")
    cfg = small_gpu_config(num_attention_heads=16)
    sd = init_weights(cfg, 0)
    g = torch.Generator().manual_seed(21)
    prompt = torch.randint(0, cfg.vocab_size, (300,), generator=g).tolist()

    def first_logits(eng, **kw):
        seen = []
        orig = eng._sample
        eng._sample = lambda st, lg: seen.append(lg.float().cpu()) or orig(st, lg)
        r = eng.add_request(prompt, SamplingParams(max_tokens=2), **kw)
        while not r.finished:
            eng.step()
        return r, (seen[0] if seen else None)

    # chunks of 256 rows (128 a rank: the fused expert-parallel exchange) and 44
    ecfg = EngineConfig(tp_size=1, ep_size=world, dp_attention=True, context_parallel=True, cuda_graphs=False,
                        max_prefill_tokens=128, enable_prefix_cache=False)
    eng = Engine(build_model(cfg, ecfg, ps, sd, device=ps.device), ecfg, num_pages=16)
    try:
        r, got = first_logits(eng, cp_owner=1)
        eng._drain_dp()
    finally:
        torch.cuda.synchronize()
        dist.barrier(group=ps.cpu_group)
    for obj in (ps.fused_ar, ps.fused_ep):
        if obj is not None:
            obj.check()
    if rank != 1:
        return rank, r.finish_reason, None, None
    one = EngineConfig(cuda_graphs=False, enable_prefix_cache=False)
    single = Engine(build_model(cfg, one, ParallelState(device=ps.device), sd, device=ps.device), one, num_pages=16)
    _, want = first_logits(single)
    return rank, r.finish_reason, got, want


def test_cp2_prefill_matches_single_gpu():
    """Context-parallel prefill of a 300-token prompt on 2 GPUs (rows split
    round-robin, each layer's new fp8 cache rows all-gathered over NCCL,
    MoE through the fused expert-parallel exchange): the owner's first-token
    logits follow a 1-GPU prefill of the same prompt (fp8 noise only)."""
    _needs(2)
    res = run_ranks(_cp_rank, 2, timeout=600)
    for rank, reason, got, want in res:
        if rank == 1:
            assert reason == "length"
            assert _rel(got, want) < 0.15, _rel(got, want)
        else:
            assert reason == "context_parallel_peer"


def _tbo_rank(rank, world):
    import torch
    import torch.distributed as dist
    from b200ds import ops
    from b200ds.config import EngineConfig, small_gpu_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.loader import build_model
    from b200ds.models.reference import init_weights
    from b200ds.parallel.state import ParallelState, init_parallel
    ps = init_parallel(backend="nccl", dp_attention=True, timeout_s=60)
    ops.set_impl("native")
    cfg = small_gpu_config(num_attention_heads=16)
    sd = init_weights(cfg, 0)
    g = torch.Generator().manual_seed(31 + rank)
    prompt = torch.randint(0, cfg.vocab_size, (40 if rank == 0 else 25,), generator=g).tolist()

    def first_logits(eng):
        seen = []
        orig = eng._sample
        eng._sample = lambda st, lg: seen.append(lg.float().cpu()) or orig(st, lg)
        r = eng.add_request(prompt, SamplingParams(max_tokens=2))
        while not r.finished:
            eng.step()
        return seen[0]

    # NCCL exchange (the host-collective path the overlap interleaves)
    ecfg = EngineConfig(tp_size=1, ep_size=world, dp_attention=True, comm_impl="nccl", cuda_graphs=False,
                        tbo=True, tbo_min_tokens=2, enable_prefix_cache=False)
    eng = Engine(build_model(cfg, ecfg, ps, sd, device=ps.device), ecfg, num_pages=8)
    try:
        got = first_logits(eng)
        eng._drain_dp()
    finally:
        torch.cuda.synchronize()
        dist.barrier(group=ps.cpu_group)
    one = EngineConfig(cuda_graphs=False, enable_prefix_cache=False)
    single = Engine(build_model(cfg, one, ParallelState(device=ps.device), sd, device=ps.device), one, num_pages=8)
    return rank, eng.stats.get("tbo_steps", 0), got, first_logits(single)


def test_dp2_two_batch_overlap_gpu():
    """Two-batch overlap on 2 GPUs: each rank's prefill rows run as two
    micro-batches whose NCCL all-gather / reduce-scatter overlap the other
    micro-batch's kernels; first-token logits follow a 1-GPU run."""
    _needs(2)
    res = run_ranks(_tbo_rank, 2, timeout=600)
    for rank, steps, got, want in res:
        assert steps >= 1
        assert _rel(got, want) < 0.15, (rank, _rel(got, want))


def _cp_v4_rank(rank, world):
    import torch
    import torch.distributed as dist
    from b200ds import build_model_from, ops
    from b200ds.config import EngineConfig, small_v4_gpu_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference_v4 import init_weights_v4
    from b200ds.parallel.state import ParallelState, init_parallel
    ps = init_parallel(backend="nccl", dp_attention=True, timeout_s=60)
    ops.set_impl("native")
    cfg = small_v4_gpu_config()
    sd = init_weights_v4(cfg, 0)
    g = torch.Generator().manual_seed(23)
    prompt = torch.randint(0, cfg.vocab_size, (200,), generator=g).tolist()

    def first_logits(eng, **kw):
        seen = []
        orig = eng._sample
        eng._sample = lambda st, lg: seen.append(lg.float().cpu()) or orig(st, lg)
        r = eng.add_request(prompt, SamplingParams(max_tokens=2), **kw)
        while not r.finished:
            eng.step()
        return r, (seen[0] if seen else None)

    ecfg = EngineConfig(tp_size=1, ep_size=world, dp_attention=True, context_parallel=True, cuda_graphs=False,
                        max_prefill_tokens=64, enable_prefix_cache=False)
    eng = Engine(build_model_from(cfg, ecfg, sd, device=ps.device, ps=ps), ecfg, num_pages=8)
    try:
        r, got = first_logits(eng, cp_owner=0)
        eng._drain_dp()
    finally:
        torch.cuda.synchronize()
        dist.barrier(group=ps.cpu_group)
    if rank != 0:
        return rank, r.finish_reason, None, None
    one = EngineConfig(cuda_graphs=False, enable_prefix_cache=False)
    single = Engine(build_model_from(cfg, one, sd, device=ps.device, ps=ParallelState(device=ps.device)), one,
                    num_pages=8)
    _, want = first_logits(single)
    return rank, r.finish_reason, got, want


def test_cp2_v4_prefill_matches_single_gpu():
    """Context-parallel prefill of the V4 family on 2 GPUs (n-gram hashes over
    the whole chunk's token cache, mHC per row, chunks of 128 rows): the
    owner's first-token logits follow a 1-GPU prefill (fp8 noise only)."""
    _needs(2)
    res = run_ranks(_cp_v4_rank, 2, timeout=600)
    for rank, reason, got, want in res:
        if rank == 0:
            assert reason == "length"
            assert _rel(got, want) < 0.15, _rel(got, want)
        else:
            assert reason == "context_parallel_peer"
