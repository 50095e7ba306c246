"""Library comparison arm (b200ds.ops.baseline) on the CPU: the routing
layout around the grouped MXFP8 GEMM and the static-shape decode attention
follow the fp32 references.  The grouped GEMM itself (a PyTorch CUDA op) is
replaced here by a dequantize-and-matmul per group with the same contract."""
from types import SimpleNamespace

import torch

from b200ds.ops import ExpertWeights, baseline, ref
from b200ds.ops.quant import MXFP8Tensor, dequant_mxfp8, quant_mxfp8_ref


def _grouped_ref(aq, asf, w, offs):
    """The grouped GEMM's contract: rows [offs[g-1], offs[g]) times expert g."""
    R, K = aq.shape
    E, N = w.data.shape[0], w.data.shape[1]
    a = dequant_mxfp8(aq, asf)
    out = torch.zeros(R, N)
    lo = 0
    for g in range(E):
        hi = int(offs[g])
        if hi > lo:
            wg = dequant_mxfp8(w.data[g], w.sf[g])
            out[lo:hi] = a[lo:hi] @ wg.t()
        lo = hi
    return out.to(torch.bfloat16)


def test_library_grouped_moe_layout(monkeypatch):
    monkeypatch.setattr(baseline, "_scaled_grouped", _grouped_ref)
    g = torch.Generator().manual_seed(0)
    E, H, I, T, K, first = 4, 256, 128, 37, 3, 4          # this rank owns experts 4..7 of 12
    mk = lambda n, k: MXFP8Tensor(*quant_mxfp8_ref(torch.randn(E * n, k, generator=g) * 0.1))
    w13, w2 = mk(2 * I, H), mk(H, I)
    ex = ExpertWeights(first, E, MXFP8Tensor(w13.data.view(E, 2 * I, H), w13.sf.view(E, -1)),
                       MXFP8Tensor(w2.data.view(E, H, I), w2.sf.view(E, -1)), I)
    x = torch.randn(T, H, generator=g)
    ids = torch.stack([torch.randperm(12, generator=g)[:K] for _ in range(T)]).int()
    w = torch.rand(T, K, generator=g)
    got = baseline.moe_experts_grouped(x, w, ids, ex, torch.float32)
    want = baseline.moe_experts(baseline.quant(x), w, ids, ex, torch.float32)
    # bf16 FC1 / FC2 outputs against the loop's fp32 ones: a few percent; a
    # wrong row or expert mapping is O(1)
    assert ((got - want).norm() / want.norm()).item() < 6e-2
    assert torch.equal(got.abs().sum(-1) == 0, want.abs().sum(-1) == 0)


def test_library_decode_attention_matches_reference():
    g = torch.Generator().manual_seed(1)
    B, H, L, R, ps = 3, 4, 512, 64, 16
    lens = [40, 7, 33]
    pages = 3
    bt = torch.tensor([[2, 5, 1], [3, 0, 0], [4, 6, 7]], dtype=torch.int32)
    cache = (torch.randn(8 * ps, L + R, generator=g) * 0.5).to(torch.float8_e4m3fn)
    q_abs = torch.randn(B, H, L, generator=g) * 0.1
    q_pe = torch.randn(B, H, R, generator=g) * 0.1
    pos = torch.tensor([n - 1 for n in lens], dtype=torch.int32)
    fb = SimpleNamespace(block_table=bt, positions=pos, is_decode=True)
    got = baseline.mla_decode_torch(q_abs, q_pe, cache, 0.5, fb, 0.07, ps).float()
    want = ref.mla_attention(q_abs, q_pe, cache, 0.5, bt, torch.tensor(lens), torch.arange(B, dtype=torch.int32),
                             pos, 0.07, ps)
    assert pages == bt.shape[1]
    assert ((got - want).norm() / want.norm()).item() < 2e-2


def test_library_sampler_matches_reference():
    g = torch.Generator().manual_seed(2)
    T, V = 6, 300
    logits = torch.randn(T, V, generator=g) * 3
    temperature = torch.tensor([0.0, 0.7, 1.0, 1.3, 0.5, 0.9])
    top_p = torch.tensor([1.0, 0.9, 0.5, 1.0, 0.95, 0.8])
    top_k = torch.tensor([0, 0, 20, 5, 0, 50], dtype=torch.int32)
    for trial in range(5):
        uniform = torch.rand(T, generator=g)
        got = baseline.sample_torch(logits, temperature, top_p, top_k, uniform)
        want = ref.sample(logits, temperature, top_p, top_k, uniform)
        assert torch.equal(got, want), (trial, got, want)
