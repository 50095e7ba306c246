"""Out-of-bounds write checks on a B200: kernels write into output buffers
that sit between guard regions filled with a known byte; after the launch the
guards must be untouched (a write past either end of an output shows up here
even when the result values look right).  Covers quantisation, the fused
RMSNorm, the MoE combine, both top-k selects and the mHC boundary kernel."""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"
PAD = 4096
CANARY = 0xA5


@pytest.fixture(autouse=True)
def _native():
    from b200ds import ops
    ops.set_impl("native")
    import b200ds._C  # noqa: F401  (loud failure if the extension is missing)


class Guarded:
    """A tensor view with PAD canary bytes on both sides."""

    def __init__(self, shape, dtype):
        n = 1
        for d in shape:
            n *= d
        self.nbytes = n * torch.tensor([], dtype=dtype).element_size()
        self.raw = torch.full((self.nbytes + 2 * PAD,), CANARY, dtype=torch.uint8, device=DEV)
        self.t = self.raw[PAD:PAD + self.nbytes].view(dtype).view(*shape)

    def intact(self) -> bool:
        torch.cuda.synchronize()
        head = self.raw[:PAD]
        tail = self.raw[PAD + self.nbytes:]
        return bool((head == CANARY).all()) and bool((tail == CANARY).all())


def test_quant_and_norm_stay_in_bounds():
    from b200ds import _C
    T, K = 37, 1024
    x = torch.randn(T, K, device=DEV).to(torch.bfloat16)
    q = Guarded((T, K), torch.uint8)
    sf = Guarded(((T + 127) // 128 * 128 * K // 32,), torch.uint8)
    _C.quant(x, q.t, sf.t)
    assert q.intact() and sf.intact()
    res = torch.randn(T, K, device=DEV)
    w = torch.rand(K, device=DEV)
    y = Guarded((T, K), torch.bfloat16)
    q2 = Guarded((T, K), torch.uint8)
    sf2 = Guarded(((T + 127) // 128 * 128 * K // 32,), torch.uint8)
    _C.rmsnorm(x, res, w, 1e-6, y.t, q2.t, sf2.t)
    assert y.intact() and q2.intact() and sf2.intact()


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_moe_combine_stays_in_bounds(out_dtype):
    from b200ds import _C
    T, K, D, R = 45, 8, 7168, 400
    y = torch.randn(R, D, device=DEV).to(torch.bfloat16)
    pair_row = torch.randint(0, R, (T, K), dtype=torch.int32, device=DEV)
    pair_row[::3, 1] = -1
    out = Guarded((T, D), out_dtype)
    _C.moe_combine(y, pair_row, None, out.t)
    assert out.intact()
    want = torch.zeros(T, D, device=DEV)
    for k in range(K):
        r = pair_row[:, k].long()
        want += torch.where((r >= 0).unsqueeze(1), y[r.clamp(min=0)].float(), torch.zeros_like(want))
    assert torch.allclose(out.t.float(), want, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("max_n", [0, 33000])
def test_topk_select_stays_in_bounds(max_n):
    from b200ds import _C
    lens = [1, 2048, 2049, 33000, 9000]
    T, K, cap = len(lens), 2048, 33024
    scores = torch.randn(T, cap, device=DEV)
    pos = torch.tensor([n - 1 for n in lens], dtype=torch.int32, device=DEV)
    out = Guarded((T, K), torch.int32)
    _C.topk_select(scores, pos, out.t, max_n)
    assert out.intact()


def test_hc_boundary_stays_in_bounds():
    from b200ds.ops import HcWeights
    from b200ds.config import small_v4_gpu_config
    from b200ds import _C
    cfg = small_v4_gpu_config()
    T, D = 13, 5120
    X = Guarded((T, 4, D), torch.bfloat16)
    X.t.copy_(torch.randn(T, 4, D, device=DEV).to(torch.bfloat16))
    y = torch.randn(T, D, device=DEV).to(torch.bfloat16)
    p_in = torch.rand(T, 4, device=DEV)
    c_in = torch.rand(T, 16, device=DEV)
    hw = HcWeights(torch.randn(24, 4 * D, device=DEV) * 0.02, torch.ones(3, device=DEV), torch.zeros(24, device=DEV))
    w = torch.rand(D, device=DEV)
    post = Guarded((T, 4), torch.float32)
    comb = Guarded((T, 16), torch.float32)
    q = Guarded((T, D), torch.uint8)
    sf = Guarded(((T + 127) // 128 * 128 * D // 32,), torch.uint8)
    hb = Guarded((T, D), torch.bfloat16)
    _C.hc_boundary(X.t, y, p_in, c_in, hw.fn, hw.scale, hw.base, 0, cfg.hc_sinkhorn_iters, cfg.hc_eps, w, 1e-6,
                   post.t, comb.t, q.t, sf.t, hb.t, None)
    assert all(g.intact() for g in (X, post, comb, q, sf, hb))
