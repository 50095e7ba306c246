"""Property tests (hypothesis) of the format and routing references the
kernels are checked against: scale-layout packing, tiling, MXFP8 / NVFP4
error bounds, Sinkhorn, E5 prune invariants, Engram hash ranges, the context-parallel
row layout and the all-to-all send plan."""
import torch
from hypothesis import given, settings
from hypothesis import strategies as st


@settings(max_examples=25, deadline=None)
@given(st.integers(1, 300), st.sampled_from([128, 256, 640]), st.integers(0, 2 ** 31 - 1))
def test_sf_pack_unpack_inverse(rows, k, seed):
    from b200ds.ops.quant import pack_sf, unpack_sf
    g = torch.Generator().manual_seed(seed)
    sf = torch.randint(0, 255, (rows, k // 32), generator=g, dtype=torch.uint8)
    assert torch.equal(unpack_sf(pack_sf(sf), rows, k), sf)


@settings(max_examples=15, deadline=None)
@given(st.integers(1, 4), st.integers(1, 3), st.integers(0, 2 ** 31 - 1))
def test_tile_rows_inverse(rb, kb, seed):
    from b200ds.ops.quant import tile_rows128, untile_rows128
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(0, 255, (rb * 128, kb * 128), generator=g, dtype=torch.uint8)
    assert torch.equal(untile_rows128(tile_rows128(x)), x)


@settings(max_examples=25, deadline=None)
@given(st.integers(1, 40), st.sampled_from([128, 256, 640]), st.floats(1e-3, 1e3), st.integers(0, 2 ** 31 - 1))
def test_mxfp8_block_error_bound(rows, k, mag, seed):
    """e4m3 keeps 3 mantissa bits: every element is within 1/16 of its value
    plus the block's smallest step (block amax / 448 / 8)."""
    from b200ds.ops.quant import dequant_mxfp8, quant_mxfp8_ref
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, k, generator=g) * mag
    q, sf = quant_mxfp8_ref(x)
    y = dequant_mxfp8(q, sf)
    amax = x.view(rows, k // 32, 32).abs().amax(-1, keepdim=True).expand(-1, -1, 32).reshape(rows, k)
    assert bool(((y - x).abs() <= x.abs() / 16 + amax / 448 / 8 * 2 + 1e-30).all())


@settings(max_examples=20, deadline=None)
@given(st.integers(1, 20), st.sampled_from([64, 256]), st.integers(0, 2 ** 31 - 1))
def test_nvfp4_rows_relative_error(rows, k, seed):
    from b200ds.ops.quant import dequant_nvfp4_rows, quant_nvfp4_rows
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, k, generator=g)
    y = dequant_nvfp4_rows(*quant_nvfp4_rows(x))
    assert ((y - x).norm() / x.norm()).item() < 0.2


@settings(max_examples=25, deadline=None)
@given(st.integers(1, 6), st.floats(0.1, 3.0), st.integers(0, 2 ** 31 - 1))
def test_sinkhorn_columns_exact_rows_close(t, scale, seed):
    from b200ds.ops import ref
    g = torch.Generator().manual_seed(seed)
    m = ref.sinkhorn(torch.randn(t, 4, 4, generator=g) * scale, 20, 1e-6)
    assert torch.allclose(m.sum(-2), torch.ones(t, 4), atol=1e-4)
    assert torch.allclose(m.sum(-1), torch.ones(t, 4), atol=5e-2)
    assert bool((m >= 0).all())


@settings(max_examples=30, deadline=None)
@given(st.integers(1, 12), st.integers(1, 4), st.floats(0.05, 0.9), st.integers(1, 3), st.integers(0, 2 ** 31 - 1))
def test_e5_prune_invariants(T, K, budget, max_count, seed):
    from b200ds.ops import ref
    g = torch.Generator().manual_seed(seed)
    E = 16
    ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).int()
    w = torch.rand(T, K, generator=g)
    w2, ids2 = ref.e5_prune(ids, w, budget, max_count)
    kept = ids2 >= 0
    assert torch.equal(ids2[kept], ids[kept]) and torch.equal(w2[kept], w[kept])
    assert bool((w2[~kept] == 0).all())
    dropped = set(ids[~kept].tolist())
    for e in dropped:                         # a dropped expert is dropped in every row that picked it
        assert not bool((ids2 == e).any())
        assert int((ids == e).sum()) <= max_count


@settings(max_examples=20, deadline=None)
@given(st.integers(1, 30), st.integers(1, 8), st.integers(2, 4), st.integers(0, 2 ** 31 - 1))
def test_engram_hash_head_ranges(T, heads, n, seed):
    from b200ds.ops import ref
    g = torch.Generator().manual_seed(seed)
    rows = heads * 97
    ctx = torch.randint(-1, 5000, (T, n), generator=g)
    out = ref.engram_hash(ctx, heads, rows, n)
    per = rows // heads
    j = torch.arange(heads).unsqueeze(0)
    assert bool(((out >= j * per) & (out < (j + 1) * per)).all())
    assert torch.equal(out, ref.engram_hash(ctx, heads, rows, n))


@settings(max_examples=40, deadline=None)
@given(st.integers(0, 200), st.integers(1, 300), st.integers(1, 8), st.sampled_from([8, 16, 64]),
       st.integers(0, 2 ** 31 - 1))
def test_cp_layout_covers_the_chunk(start, n, world, page, seed):
    """Context-parallel layout: every chunk position is computed by exactly
    one rank, gathered rows land on that position's slot, and each rank's
    batch holds its strided rows (or one dummy row on the scratch page)."""
    import random
    from b200ds.parallel.cp import build_cp_batch, layout
    rnd = random.Random(seed)
    npages = (start + n + page - 1) // page
    pages = rnd.sample(range(1, 4 * npages + 2), npages)
    prompt = [rnd.randrange(1000) for _ in range(start + n)]
    lay = layout(start, n, world, pages, page, prompt)
    assert sum(lay.counts) == n and lay.tmax == max(max(lay.counts), 1)
    gathered = {}
    for q in range(world):
        fb = build_cp_batch(prompt, start, n, world, q, pages, page)
        if lay.counts[q] == 0:
            assert fb.out_slots.tolist() == [0]
            continue
        assert fb.positions.tolist() == list(range(start + q, start + n, world))
        for j, (p, slot) in enumerate(zip(fb.positions.tolist(), fb.out_slots.tolist())):
            gathered[q * lay.tmax + j] = (p, slot, fb.input_ids[j].item())
    for k in range(n):
        p, slot, tok = gathered[int(lay.src_rows[k])]
        assert p == start + k and slot == int(lay.dst_slots[k]) and tok == int(lay.ids[k]) == prompt[p]


@settings(max_examples=40, deadline=None)
@given(st.integers(1, 60), st.integers(1, 8), st.sampled_from([1, 2, 4, 8]), st.integers(1, 4),
       st.integers(0, 2 ** 31 - 1))
def test_a2a_send_plan_properties(T, K, world, e_local, seed):
    """All-to-all send plan: row t goes to rank d exactly when one of its
    experts lives there, once, in destination-then-row order."""
    from b200ds.parallel.ep_a2a import send_plan
    g = torch.Generator().manual_seed(seed)
    E = world * e_local
    ids = torch.randint(-1, E, (T, K), generator=g)
    row, counts = send_plan(ids, e_local, world)
    want = [sorted({t for t in range(T) for e in ids[t].tolist() if e >= 0 and e // e_local == d})
            for d in range(world)]
    assert counts.tolist() == [len(w) for w in want]
    assert row.tolist() == [t for w in want for t in w]
