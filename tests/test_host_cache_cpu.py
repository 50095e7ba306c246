"""Host-memory tier of the prefix cache: evicted pages move to host memory
with their rows intact, a later match copies them back, a full host tier
drops its LRU host-only leaves, and serving through it gives the same
tokens as serving without a cache."""
import torch

from b200ds.engine.request import SamplingParams
from b200ds.kv.host_cache import HostKVPool
from b200ds.kv.pool import PagePool
from b200ds.kv.radix import RadixCache


def _setup(gpu_pages=6, host_pages=4, ps=4):
    pool = PagePool(gpu_pages, ps)
    kv = [torch.zeros(gpu_pages * ps, 3), torch.zeros(gpu_pages * ps, dtype=torch.int32)]
    host = HostKVPool(kv, host_pages, ps)
    return pool, kv, RadixCache(pool, host)


def _fill(kv, page, ps, v):
    kv[0][page * ps:(page + 1) * ps] = v
    kv[1][page * ps:(page + 1) * ps] = int(v)


def test_offload_restore_keeps_rows():
    pool, kv, radix = _setup()
    toks = list(range(100, 112))                      # 3 pages of 4
    pages = pool.alloc(3)
    for i, p in enumerate(pages):
        _fill(kv, p, 4, 10 + i)
    radix.insert(toks, pages)
    pool.release(pages)
    assert radix.evict(3) == 3 and radix.offloads == 3 and pool.num_free == 5
    for p in pages:                                   # the device pages are reused by someone else
        _fill(kv, p, 4, -1)
    got, nodes = radix.match(toks + [1])
    assert radix.restores == 3 and len(got) == 3
    for i, p in enumerate(got):
        assert torch.all(kv[0][p * 4:(p + 1) * 4] == 10 + i) and torch.all(kv[1][p * 4:(p + 1) * 4] == 10 + i)
    radix.unlock(nodes)


def test_evicts_deepest_first_and_drops_lru_when_host_full():
    pool, kv, radix = _setup(gpu_pages=8, host_pages=2)
    a = list(range(0, 12))
    b = list(range(50, 58))
    pa, pb = pool.alloc(3), pool.alloc(2)
    radix.insert(a, pa)
    radix.insert(b, pb)
    pool.release(pa)
    pool.release(pb)
    nodes_b = radix.match(b)[1]                       # b recently used and locked
    assert radix.evict(3) == 3                        # a's three pages (leaf first); host holds 2
    assert radix.offloads == 3 and radix.host.num_free == 0
    # the host tier overflowed: a's deepest host-only page was dropped to make room
    assert radix.match_len(a) == 2
    radix.unlock(nodes_b)


def test_engine_serves_through_the_host_tier():
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.engine.engine import Engine
    from b200ds.models.reference import init_weights
    cfg = tiny_config()
    sd = init_weights(cfg, 0)
    g = torch.Generator().manual_seed(31)
    A = torch.randint(0, cfg.vocab_size, (40,), generator=g).tolist()
    others = [torch.randint(0, cfg.vocab_size, (40,), generator=g).tolist() for _ in range(3)]

    def engine(**kw):
        ecfg = EngineConfig(page_size=8, cuda_graphs=False, max_kv_pages=12, **kw)
        return Engine(build_model_from(cfg, ecfg, sd, device="cpu"), ecfg)
    eng = engine(enable_prefix_cache=True, host_kv_pages=32)
    ref = engine(enable_prefix_cache=False)
    seq = [A] + others + [A + [3, 4]]
    got = [eng.generate([p], SamplingParams(max_tokens=4))[0].token_ids for p in seq]
    want = [ref.generate([p], SamplingParams(max_tokens=4))[0].token_ids for p in seq]
    assert got == want
    g = eng.gauges()
    assert g["host_offloads"] > 0 and g["host_restores"] > 0 and g["prefix_hit_tokens"] >= 40
