"""Kernel tactics as data: table matching (exact ints, inclusive bands,
first match wins), legality checks, and the CUDA op layer's heuristics
taking the table's value only where it names the shape."""
import json

import pytest


def test_table_matching_and_legality(tmp_path):
    from b200ds.ops import tactics
    p = tmp_path / "t.json"
    p.write_text(json.dumps({
        "gemm_splits": [{"N": 7168, "K": 16384, "rows": [1, 32], "value": 2},
                        {"N": 7168, "K": 16384, "rows": [1, 64], "value": 8},
                        {"N": 2176, "value": 16}],
        "moe_tile": [{"cap": 64, "rows_per_expert": [0, 4], "value": 128}],
        "mla_splits": [{"H": 16, "rows": 64, "value": 3}]}))
    try:
        tactics.load(str(p))
        ctx = dict(N=7168, K=16384, max_ctas=296)
        assert tactics.pick("gemm_splits", 4, rows=16, **ctx) == 2        # first match
        assert tactics.pick("gemm_splits", 4, rows=64, **ctx) == 4        # 8 splits: 448 CTAs > cap -> default
        assert tactics.pick("gemm_splits", 4, rows=65, **ctx) == 4        # no entry
        assert tactics.pick("gemm_splits", 1, N=2176, K=7168, rows=8, max_ctas=296) == 1   # 16: not a factor
        assert tactics.pick("moe_tile", 16, cap=64, rows_per_expert=2.0) == 16            # 128 > cap
        assert tactics.pick("mla_splits", 1, H=16, rows=64, keys=1040) == 3
        assert tactics.pick("mla_splits", 1, H=16, rows=63, keys=1040) == 1
        bad = tmp_path / "bad.json"
        bad.write_text(json.dumps({"warp_tile": []}))
        with pytest.raises(ValueError):
            tactics.load(str(bad))
    finally:
        tactics.set_table(None)


def test_heuristics_take_table_values():
    try:
        from b200ds.ops import cuda
    except ImportError as e:          # native library absent or stale on this machine
        pytest.skip(str(e))
    from b200ds.ops import tactics
    try:
        tactics.set_table({})
        d_split, d_tile, d_mla = cuda.choose_splits(64, 7168, 16384), cuda.moe_tile_n(2.0, 64), \
            cuda.mla_splits(64, 16, 1040)
        assert (d_split, d_tile) == (4, 16)
        tactics.set_table({"gemm_splits": [{"N": 7168, "K": 16384, "rows": [1, 64], "value": 2}],
                           "moe_tile": [{"cap": 64, "rows_per_expert": [0, 8], "value": 32}],
                           "mla_splits": [{"H": 16, "keys": [0, 2048], "value": d_mla + 1}]})
        assert cuda.choose_splits(64, 7168, 16384) == 2
        assert cuda.choose_splits(65, 7168, 16384) == d_split             # outside the band
        assert cuda.choose_splits(64, 7168, 16384, max_ctas=222) == 2
        assert cuda.moe_tile_n(2.0, 64) == 32 and cuda.moe_tile_n(2.0, 128) == 16
        assert cuda.mla_splits(64, 16, 1040) == d_mla + 1 and cuda.mla_splits(64, 128, 1040) >= 1
    finally:
        tactics.set_table(None)
