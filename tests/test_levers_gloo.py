"""Switch registry and fail-closed self-checks: a check that fails on one
rank turns its path off on every rank (MIN agreement over gloo)."""
from mp_util import run_ranks


def _rank(rank, world):
    from b200ds.parallel.state import init_parallel
    from b200ds.utils import levers
    ps = init_parallel(backend="gloo")
    levers.register("t_good", "B200_T_GOOD", True, "test: passes everywhere")
    levers.register("t_bad", "B200_T_BAD", True, "test: fails on rank 1")
    levers.register("t_raise", "B200_T_RAISE", True, "test: raises on rank 0")
    levers.add_check("t_good", lambda: True)
    levers.add_check("t_bad", lambda: rank != 1)

    def boom():
        if rank == 0:
            raise ValueError("x")
        return True
    levers.add_check("t_raise", boom)
    res = levers.selfcheck(ps.cpu_group)
    # no group: a single-rank parallel state inside the job agrees locally
    # (only this rank calls it; a collective here would never complete)
    local = levers.agree_min([10 + rank], None) if rank == 1 else [10]
    return res, levers.on("t_good"), levers.on("t_bad"), levers.on("t_raise"), local


def test_selfcheck_agrees_min_over_ranks():
    out = run_ranks(_rank, 2)
    for rank, (res, good, bad, rz, local) in enumerate(out):
        assert res["t_good"] and not res["t_bad"] and not res["t_raise"]
        assert good and not bad and not rz
        assert local == [10 + rank]


def test_switch_env_override(monkeypatch):
    from b200ds.utils import levers
    sw = levers.register("t_env", "B200_T_ENV", True, "test")
    monkeypatch.setenv("B200_T_ENV", "0")
    sw.value = None
    assert not levers.on("t_env")
    levers.set_switch("t_env", True)
    assert levers.on("t_env") and "moe_fused" in levers.switches()
