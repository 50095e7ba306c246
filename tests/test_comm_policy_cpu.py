"""Host-side choices of the fused all-reduce (no GPU needed): which protocol
a tensor-parallel all-reduce takes, from the measured sweep on one B200 box."""
import os

from b200ds.parallel.symm import FusedAllReduce, _Nvls
from b200ds.utils import levers


def _far(world, nvls=None):
    f = FusedAllReduce.__new__(FusedAllReduce)
    f.world, f.nvls = world, nvls
    return f


def test_one_kernel_only_for_few_pushed_rows():
    assert _far(2)._one_kernel(64)          # 2 ranks x 64 rows: one kernel measured faster
    f = _far(8)
    assert f._one_kernel(1)                 # 8 ranks x 1 row: one kernel
    assert not f._one_kernel(64)            # 8 ranks x 64 rows: push + reduce kernels
    before = levers.switches()["ar_one_kernel"]
    try:
        levers.set_switch("ar_one_kernel", False)
        assert not f._one_kernel(1)
    finally:
        levers.set_switch("ar_one_kernel", before)


def test_nvls_is_opt_in_on_one_box():
    old = os.environ.pop("B200_NVLS_MIN_WORLD", None)
    try:
        # the default leaves 8-rank groups on the push protocol, before any device work
        assert _Nvls.create(None, "t", None, 8, 0, 8, 256, "cpu") is None
    finally:
        if old is not None:
            os.environ["B200_NVLS_MIN_WORLD"] = old
