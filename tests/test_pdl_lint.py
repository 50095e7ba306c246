"""Static checks of the CUDA sources for the programmatic-dependent-launch
rules every kernel relies on (no GPU needed):

* a kernel launched with PDL (`launch_pdl(kernel, ...)`) may start while its
  predecessor still runs, so its body must execute `pdl_wait()` (which also
  makes the predecessor's writes visible) before touching dependent data;
* after that wait, predecessor outputs must not be read through the
  non-coherent path (`__ldg` / `ld.global.nc`): a line cached there earlier
  would not see the predecessor's writes.  The sources use `__ldcg` instead.
"""
import glob
import os
import re

ROOT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "csrc")


def _sources():
    for p in sorted(glob.glob(os.path.join(ROOT, "**", "*.cu"), recursive=True) +
                    glob.glob(os.path.join(ROOT, "**", "*.cuh"), recursive=True)):
        with open(p) as f:
            yield p, f.read()


def _kernel_bodies(src):
    """name -> body text of every __global__ function."""
    out = {}
    for m in re.finditer(r"__global__\s+void\s+(?:__launch_bounds__\([^)]*\)\s*)?(\w+)\s*\(", src):
        i = src.index("{", m.end())
        depth, j = 0, i
        while True:
            if src[j] == "{":
                depth += 1
            elif src[j] == "}":
                depth -= 1
                if depth == 0:
                    break
            j += 1
        out[m.group(1)] = src[i:j + 1]
    return out


def test_no_noncoherent_loads():
    bad = []
    for p, src in _sources():
        code = re.sub(r"//[^\n]*", "", src)
        for tok in ("__ldg(", "ld.global.nc"):
            if tok in code:
                bad.append((os.path.relpath(p, ROOT), tok))
    assert not bad, bad


def test_pdl_launched_kernels_wait():
    bodies, launched = {}, set()
    for _, src in _sources():
        bodies.update(_kernel_bodies(src))
        for m in re.finditer(r"launch_pdl\(\s*([\w:<>, ]+?)\s*,\s*dim3", src):
            launched.add(m.group(1).split("::")[-1].split("<")[0].strip())
    assert launched, "no PDL launches found"
    missing = [k for k in sorted(launched) if k in bodies and "pdl_wait()" not in bodies[k]]
    assert not missing, missing
