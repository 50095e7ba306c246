"""Source-hash pin of the native library: the digest covers every native
source, changes with any byte or file name, and a library whose pin differs
from the tree's sources is reported stale."""
import os


def test_pin_detects_changed_sources(tmp_path):
    from b200ds.utils.srcpin import check_pin, source_digest, write_pin
    csrc = tmp_path / "csrc"
    (csrc / "gemm").mkdir(parents=True)
    (csrc / "gemm" / "a.cu").write_text("__global__ void k() {}\n")
    (csrc / "b.h").write_text("#pragma once\n")
    (csrc / "notes.txt").write_text("not a source")
    pin = str(tmp_path / "_C.srcpin")
    assert check_pin(str(csrc), pin) is None              # no pin file: announced, not refused
    d0 = write_pin(str(csrc), pin)
    assert check_pin(str(csrc), pin) is None
    (csrc / "notes.txt").write_text("still not a source")
    assert source_digest(str(csrc)) == d0
    (csrc / "b.h").write_text("#pragma once\n// edit\n")
    assert "rebuild" in check_pin(str(csrc), pin)
    write_pin(str(csrc), pin)
    os.rename(csrc / "gemm" / "a.cu", csrc / "gemm" / "c.cu")     # same bytes, new name
    assert check_pin(str(csrc), pin) is not None
    assert source_digest(str(tmp_path / "absent")) is None and check_pin(str(tmp_path / "absent"), pin) is None
