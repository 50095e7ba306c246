"""Source-hash pin of the native extension.

The build records a digest of every native source under csrc/ next to the
built library (`b200ds/_C.srcpin`).  Importing the CUDA op layer from a source
tree whose csrc/ no longer matches that digest raises, so a library built
from older sources is never run in place of the current kernels (switch
`srcpin`, B200_SRCPIN=0 to skip the check; a library without a pin file is
announced, not refused).

Reference parity: the reference pins the stock sources its levers patch by
hash and turns a lever off when they drift (levers.py:172-194, *_PINS).
"""
from __future__ import annotations

import hashlib
import os
from typing import Optional

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ROOT = os.path.dirname(PKG)
PIN_FILE = os.path.join(PKG, "_C.srcpin")
_EXT = (".cu", ".cuh", ".h", ".hpp", ".cpp")


def source_digest(csrc: Optional[str] = None) -> Optional[str]:
    """sha256 over (relative path, bytes) of the native sources, in path
    order; None when there is no csrc/ (an installed package)."""
    csrc = csrc or os.path.join(ROOT, "csrc")
    if not os.path.isdir(csrc):
        return None
    h = hashlib.sha256()
    files = []
    for d, _, names in os.walk(csrc):
        files += [os.path.join(d, n) for n in names if n.endswith(_EXT)]
    for f in sorted(files, key=lambda p: os.path.relpath(p, csrc)):
        h.update(os.path.relpath(f, csrc).replace(os.sep, "/").encode() + b"\0")
        with open(f, "rb") as fh:
            h.update(fh.read())
        h.update(b"\0")
    return h.hexdigest()


def write_pin(csrc: Optional[str] = None, pin_file: str = PIN_FILE) -> Optional[str]:
    d = source_digest(csrc)
    if d is not None:
        with open(pin_file, "w") as f:
            f.write(d + "\n")
    return d


def check_pin(csrc: Optional[str] = None, pin_file: str = PIN_FILE) -> Optional[str]:
    """None when the built library matches the sources (or there is nothing
    to compare: no csrc/, or a library built without a pin, which is only
    announced), else a one-line reason."""
    cur = source_digest(csrc)
    if cur is None:
        return None
    if not os.path.exists(pin_file):
        from . import levers
        levers.announce("srcpin-missing", "native library without a source pin (not built by setup.py): "
                        "its sources are not checked")
        return None
    with open(pin_file) as f:
        pinned = f.read().strip()
    if pinned != cur:
        return "csrc/ changed since the native library was built: rebuild (python setup.py build_ext --inplace)"
    return None
