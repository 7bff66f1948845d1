"""Loads the package's in-tree native libraries. There is no fallback: a missing
library is an error that names the build step to run."""
from __future__ import annotations

import ctypes as C
import os

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
_cache: dict[str, C.CDLL] = {}


class NativeLibraryMissing(ImportError):
    pass


def path(name: str) -> str:
    return os.path.join(PKG_DIR, name)


def load(name: str) -> C.CDLL:
    if name not in _cache:
        p = path(name)
        if not os.path.exists(p):
            raise NativeLibraryMissing(
                f"{p} is not built; run `python -c 'import __graft_entry__ as g; g.build()'` "
                f"or `make -C {PKG_DIR}/csrc`")
        _cache[name] = C.CDLL(p, mode=C.RTLD_GLOBAL)
    return _cache[name]
