"""Loader for the reference's own CPU extension built by oracle/build.py.

TEST INFRASTRUCTURE ONLY.  The modules come from the reference's source files
(flashlog_kernel/source/flashlog.cpp and csr.cpp) compiled into oracle/_ref;
they are used to pin the C oracle and as the timed CPU baseline.
"""
from __future__ import annotations

import importlib.util
import os

from . import build as _build

_mods = {}


def available() -> bool:
    return all(os.path.exists(_build.ref_module_path(n)) for n in ("flashlog_ref_cpu", "flashlog_ref_csr"))


def module(name: str = "flashlog_ref_cpu"):
    if name not in _mods:
        path = _build.ref_module_path(name)
        if not os.path.exists(path):
            raise FileNotFoundError(f"reference module {path} is not built (run oracle/build.py)")
        import torch  # noqa: F401  (the extension links against libtorch)
        spec = importlib.util.spec_from_file_location(name, path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _mods[name] = mod
    return _mods[name]


def build_csr(head, tail, rel, nodes):
    """The reference CSR builder (csr.cpp) in the 16-tuple order of flashlog_kernel.py:695-697."""
    import numpy as np
    csr = module("flashlog_ref_csr")
    h, t, r = (np.ascontiguousarray(x, dtype=np.int64) for x in (head, tail, rel))
    ori = csr.build_side(h, t, r, int(nodes))
    inv = csr.build_side(t, h, r, int(nodes))
    return (*ori[:4], *inv[:4], *ori[4:], *inv[4:])
