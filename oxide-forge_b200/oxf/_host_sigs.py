"""ctypes signatures of the host-layer C ABI (include/oxf_host.h)."""
from __future__ import annotations

import ctypes as C

SIGS: dict = {}


def bind(h: C.CDLL) -> None:
    for name, (res, args) in SIGS.items():
        f = getattr(h, name)
        f.restype = res
        f.argtypes = args
