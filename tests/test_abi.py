"""CPU checks of the drop-in boundary: liboxf.so loads without a GPU and
exports every function the public headers declare (no compute calls)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions() -> list[str]:
    names = set()
    for h in HEADERS:
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(oxf_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_headers_declare_functions():
    assert len(declared_functions()) > 20


def test_library_exports_every_declared_symbol():
    from oxf import _lib

    h = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(h, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    from oxf import _host_sigs, _lib

    bound = set(_lib._SIGS) | set(_host_sigs.SIGS)
    missing = [n for n in declared_functions() if n not in bound]
    assert not missing, missing


def test_status_strings_without_gpu():
    from oxf import _lib

    lib = _lib.lib()
    assert b"sm_100a" in lib.oxf_version()
    # argument validation runs on the host and never touches the device
    st = lib.oxf_matrix_softmax_rows(_lib.Slice(None, 10), 3, 1.0, 0, None)
    assert st == _lib.INVALID_ARG
    assert b"len % cols" in lib.oxf_last_error_string()


def test_product_never_imports_oracle():
    pkg = ROOT / "oxide-forge_b200"
    for f in list(pkg.rglob("*.py")) + list(pkg.rglob("*.cu")) + list(pkg.rglob("*.cpp")):
        if "_build" in f.parts:
            continue
        text = f.read_text()
        assert "oxf_oracle" not in text and "import oracle" not in text, f
