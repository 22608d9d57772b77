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


# ctypes structure -> (C type name, {ctypes field: C member})
def _layouts():
    from oxf import _host_sigs as H, _lib as L

    def same(cls, **rename):
        return {f: rename.get(f, f) for f, _ in cls._fields_}

    return {
        L.CSlice: ("oxf_cslice", same(L.CSlice)),
        L.Slice: ("oxf_slice", same(L.Slice)),
        L.GemmDesc: ("oxf_gemm_desc", same(L.GemmDesc)),
        L.GemmPlanInfo: ("oxf_gemm_plan_info", same(L.GemmPlanInfo)),
        L.IpcHandle: ("oxf_ipc_handle", same(L.IpcHandle)),
        L.ExchangeDesc: ("oxf_exchange_desc", same(L.ExchangeDesc)),
        H.LayerSpec: ("oxf_layer_spec", same(H.LayerSpec, in_="in")),
        H.MlpSpec: ("oxf_mlp_spec", same(H.MlpSpec)),
        H.TransformerSpec: ("oxf_transformer_spec", same(H.TransformerSpec)),
    }


# Python constant -> C constant of the headers
_CONSTANTS = {
    "OK": "OXF_OK", "INVALID_ARG": "OXF_ERR_INVALID_ARG",
    "UNSUPPORTED_SHAPE": "OXF_ERR_UNSUPPORTED_SHAPE", "CUDA_ERROR": "OXF_ERR_CUDA",
    "TIMEOUT": "OXF_ERR_TIMEOUT", "DEVICE_CHECK": "OXF_ERR_DEVICE_CHECK", "IO": "OXF_ERR_IO",
    "STATE": "OXF_ERR_STATE",
    "ADD": "OXF_ADD", "SUB": "OXF_SUB", "MUL": "OXF_MUL", "DIV": "OXF_DIV",
    "ACT_IDENTITY": "OXF_ACT_IDENTITY", "ACT_GELU": "OXF_ACT_GELU", "ACT_RELU": "OXF_ACT_RELU",
    "ACT_SILU": "OXF_ACT_SILU",
    "UNARY_SCALE": "OXF_UNARY_SCALE", "UNARY_ADD_SCALAR": "OXF_UNARY_ADD_SCALAR",
    "UNARY_ACT_FORWARD": "OXF_UNARY_ACT_FORWARD", "UNARY_ACT_DERIV": "OXF_UNARY_ACT_DERIV",
    "UNARY_HALF_SQUARE": "OXF_UNARY_HALF_SQUARE",
    "PREC_TF32": "OXF_PREC_TF32", "PREC_TF32X3": "OXF_PREC_TF32X3", "PREC_F32": "OXF_PREC_F32",
    "GEMM_PATH_NONE": "OXF_GEMM_PATH_NONE", "GEMM_PATH_SIMT": "OXF_GEMM_PATH_SIMT",
    "GEMM_PATH_TINY": "OXF_GEMM_PATH_TINY", "GEMM_PATH_ONE_CTA": "OXF_GEMM_PATH_ONE_CTA",
    "GEMM_PATH_CTA_PAIR": "OXF_GEMM_PATH_CTA_PAIR",
    "NORM_RMS": "OXF_NORM_RMS", "NORM_LAYER": "OXF_NORM_LAYER",
    "EXCHANGE_MAX_RANKS": "OXF_EXCHANGE_MAX_RANKS",
    "EXCHANGE_MAX_BLOCKS": "OXF_EXCHANGE_MAX_BLOCKS",
    "EXCHANGE_SIGNAL_BYTES": "OXF_EXCHANGE_SIGNAL_BYTES",
    "DEVERR_EXCHANGE_START": "OXF_DEVERR_EXCHANGE_START",
    "DEVERR_EXCHANGE_END": "OXF_DEVERR_EXCHANGE_END",
}


def test_binding_layouts_match_headers(tmp_path):
    """Every structure the binding passes by value or pointer has the C
    header's size and member offsets, and every constant its value, as the
    host C compiler lays them out (a mismatch would hand the library
    shifted arguments without any error)."""
    import shutil
    import subprocess

    from oxf import _host_sigs as H, _lib as L

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    layouts = _layouts()
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "oxf_host.h"',
             "int main(void) {"]
    for cls, (cname, fields) in layouts.items():
        lines.append(f'  printf("{cls.__name__} size %zu\\n", sizeof({cname}));')
        for py, c in fields.items():
            lines.append(f'  printf("{cls.__name__} {py} %zu\\n", offsetof({cname}, {c}));')
    for py, c in _CONSTANTS.items():
        lines.append(f'  printf("const {py} %lld\\n", (long long)({c}));')
    lines.append(f'  printf("const MAX_LAYERS %d\\n", OXF_MAX_LAYERS);')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-std=c11", "-Wall", "-Werror", "-I", str(ROOT / "include"), str(src),
                    "-o", str(exe)], check=True, capture_output=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    got = {}
    for line in out.splitlines():
        owner, name, value = line.split()
        got[(owner, name)] = int(value)
    bad = []
    for cls, (_, fields) in layouts.items():
        if got[(cls.__name__, "size")] != ctypes.sizeof(cls):
            bad.append((cls.__name__, "size", got[(cls.__name__, "size")], ctypes.sizeof(cls)))
        for py in fields:
            off = getattr(cls, py).offset
            if got[(cls.__name__, py)] != off:
                bad.append((cls.__name__, py, got[(cls.__name__, py)], off))
    for py in _CONSTANTS:
        if got[("const", py)] != getattr(L, py):
            bad.append(("const", py, got[("const", py)], getattr(L, py)))
    if got[("const", "MAX_LAYERS")] != H.MAX_LAYERS:
        bad.append(("const", "MAX_LAYERS", got[("const", "MAX_LAYERS")], H.MAX_LAYERS))
    assert not bad, bad


def _header_signatures() -> dict[str, int]:
    """Function name -> parameter count, from the public headers."""
    sigs = {}
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"#.*", "", text)
        for m in re.finditer(r"\b(oxf_[a-z0-9_]+)\s*\(([^;{)]*)\)\s*;", text):
            args = m.group(2).strip()
            sigs[m.group(1)] = 0 if args in ("", "void") else args.count(",") + 1
    return sigs


def test_rust_binding_matches_headers():
    """include/oxf_ffi.rs, the complete Rust binding for the reference's
    maintainers, declares exactly the headers' functions with the headers'
    parameter counts, and its structures list the C members in the C order."""
    block = (ROOT / "include" / "oxf_ffi.rs").read_text()
    rust = {}
    for m in re.finditer(r"pub fn (oxf_[a-z0-9_]+)\(([^)]*)\)", block):
        args = m.group(2).strip()
        rust[m.group(1)] = 0 if not args else args.count(":")
    assert rust == _header_signatures()
    for cls, (cname, fields) in _layouts().items():
        m = re.search(r"pub struct " + cname + r"\s*\{([^}]*)\}", block)
        assert m, cname
        names = re.findall(r"pub (\w+):", m.group(1))
        assert names == [c if c != "in" else "in_" for c in fields.values()], cname


def test_plain_c_client(tmp_path):
    """tests/c_client/abi_client.c, compiled by the host C compiler against
    the public headers only and linked to liboxf.so, runs its checks (no GPU
    calls): the library is a drop-in for a C-ABI host as it stands."""
    import shutil
    import subprocess

    from oxf import _lib

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lib_dir = Path(_lib.LIB_PATH).parent
    exe = tmp_path / "abi_client"
    subprocess.run([cc, "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "c_client" / "abi_client.c"), "-o", str(exe),
                    "-L", str(lib_dir), "-loxf", f"-Wl,-rpath,{lib_dir}"],
                   check=True, capture_output=True)
    r = subprocess.run([str(exe), str(tmp_path / "mlp_ckpt")], capture_output=True, text=True,
                       timeout=60)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "ok"
    assert (tmp_path / "mlp_ckpt.toml").exists() and (tmp_path / "mlp_ckpt.bin").exists()


def test_stack_validates_block_widths_without_gpu():
    """TransformerStack refuses blocks whose widths do not chain (block i's
    output must be block i+1's hidden width, at the same sequence length)
    before it creates any engine."""
    from oxf import models
    a = models.transformer_config(16, 64, 128, out=32)
    b = models.transformer_config(16, 64, 128)
    c = models.transformer_config(8, 64, 128)
    for cfgs in ([a, b], [b, c], []):
        with pytest.raises(ValueError):
            models.TransformerStack(cfgs)
