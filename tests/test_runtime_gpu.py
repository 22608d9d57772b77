"""The C++ host layer that mirrors the reference's CudaRuntime, Matrix,
Vector and Linear (oxide-forge_b200/host/runtime.hpp, linear.hpp;
src/cuda/runtime.rs, src/cuda/container/*.rs, src/net/linear.rs), driven by
a compiled C++ client (tests/c_client/runtime_client.cpp) linked to
liboxf.so only. The client checks the pool's exact-size reuse and
reserve_buffers itself; every device result it writes is checked here
against the oracle.

Tolerances: TF32 products 5e-3 of max|want| (oracle with the reference's
RNA operand rounding); row / elementwise operations 1e-5 (backward kernels:
of the scale of the terms they combine).
"""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from conftest import rel_err

ROOT = Path(__file__).resolve().parent.parent
RNA = O.GEMM_TF32_RNA
F32 = np.float32
R, C, N, S = 96, 160, 72, 48


def build_client(out_dir: Path) -> Path:
    """Compiles the client against the public headers and the host layer's
    headers, linked to liboxf.so (no CUDA library of its own)."""
    from oxf import _lib
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    lib_dir = Path(_lib.LIB_PATH).parent
    exe = out_dir / "runtime_client"
    subprocess.run([cxx, "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror",
                    "-I", str(ROOT / "include"), "-I", str(ROOT / "oxide-forge_b200" / "host"),
                    "-I", "/usr/local/cuda/include",
                    str(ROOT / "tests" / "c_client" / "runtime_client.cpp"), "-o", str(exe),
                    "-L", str(lib_dir), "-loxf", f"-Wl,-rpath,{lib_dir}"],
                   check=True, capture_output=True)
    return exe


def test_client_builds_against_the_host_layer(tmp_path):
    """CPU check: the host layer's C++ classes are exported by liboxf.so and
    a client links against them."""
    assert build_client(tmp_path).exists()


@pytest.mark.gpu
def test_runtime_matrix_vector_linear_on_the_gpu(tmp_path):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    exe = build_client(tmp_path)
    rng = np.random.default_rng(77)
    ins = {
        "a": rng.standard_normal((R, C)), "a2": rng.standard_normal((R, C)),
        "b": rng.uniform(-1, 1, (C, N)), "v": rng.standard_normal(C) + 2.0,
        "sq": rng.standard_normal((S, S)), "dyc": rng.standard_normal((R, C)),
        "w": rng.uniform(-0.15, 0.15, (C, N)), "bias": 0.1 * rng.standard_normal(N),
        "dyn": rng.standard_normal((R, N)), "t": rng.standard_normal((R, N)),
    }
    ins = {k: np.ascontiguousarray(v, F32) for k, v in ins.items()}
    for k, v in ins.items():
        v.tofile(tmp_path / f"{k}.bin")
    (tmp_path / "dims.txt").write_text(f"{R} {C} {N} {S}\n")
    r = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    lines = dict(l.split(" ", 1) for l in r.stdout.strip().splitlines() if " " in l)
    assert r.stdout.strip().endswith("ok")

    def out(name, shape):
        return np.fromfile(tmp_path / f"out_{name}.bin", F32).reshape(shape)

    a, a2, b, v = ins["a"], ins["a2"], ins["b"], ins["v"]
    dyc = ins["dyc"]
    assert rel_err(out("mm", (R, N)), O.gemm(a, b, rounding=RNA)) < 5e-3
    np.testing.assert_array_equal(out("transpose", (C, R)), a.T)
    assert rel_err(out("sum_rows", (R,)), O.sum_rows(a)) < 1e-5
    assert rel_err(out("sum_cols", (C,)), O.sum_cols(a)) < 1e-5
    np.testing.assert_array_equal(out("sub", (R, C)), a - a2)
    np.testing.assert_array_equal(out("mul", (R, C)), a * a2)
    p = O.softmax_rows(a)
    assert rel_err(out("softmax", (R, C)), p) < 1e-5
    got = out("softmax_bwd", (R, C))
    assert np.abs(got - O.softmax_backward(out("softmax", (R, C)), dyc)).max() <= \
        1e-5 * np.abs(p * dyc).max()
    assert rel_err(out("layer_norm", (R, C)), O.layer_norm_rows(a)) < 1e-5
    inv_std = 1 / np.sqrt(a.var(axis=1, keepdims=True) + 1e-5)
    assert np.abs(out("layer_norm_bwd", (R, C)) - O.layer_norm_backward(a, dyc)).max() <= \
        1e-5 * np.abs(inv_std * dyc).max()
    assert rel_err(out("rms_norm", (R, C)), O.rms_norm_rows(a)) < 1e-5
    inv_r = 1 / np.sqrt((a * a).mean(axis=1, keepdims=True) + 1e-5)
    assert np.abs(out("rms_norm_bwd", (R, C)) - O.rms_norm_backward(a, dyc)).max() <= \
        1e-5 * np.abs(inv_r * dyc).max()
    assert rel_err(out("gelu", (R, C)), O.act_forward(O.GELU, a)) < 1e-5
    assert rel_err(out("gelu_deriv", (R, C)), O.act_derivative(O.GELU, a)) < 1e-5
    want = O.binary_assign_by_rows(a, v, 2) * F32(0.5) + F32(1.0)
    assert rel_err(out("by_rows_scale_add", (R, C)), want) < 1e-5
    np.testing.assert_array_equal(out("causal_mask", (S, S)), O.causal_mask(ins["sq"]))
    assert abs(float(lines["v_sum"]) - float(v.astype(np.float64).sum())) <= \
        1e-5 * float(np.abs(v).sum())
    assert F32(float(lines["v_max"])) == v.max()  # printed with 9 digits: f32 round trip
    assert rel_err(out("fork_join", (R, C)), (a * F32(3) - F32(1)) + np.maximum(a2, 0)) < 1e-6

    # Linear: forward, affine, loss_rows, backward, input_gradient, learn
    w, bias, dyn, t = ins["w"], ins["bias"], ins["dyn"], ins["t"]
    y_ref, z_ref = O.linear_forward(O.LinearParams(w, bias, O.GELU), a, rounding=RNA)
    assert rel_err(out("lin_y", (R, N)), y_ref) < 5e-3
    assert rel_err(out("lin_z", (R, N)), z_ref) < 5e-3
    assert rel_err(out("lin_loss", (R,)), O.loss_rows(out("lin_y", (R, N)), t)) < 1e-5
    z = out("lin_z", (R, N))
    g_ref = dyn * O.act_derivative(O.GELU, z)
    assert rel_err(out("lin_g", (R, N)), g_ref) < 1e-5
    assert rel_err(out("lin_bg", (N,)), O.sum_cols(g_ref)) < 1e-5
    g = out("lin_g", (R, N))
    assert rel_err(out("lin_dx", (R, C)), O.gemm(g, w, b_trans=True, rounding=RNA)) < 5e-3
    assert rel_err(w - out("lin_w_new", (C, N)),
                   0.05 * O.gemm(a, g, a_trans=True, rounding=RNA)) < 5e-3
    assert rel_err(bias - out("lin_b_new", (N,)), 0.05 * out("lin_bg", (N,))) < 1e-4
    # every Matrix / Vector the client dropped went back to the exact-size pool
    assert int(lines["pooled_at_end"]) > int(lines["pooled_after_scope"])
