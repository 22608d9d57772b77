"""Generates tests/golden/golden.npz: small seeded inputs with expected
outputs from an independent numpy float64 restatement of the reference
formulas (MeccBai/oxide-forge). The C oracle (oracle/oxf_oracle.c) is checked
against these fixtures; neither is derived from the other.

The reference itself ships no tests, golden vectors or fixtures and cannot
be built here (Rust + cuda-oxide toolchain absent), so these fixtures pin the
oracle to the formulas as written in the reference source, cited per entry.

Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "golden.npz"
EPS = 1e-5
GELU_SCALE = 0.7978846
GELU_CUBIC = 0.044715


def gelu(x):  # linear.rs:30-33
    return 0.5 * x * (1.0 + np.tanh(GELU_SCALE * (x + GELU_CUBIC * x ** 3)))


def gelu_d(x):  # linear.rs:49-56
    th = np.tanh(GELU_SCALE * (x + GELU_CUBIC * x ** 3))
    return 0.5 * (1 + th) + 0.5 * x * (1 - th * th) * (GELU_SCALE + 3 * GELU_SCALE * GELU_CUBIC * x * x)


def softmax(x):  # row.rs:55-113
    m = x.max(axis=1, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=1, keepdims=True)


def layer_norm(x):  # row.rs:115-177
    mu = x.mean(axis=1, keepdims=True)
    var = ((x - mu) ** 2).mean(axis=1, keepdims=True)
    return (x - mu) / np.sqrt(var + EPS)


def rms_norm(x):  # row.rs:349-396
    return x / np.sqrt((x * x).mean(axis=1, keepdims=True) + EPS)


def softmax_bwd(p, dy):  # row.rs:193-237
    return p * (dy - (p * dy).sum(axis=1, keepdims=True))


def layer_norm_bwd(x, dy):  # row.rs:239-347
    n = x.shape[1]
    mu = x.mean(axis=1, keepdims=True)
    inv = 1.0 / np.sqrt(((x - mu) ** 2).mean(axis=1, keepdims=True) + EPS)
    xh = (x - mu) * inv
    return inv / n * (n * dy - dy.sum(axis=1, keepdims=True) - xh * (dy * xh).sum(axis=1, keepdims=True))


def rms_norm_bwd(x, dy):  # row.rs:398-468
    n = x.shape[1]
    r = np.sqrt((x * x).mean(axis=1, keepdims=True) + EPS)
    return dy / r - x * ((x * dy).sum(axis=1, keepdims=True) / n) / r ** 3


def transformer_step(p, x, t, norm, lr):
    """TrainingTransformer forward + backward on one sequence with immediate
    SGD (encoder.rs:114-186, attention.rs:258-321, mlp.rs:121-168), all
    Linears Identity except FFN layer 0 (GELU), no biases. Returns y, dx and
    the updated parameters."""
    nf = layer_norm if norm == "layer" else rms_norm
    nb = layer_norm_bwd if norm == "layer" else rms_norm_bwd
    Wq, Wk, Wv, P, W1, W2, Wo = (p[k].astype(np.float64) for k in ("wq", "wk", "wv", "pos", "w1", "w2", "wo"))
    D = Wq.shape[1]
    s = 1.0 / np.sqrt(D)
    pos = x + P
    q, k, v = pos @ Wq, pos @ Wk, pos @ Wv
    pr = softmax((q @ k.T) * s)
    pre = pos + pr @ v
    h1 = nf(pre)
    z1 = h1 @ W1
    a1 = gelu(z1)
    f = a1 @ W2
    pre2 = h1 + f
    enc = nf(pre2)
    y = enc @ Wo
    dy = (y - t) / y.shape[1]
    d_enc = dy @ Wo.T
    gWo = enc.T @ dy
    d2 = nb(pre2, d_enc)
    gW2 = a1.T @ d2
    da1 = d2 @ W2.T
    dz1 = da1 * gelu_d(z1)
    gW1 = h1.T @ dz1
    dh1 = dz1 @ W1.T
    d1 = d2 + dh1
    dr = nb(pre, d1)
    dp = dr @ v.T
    dv = pr.T @ dr
    ds = softmax_bwd(pr, dp) * s
    dq = ds @ k
    dk = ds.T @ q
    gWq, gWk, gWv = pos.T @ dq, pos.T @ dk, pos.T @ dv
    dpos = dr + dq @ Wq.T + dk @ Wk.T + dv @ Wv.T
    new = {"wq": Wq - lr * gWq, "wk": Wk - lr * gWk, "wv": Wv - lr * gWv, "pos": P - lr * dpos,
           "w1": W1 - lr * gW1, "w2": W2 - lr * gW2, "wo": Wo - lr * gWo}
    return y, dpos, new


def main() -> None:
    rng = np.random.default_rng(20261201)
    g = {}
    R, Cc = 7, 36
    x = rng.standard_normal((R, Cc)).astype(np.float32)
    dy = rng.standard_normal((R, Cc)).astype(np.float32)
    xd = x.astype(np.float64)
    g["rows_x"], g["rows_dy"] = x, dy
    g["softmax"] = softmax(xd)
    g["layer_norm"] = layer_norm(xd)
    g["rms_norm"] = rms_norm(xd)
    pr = softmax(xd)
    g["softmax_bwd"] = softmax_bwd(pr, dy.astype(np.float64))
    g["layer_norm_bwd"] = layer_norm_bwd(xd, dy.astype(np.float64))
    g["rms_norm_bwd"] = rms_norm_bwd(xd, dy.astype(np.float64))
    g["gelu"] = gelu(xd)
    g["gelu_d"] = gelu_d(xd)
    g["sum_rows"] = xd.sum(axis=1)
    g["sum_cols"] = xd.sum(axis=0)
    t = rng.standard_normal((R, Cc)).astype(np.float32)
    g["loss_t"] = t
    g["loss_rows"] = (0.5 * (xd - t) ** 2).mean(axis=1)  # linear.rs:325-333
    A = rng.uniform(-1, 1, (24, 40)).astype(np.float32)
    B = rng.uniform(-1, 1, (40, 16)).astype(np.float32)
    g["gemm_a"], g["gemm_b"] = A, B
    g["gemm_c"] = A.astype(np.float64) @ B.astype(np.float64)
    # tiny transformer step, both norms
    S, H, F = 8, 12, 20
    for norm in ("layer", "rms"):
        p = {
            "wq": rng.uniform(-0.4, 0.4, (H, H)), "wk": rng.uniform(-0.4, 0.4, (H, H)),
            "wv": rng.uniform(-0.4, 0.4, (H, H)), "pos": 0.02 * rng.standard_normal((S, H)),
            "w1": rng.uniform(-0.4, 0.4, (H, F)), "w2": rng.uniform(-0.3, 0.3, (F, H)),
            "wo": rng.uniform(-0.4, 0.4, (H, H)),
        }
        p = {k: v.astype(np.float32) for k, v in p.items()}
        xs = rng.standard_normal((S, H)).astype(np.float32)
        ts = rng.standard_normal((S, H)).astype(np.float32)
        y, dpos, new = transformer_step(p, xs.astype(np.float64), ts.astype(np.float64), norm, 0.05)
        for k, v in p.items():
            g[f"tf_{norm}_{k}"] = v
            g[f"tf_{norm}_{k}_new"] = new[k]
        g[f"tf_{norm}_x"], g[f"tf_{norm}_t"] = xs, ts
        g[f"tf_{norm}_y"], g[f"tf_{norm}_dx"] = y, dpos
    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({len(g)} arrays)")


if __name__ == "__main__":
    main()
