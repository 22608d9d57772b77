/*
 * oxf_oracle.c — CPU oracle for the OxideForge compute hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see oxf_oracle.h): a scalar f32 restatement of
 * the reference's arithmetic, used by tests/ as the parity checker and by
 * bench.py as the timed CPU baseline. The product library never links it.
 *
 * PARITY UNPINNED against the reference itself: the reference (Rust +
 * cuda-oxide) has no tests or golden vectors and cannot be built here. The
 * oracle is pinned by hand-derived known answers and by golden fixtures from
 * an independent numpy restatement (tests/golden/make_golden.py).
 *
 * Reference paths below are relative to the MeccBai/oxide-forge project root.
 */
#include "oxf_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------------ */
/* threads                                                                   */

static int g_threads = 0;

int oxo_set_threads(int n) {
    if (n <= 0) {
        long c = sysconf(_SC_NPROCESSORS_ONLN);
        n = c > 0 ? (int)c : 1;
    }
    g_threads = n;
    return g_threads;
}

int oxo_get_threads(void) {
    if (g_threads <= 0) oxo_set_threads(0);
    return g_threads;
}

/* ------------------------------------------------------------------------ */
/* pairwise sums                                                             */

/* Row reductions in the reference are shuffle trees over 32 lanes and then
 * over 32 warps (row.rs:35-48): a pairwise sum restates them faithfully and,
 * unlike a running sum, keeps the error O(log n) for wide rows. */
static float psum(const float* x, size_t n) {
    if (n <= 32) {
        float s = 0.0f;
        for (size_t i = 0; i < n; ++i) s += x[i];
        return s;
    }
    size_t h = n / 2;
    return psum(x, h) + psum(x + h, n - h);
}

static float* g_tmp = NULL;
static size_t g_tmp_n = 0;
static float* tmpbuf(size_t n) {
    if (n > g_tmp_n) {
        free(g_tmp);
        g_tmp = (float*)malloc((n ? n : 1) * sizeof(float));
        g_tmp_n = n;
    }
    return g_tmp;
}

/* ------------------------------------------------------------------------ */
/* TF32 rounding                                                             */

static inline uint32_t f2u(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static inline float u2f(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

/* cvt.rna.tf32.f32 as used by gemm.rs:286-347: keep 10 explicit mantissa
 * bits, round half away from zero on the 13 dropped bits. Non-finite values
 * pass through. */
float oxo_tf32_rna(float x) {
    uint32_t u = f2u(x);
    if ((u & 0x7f800000u) == 0x7f800000u) return x;
    u += 0x1000u;              /* half of the dropped 13-bit field */
    u &= 0xffffe000u;
    return u2f(u);
}

/* Truncation to TF32 (the tensor core reading raw f32 operands). */
float oxo_tf32_rz(float x) {
    uint32_t u = f2u(x);
    if ((u & 0x7f800000u) == 0x7f800000u) return x;
    return u2f(u & 0xffffe000u);
}

static inline float round_op(float x, int rounding) {
    if (rounding == OXO_GEMM_TF32_RNA) return oxo_tf32_rna(x);
    if (rounding == OXO_GEMM_TF32_RZ) return oxo_tf32_rz(x);
    return x;
}

/* ------------------------------------------------------------------------ */
/* GEMM                                                                      */

static inline float a_at(const float* A, size_t M, size_t K, int at, size_t m, size_t k) {
    return at ? A[k * M + m] : A[m * K + k];
}
static inline float b_at(const float* B, size_t N, size_t K, int bt, size_t k, size_t n) {
    return bt ? B[n * K + k] : B[k * N + n];
}

/* matrix_multiply_device, gemm.rs:202-373: each output is an f32 sum of
 * products of (optionally TF32-rounded) operands over k ascending.
 * Operands are first copied into row-major A[M,K] and B[K,N] with the
 * rounding applied (so transposed inputs cost one O(MK + KN) pass), then
 * rows are processed four at a time against 512-column panels of B: the
 * same sums in the same order, with a quarter of the B traffic. */
enum { RB = 4, NB = 512 };

static void gemm_panel(const float* restrict A, const float* restrict B, float* restrict C,
                       size_t N, size_t K, float alpha, float beta, size_t r0, size_t r1) {
    float acc[RB][NB];
    for (size_t m0 = r0; m0 < r1; m0 += RB) {
        const size_t rb = (r1 - m0) < RB ? (r1 - m0) : RB;
        for (size_t n0 = 0; n0 < N; n0 += NB) {
            const size_t nb = (N - n0) < NB ? (N - n0) : NB;
            for (size_t r = 0; r < RB; ++r)
                for (size_t j = 0; j < NB; ++j) acc[r][j] = 0.0f;
            for (size_t k = 0; k < K; ++k) {
                const float* restrict b = B + k * N + n0;
                if (rb == RB && nb == NB) {
                    const float a0 = A[(m0 + 0) * K + k], a1 = A[(m0 + 1) * K + k];
                    const float a2 = A[(m0 + 2) * K + k], a3 = A[(m0 + 3) * K + k];
                    for (size_t j = 0; j < NB; ++j) {
                        const float bj = b[j];
                        acc[0][j] += a0 * bj;
                        acc[1][j] += a1 * bj;
                        acc[2][j] += a2 * bj;
                        acc[3][j] += a3 * bj;
                    }
                } else {
                    for (size_t r = 0; r < rb; ++r) {
                        const float a = A[(m0 + r) * K + k];
                        for (size_t j = 0; j < nb; ++j) acc[r][j] += a * b[j];
                    }
                }
            }
            for (size_t r = 0; r < rb; ++r)
                for (size_t j = 0; j < nb; ++j) {
                    float v = alpha * acc[r][j];
                    float* c = C + (m0 + r) * N + n0 + j;
                    if (beta != 0.0f) v += beta * *c;
                    *c = v;
                }
        }
    }
}

/* Row-major, rounded copies of the operands. */
static float* prep_a(const float* A, size_t M, size_t K, int at, int rounding) {
    const size_t na = M * K;
    float* a = (float*)malloc((na ? na : 1) * sizeof(float));
    for (size_t m = 0; m < M; ++m)
        for (size_t k = 0; k < K; ++k) a[m * K + k] = round_op(a_at(A, M, K, at, m, k), rounding);
    return a;
}
static float* prep_b(const float* B, size_t N, size_t K, int bt, int rounding) {
    const size_t nbk = N * K;
    float* b = (float*)malloc((nbk ? nbk : 1) * sizeof(float));
    if (bt) {
        for (size_t n = 0; n < N; ++n)
            for (size_t k = 0; k < K; ++k) b[k * N + n] = round_op(B[n * K + k], rounding);
    } else {
        for (size_t i = 0; i < N * K; ++i) b[i] = round_op(B[i], rounding);
    }
    return b;
}

void oxo_gemm(const float* A, const float* B, float* C, size_t M, size_t N, size_t K,
              int a_trans, int b_trans, int rounding, float alpha, float beta) {
    float* a = prep_a(A, M, K, a_trans, rounding);
    float* b = prep_b(B, N, K, b_trans, rounding);
    gemm_panel(a, b, C, N, K, alpha, beta, 0, M);
    free(a);
    free(b);
}

typedef struct {
    const float *A, *B;
    float* C;
    size_t N, K;
    float alpha, beta;
    size_t r0, r1;
} gemm_job;

static void* gemm_worker(void* p) {
    gemm_job* j = (gemm_job*)p;
    gemm_panel(j->A, j->B, j->C, j->N, j->K, j->alpha, j->beta, j->r0, j->r1);
    return NULL;
}

void oxo_gemm_mt(const float* A, const float* B, float* C, size_t M, size_t N, size_t K,
                 int a_trans, int b_trans, int rounding, float alpha, float beta) {
    int t = oxo_get_threads();
    if (t <= 1 || M < 2 * RB) {
        oxo_gemm(A, B, C, M, N, K, a_trans, b_trans, rounding, alpha, beta);
        return;
    }
    float* a = prep_a(A, M, K, a_trans, rounding);
    float* b = prep_b(B, N, K, b_trans, rounding);
    size_t blocks = (M + RB - 1) / RB;
    if ((size_t)t > blocks) t = (int)blocks;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)t);
    gemm_job* jobs = (gemm_job*)malloc(sizeof(gemm_job) * (size_t)t);
    size_t per = (blocks + (size_t)t - 1) / (size_t)t * RB;
    int launched = 0;
    for (int i = 0; i < t; ++i) {
        size_t r0 = (size_t)i * per, r1 = r0 + per;
        if (r0 >= M) break;
        if (r1 > M) r1 = M;
        jobs[i] = (gemm_job){a, b, C, N, K, alpha, beta, r0, r1};
        pthread_create(&th[i], NULL, gemm_worker, &jobs[i]);
        ++launched;
    }
    for (int i = 0; i < launched; ++i) pthread_join(th[i], NULL);
    free(th);
    free(jobs);
    free(a);
    free(b);
}

void oxo_gemm_f64(const float* A, const float* B, double* C, size_t M, size_t N, size_t K,
                  int a_trans, int b_trans) {
    for (size_t m = 0; m < M; ++m)
        for (size_t n = 0; n < N; ++n) {
            double s = 0.0;
            for (size_t k = 0; k < K; ++k)
                s += (double)a_at(A, M, K, a_trans, m, k) * (double)b_at(B, N, K, b_trans, k, n);
            C[m * N + n] = s;
        }
}

/* ------------------------------------------------------------------------ */
/* elementwise                                                               */

/* apply_binary, elementwise.rs:5-13. */
float oxo_apply_binary(float lhs, float rhs, int op) {
    switch (op) {
        case OXO_ADD: return lhs + rhs;
        case OXO_SUB: return lhs - rhs;
        case OXO_MUL: return lhs * rhs;
        default: return lhs / rhs;
    }
}

/* slice_binary_device, elementwise.rs:45-56. */
void oxo_binary(const float* lhs, const float* rhs, float* out, size_t n, int op) {
    for (size_t i = 0; i < n; ++i) out[i] = oxo_apply_binary(lhs[i], rhs[i], op);
}

/* slice_binary_assign_device, elementwise.rs:58-68. */
void oxo_binary_assign(float* target, const float* rhs, size_t n, int op) {
    for (size_t i = 0; i < n; ++i) target[i] = oxo_apply_binary(target[i], rhs[i], op);
}

/* matrix_binary_assign_by_rows_device, row.rs:179-191. */
void oxo_binary_assign_by_rows(float* m, const float* row, size_t rows, size_t cols, int op) {
    for (size_t i = 0; i < rows * cols; ++i) m[i] = oxo_apply_binary(m[i], row[i % cols], op);
}

/* Activation constants and formulas, linear.rs:21-70. */
#define GELU_SCALE 0.7978846f
#define GELU_CUBIC 0.044715f

float oxo_act_forward(int act, float x) {
    switch (act) {
        case OXO_GELU: {
            float inner = GELU_SCALE * (x + GELU_CUBIC * x * x * x);
            return 0.5f * x * (1.0f + tanhf(inner));
        }
        case OXO_RELU: return x > 0.0f ? x : 0.0f;
        case OXO_SILU: return x / (1.0f + expf(-x));
        default: return x;
    }
}

float oxo_act_derivative(int act, float x) {
    switch (act) {
        case OXO_GELU: {
            const float quad = GELU_SCALE * 3.0f * GELU_CUBIC; /* linear.rs:24 */
            float inner = GELU_SCALE * (x + GELU_CUBIC * x * x * x);
            float th = tanhf(inner);
            float dinner = GELU_SCALE + quad * x * x;
            return 0.5f * (1.0f + th) + 0.5f * x * (1.0f - th * th) * dinner;
        }
        case OXO_RELU: return x > 0.0f ? 1.0f : 0.0f;
        case OXO_SILU: {
            float e = expf(-x);
            return 1.0f / (1.0f + e) + x * e / ((1.0f + e) * (1.0f + e));
        }
        default: return 1.0f;
    }
}

void oxo_activate(float* x, size_t n, int act) {
    if (act == OXO_IDENTITY) return;
    for (size_t i = 0; i < n; ++i) x[i] = oxo_act_forward(act, x[i]);
}

/* ------------------------------------------------------------------------ */
/* row kernels                                                               */

/* slice_set_device, slice_set_seq_device, slice_set_random_device
 * (elementwise.rs:15-43) with the hash of common.rs:3-9 (wrapping u32). */
void oxo_fill(float* out, size_t n, float value) {
    for (size_t i = 0; i < n; ++i) out[i] = value;
}

void oxo_fill_seq(float* out, size_t n, int dir) {
    for (size_t i = 0; i < n; ++i) out[i] = dir ? (float)i : (float)(n - i);
}

static uint32_t ref_hash(uint32_t x) {
    x += x << 13;
    x -= x >> 17;
    x *= x << 5;
    return x;
}

void oxo_fill_random(float* out, size_t n, uint32_t seed) {
    const float denom = (float)UINT32_MAX;  /* u32::MAX as f32 = 2^32 */
    for (size_t i = 0; i < n; ++i) out[i] = (float)ref_hash(seed + (uint32_t)i) / denom;
}

float oxo_unary(int op, float x, float p) {
    switch (op) {
        case 0: return x * p;
        case 1: return x + p;
        case 2: return oxo_act_forward((int)p, x);
        case 3: return oxo_act_derivative((int)p, x);
        default: return 0.5f * x * x;
    }
}

/* slice_map_sum_device, reduction.rs:44-80 (a shuffle tree per block; the
 * pairwise sum restates the tree's order of magnitude of rounding). */
float oxo_map_sum(const float* x, size_t n, int op, float p) {
    if (n == 0) return 0.0f;
    float* t = (float*)malloc(n * sizeof(float));
    if (!t) return 0.0f;
    for (size_t i = 0; i < n; ++i) t[i] = oxo_unary(op, x[i], p);
    const float s = psum(t, n);
    free(t);
    return s;
}

/* Vector::dot, vector.rs:109-115 (vector_mul, then sum). */
float oxo_dot(const float* x, const float* y, size_t n) {
    if (n == 0) return 0.0f;
    float* t = (float*)malloc(n * sizeof(float));
    if (!t) return 0.0f;
    for (size_t i = 0; i < n; ++i) t[i] = x[i] * y[i];
    const float s = psum(t, n);
    free(t);
    return s;
}

/* Data-parallel update across ranks; contract in oxf_oracle.h. */
void oxo_exchange_sgd(float* const* params, const float* const* grads, int world, size_t offset,
                      size_t count, float lr) {
    for (size_t i = offset; i < offset + count; ++i) {
        float s = grads[0][i];
        for (int q = 1; q < world; ++q) s += grads[q][i];
        const float r = fmaf(-s, lr, params[0][i]);
        for (int q = 0; q < world; ++q) params[q][i] = r;
    }
}

/* matrix_slice_device, layout.rs:58-86. */
void oxo_matrix_slice(const float* in, float* out, size_t out_len, size_t input_cols,
                      size_t tile_rows, size_t tile_cols, size_t tiles_per_row) {
    const size_t tile = tile_rows * tile_cols;
    for (size_t l = 0; l < out_len; ++l) {
        const size_t ti = l / tile, local = l % tile;
        const size_t ty = ti / tiles_per_row, tx = ti % tiles_per_row;
        const size_t r = ty * tile_rows + local / tile_cols;
        const size_t c = tx * tile_cols + local % tile_cols;
        out[l] = in[r * input_cols + c];
    }
}

/* matrix_sum_rows_device, row.rs:16-53. */
void oxo_sum_rows(const float* m, float* out, size_t rows, size_t cols) {
    for (size_t r = 0; r < rows; ++r) out[r] = psum(m + r * cols, cols);
}

/* linear.rs:267-270 computes the bias gradient as sum_rows(transpose(G)). */
void oxo_sum_cols(const float* m, float* out, size_t rows, size_t cols) {
    for (size_t c = 0; c < cols; ++c) out[c] = 0.0f;
    for (size_t r = 0; r < rows; ++r)
        for (size_t c = 0; c < cols; ++c) out[c] += m[r * cols + c];
}

/* matrix_transpose_device, layout.rs:9-55. */
void oxo_transpose(const float* in, float* out, size_t rows, size_t cols) {
    for (size_t r = 0; r < rows; ++r)
        for (size_t c = 0; c < cols; ++c) out[c * rows + r] = in[r * cols + c];
}

/* matrix_causal_mask_device, row.rs:5-14. */
void oxo_causal_mask(float* m, size_t rows, size_t cols, size_t period) {
    if (period == 0) period = rows;
    for (size_t r = 0; r < rows; ++r) {
        size_t i = r % period;
        for (size_t c = i + 1; c < cols; ++c) m[r * cols + c] = -INFINITY;
    }
}

/* matrix_softmax_rows_device, row.rs:55-113: row max (inactive lanes pad
 * with f32::MIN, row.rs:64), exp(x - max), row sum, exp/sum. */
void oxo_softmax_rows(float* m, size_t rows, size_t cols, float scale, size_t causal_period) {
    for (size_t r = 0; r < rows; ++r) {
        float* x = m + r * cols;
        if (scale != 1.0f)
            for (size_t c = 0; c < cols; ++c) x[c] *= scale;
        if (causal_period) {
            size_t i = r % causal_period;
            for (size_t c = i + 1; c < cols; ++c) x[c] = -INFINITY;
        }
        float mx = -3.40282347e+38f; /* f32::MIN */
        for (size_t c = 0; c < cols; ++c) mx = x[c] > mx ? x[c] : mx;
        for (size_t c = 0; c < cols; ++c) x[c] = expf(x[c] - mx);
        float s = psum(x, cols);
        for (size_t c = 0; c < cols; ++c) x[c] = x[c] / s;
    }
}

/* matrix_layer_norm_rows_device, row.rs:115-177: mean, biased variance of
 * (x - mean), inv_std = 1/sqrt(var + eps), y = (x - mean) * inv_std. */
void oxo_layer_norm_rows(float* m, size_t rows, size_t cols, float eps, const float* gamma,
                         const float* beta) {
    for (size_t r = 0; r < rows; ++r) {
        float* x = m + r * cols;
        float* t = tmpbuf(cols);
        float mean = psum(x, cols) / (float)cols;
        for (size_t c = 0; c < cols; ++c) t[c] = (x[c] - mean) * (x[c] - mean);
        float v = psum(t, cols);
        float inv_std = 1.0f / sqrtf(v / (float)cols + eps);
        for (size_t c = 0; c < cols; ++c) {
            float y = (x[c] - mean) * inv_std;
            if (gamma) y *= gamma[c];
            if (beta) y += beta[c];
            x[c] = y;
        }
    }
}

/* rms_norm_assign_device, row.rs:349-396: y = x / sqrt(mean(x^2) + eps). */
void oxo_rms_norm_rows(float* m, size_t rows, size_t cols, float eps, const float* gamma) {
    for (size_t r = 0; r < rows; ++r) {
        float* x = m + r * cols;
        float* t = tmpbuf(cols);
        for (size_t c = 0; c < cols; ++c) t[c] = x[c] * x[c];
        float rms = sqrtf(psum(t, cols) / (float)cols + eps);
        for (size_t c = 0; c < cols; ++c) {
            float y = x[c] / rms;
            if (gamma) y *= gamma[c];
            x[c] = y;
        }
    }
}

/* softmax_rows_backward_device, row.rs:193-237. */
void oxo_softmax_backward(const float* p, const float* dy, float* dx, size_t rows, size_t cols,
                          float scale) {
    for (size_t r = 0; r < rows; ++r) {
        const float* pr = p + r * cols;
        const float* gr = dy + r * cols;
        float* t = tmpbuf(cols);
        for (size_t c = 0; c < cols; ++c) t[c] = pr[c] * gr[c];
        float s = psum(t, cols);
        for (size_t c = 0; c < cols; ++c) dx[r * cols + c] = pr[c] * (gr[c] - s) * scale;
    }
}

/* layer_norm_backward_device, row.rs:239-347:
 * dx = inv_std/N * (N*dy - sum(dy) - xhat*sum(dy*xhat)). */
void oxo_layer_norm_backward(const float* x, const float* dy, float* dx, size_t rows, size_t cols,
                             float eps) {
    const float n = (float)cols;
    for (size_t r = 0; r < rows; ++r) {
        const float* xr = x + r * cols;
        const float* gr = dy + r * cols;
        float* t = tmpbuf(cols);
        float mean = psum(xr, cols) / n;
        for (size_t c = 0; c < cols; ++c) t[c] = (xr[c] - mean) * (xr[c] - mean);
        float inv_std = 1.0f / sqrtf(psum(t, cols) / n + eps);
        float gs = psum(gr, cols);
        for (size_t c = 0; c < cols; ++c) t[c] = gr[c] * ((xr[c] - mean) * inv_std);
        float gns = psum(t, cols);
        for (size_t c = 0; c < cols; ++c) {
            float xh = (xr[c] - mean) * inv_std;
            dx[r * cols + c] = inv_std / n * (n * gr[c] - gs - xh * gns);
        }
    }
}

/* rms_norm_backward_device, row.rs:398-468: dx = dy/r - x*(sum(x*dy)/N)/r^3. */
void oxo_rms_norm_backward(const float* x, const float* dy, float* dx, size_t rows, size_t cols,
                           float eps) {
    const float n = (float)cols;
    for (size_t r = 0; r < rows; ++r) {
        const float* xr = x + r * cols;
        const float* gr = dy + r * cols;
        float* t = tmpbuf(cols);
        for (size_t c = 0; c < cols; ++c) t[c] = xr[c] * xr[c];
        float ss = psum(t, cols);
        for (size_t c = 0; c < cols; ++c) t[c] = xr[c] * gr[c];
        float dot = psum(t, cols);
        float rms = sqrtf(ss / n + eps);
        float inv = 1.0f / rms;
        float corr = dot / n * inv * inv * inv;
        for (size_t c = 0; c < cols; ++c) dx[r * cols + c] = gr[c] * inv - xr[c] * corr;
    }
}

/* Linear::loss_rows_default, linear.rs:325-333. */
void oxo_loss_rows(const float* y, const float* t, float* row_loss, size_t rows, size_t cols) {
    float* buf = tmpbuf(cols);
    for (size_t r = 0; r < rows; ++r) {
        for (size_t c = 0; c < cols; ++c) {
            float d = y[r * cols + c] - t[r * cols + c];
            buf[c] = 0.5f * d * d;
        }
        row_loss[r] = psum(buf, cols) * (1.0f / (float)cols);
    }
}

void oxo_mse_grad(const float* y, const float* t, float* g, size_t rows, size_t cols) {
    const float inv = 1.0f / (float)cols;
    for (size_t i = 0; i < rows * cols; ++i) g[i] = (y[i] - t[i]) * inv;
}

/* ------------------------------------------------------------------------ */
/* executors                                                                 */

static float* fdup(const float* x, size_t n) {
    float* y = (float*)malloc((n ? n : 1) * sizeof(float));
    memcpy(y, x, n * sizeof(float));
    return y;
}
static float* falloc(size_t n) { return (float*)calloc(n ? n : 1, sizeof(float)); }

/* Linear::affine_on, linear.rs:185-206: GEMM, then bias by rows, then
 * residual; Linear::activate_on, linear.rs:225-230. */
void oxo_linear_forward(const oxo_linear* l, const float* x, const float* residual, float* y,
                        float* pre, size_t rows, int rounding) {
    oxo_gemm_mt(x, l->w, y, rows, l->out, l->in, 0, 0, rounding, 1.0f, 0.0f);
    if (l->b) oxo_binary_assign_by_rows(y, l->b, rows, l->out, OXO_ADD);
    if (residual) oxo_binary_assign(y, residual, rows * l->out, OXO_ADD);
    if (pre) memcpy(pre, y, rows * l->out * sizeof(float));
    oxo_activate(y, rows * l->out, l->act);
}

/* Linear::backward_default (linear.rs:246-275) + input_gradient
 * (linear.rs:431-434) + learn (linear.rs:373-391). `pre` is the layer's
 * pre-activation (the reference recomputes it, mlp.rs:136-139). The
 * activation-scaled gradient is returned in g_out ([rows,out], caller
 * owned), dX in dx. Parameter gradients go to gw/gb (may be NULL); the SGD
 * update W -= lr * XᵀG runs when lr != 0, after dX used the old W. */
static void linear_backward(oxo_linear* l, const float* x, const float* pre, const float* dy,
                            float* g_out, float* dx, size_t rows, float lr, float* gw, float* gb,
                            int rounding) {
    const size_t n = rows * l->out;
    memcpy(g_out, dy, n * sizeof(float));
    if (l->act != OXO_IDENTITY)
        for (size_t i = 0; i < n; ++i) g_out[i] *= oxo_act_derivative(l->act, pre[i]);
    float* db = NULL;
    if (l->b) {
        db = falloc(l->out);
        oxo_sum_cols(g_out, db, rows, l->out);
    }
    if (dx) oxo_gemm_mt(g_out, l->w, dx, rows, l->in, l->out, 0, 1, rounding, 1.0f, 0.0f);
    float* dw = falloc(l->in * l->out);
    oxo_gemm_mt(x, g_out, dw, l->in, l->out, rows, 1, 0, rounding, 1.0f, 0.0f);
    if (gw)
        for (size_t i = 0; i < l->in * l->out; ++i) gw[i] += dw[i];
    if (gb && db)
        for (size_t i = 0; i < l->out; ++i) gb[i] += db[i];
    if (lr != 0.0f) {
        /* weight_gradient.scale(lr); weights -= weight_gradient */
        for (size_t i = 0; i < l->in * l->out; ++i) l->w[i] -= dw[i] * lr;
        if (l->b)
            for (size_t i = 0; i < l->out; ++i) l->b[i] -= db[i] * lr;
    }
    free(dw);
    free(db);
}

/* MlpExecutor::forward / TrainingMlp::forward, mlp.rs:53-85, 233-254. */
void oxo_mlp_forward(const oxo_mlp* m, const float* x, float* y, float** tape, size_t rows,
                     int rounding) {
    float** ins = (float**)calloc(m->n_layers + 1, sizeof(float*));
    ins[0] = fdup(x, rows * m->layers[0].in);
    for (size_t i = 0; i < m->n_layers; ++i) {
        const oxo_linear* l = &m->layers[i];
        const float* res = NULL;
        if (m->res_end >= 0 && (int)i + 1 == m->res_end) res = ins[m->res_start];
        ins[i + 1] = falloc(rows * l->out);
        oxo_linear_forward(l, ins[i], res, ins[i + 1], NULL, rows, rounding);
    }
    memcpy(y, ins[m->n_layers], rows * m->layers[m->n_layers - 1].out * sizeof(float));
    if (tape)
        for (size_t i = 0; i < m->n_layers; ++i)
            memcpy(tape[i], ins[i], rows * m->layers[i].in * sizeof(float));
    for (size_t i = 0; i <= m->n_layers; ++i) free(ins[i]);
    free(ins);
}

/* MlpExecutor::backward, mlp.rs:121-168. gws/gbs (may be NULL) receive
 * per-layer parameter gradients (added). */
static void mlp_backward_impl(oxo_mlp* m, float* const* tape, const float* dy, float* dx,
                              size_t rows, float lr, float** gws, float** gbs, int rounding) {
    size_t L = m->n_layers;
    float* grad = fdup(dy, rows * m->layers[L - 1].out);
    float* skip = NULL;
    int skip_src = -1;
    for (size_t ii = L; ii-- > 0;) {
        oxo_linear* l = &m->layers[ii];
        int res_idx = (m->res_end >= 0 && (int)ii + 1 == m->res_end) ? m->res_start : -1;
        float* pre = NULL;
        if (l->act != OXO_IDENTITY) {
            /* recompute the affine output (mlp.rs:136-139) */
            oxo_linear tmp = *l;
            tmp.act = OXO_IDENTITY;
            pre = falloc(rows * l->out);
            oxo_linear_forward(&tmp, tape[ii], res_idx >= 0 ? tape[res_idx] : NULL, pre, NULL, rows,
                               rounding);
        }
        float* g = falloc(rows * l->out);
        float* din = falloc(rows * l->in);
        linear_backward(l, tape[ii], pre, grad, g, din, rows, lr, gws ? gws[ii] : NULL,
                        gbs ? gbs[ii] : NULL, rounding);
        if (res_idx >= 0) {
            skip = fdup(g, rows * l->out);
            skip_src = res_idx;
        }
        if (skip && skip_src == (int)ii) {
            oxo_binary_assign(din, skip, rows * l->in, OXO_ADD);
            free(skip);
            skip = NULL;
            skip_src = -1;
        }
        free(pre);
        free(g);
        free(grad);
        grad = din;
    }
    memcpy(dx, grad, rows * m->layers[0].in * sizeof(float));
    free(grad);
    free(skip);
}

void oxo_mlp_backward(oxo_mlp* m, float* const* tape, const float* dy, float* dx, size_t rows,
                      float lr, int rounding) {
    mlp_backward_impl(m, tape, dy, dx, rows, lr, NULL, NULL, rounding);
}

static void norm_forward(int norm, float* x, size_t rows, size_t cols) {
    if (norm == OXO_NORM_LAYER)
        oxo_layer_norm_rows(x, rows, cols, 1e-5f, NULL, NULL);
    else
        oxo_rms_norm_rows(x, rows, cols, 1e-5f, NULL);
}

static void norm_backward(int norm, const float* x, const float* dy, float* dx, size_t rows,
                          size_t cols) {
    if (norm == OXO_NORM_LAYER)
        oxo_layer_norm_backward(x, dy, dx, rows, cols, 1e-5f);
    else
        oxo_rms_norm_backward(x, dy, dx, rows, cols, 1e-5f);
}

/* Columns [c0, c0 + w) of a row-major [rows, ld] matrix, as a contiguous
 * [rows, w] copy, and the reverse. */
static float* gather_cols(const float* m, size_t rows, size_t ld, size_t c0, size_t w) {
    float* out = falloc(rows * w);
    for (size_t r = 0; r < rows; ++r) memcpy(out + r * w, m + r * ld + c0, w * sizeof(float));
    return out;
}

static void scatter_cols(const float* src, float* m, size_t rows, size_t ld, size_t c0, size_t w) {
    for (size_t r = 0; r < rows; ++r) memcpy(m + r * ld + c0, src + r * w, w * sizeof(float));
}

/* Attention core with `heads` heads. The reference is single-head
 * (attention.rs:359-401: scores = Q·Kᵀ scaled by 1/sqrt(query.cols),
 * softmax rows, P·V) and anticipates a multi-head path that keeps the
 * projections and changes only "the projected-matrix head layout and
 * per-head score calculation" (docs/api.md:440-442). Head j takes columns
 * [j·D/h, (j+1)·D/h) of Q and K and [j·Hv/h, (j+1)·Hv/h) of V, scales its
 * scores by 1/sqrt(D/h), and writes its output into the same columns of
 * `att` [S, Hv]; heads = 1 is the reference's attention. p_keep (may be
 * NULL): [heads, S, S] probabilities, kept for backward. */
void oxo_attention_forward_heads(const float* q, const float* k, const float* v, float* p_keep,
                                 float* att, size_t S, size_t D, size_t Hv, size_t heads,
                                 int causal, int rounding) {
    const size_t dq = D / heads, dv = Hv / heads;
    const float scale = 1.0f / sqrtf((float)dq);
    for (size_t j = 0; j < heads; ++j) {
        float* qj = gather_cols(q, S, D, j * dq, dq);
        float* kj = gather_cols(k, S, D, j * dq, dq);
        float* vj = gather_cols(v, S, Hv, j * dv, dv);
        float* sc = p_keep ? p_keep + j * S * S : falloc(S * S);
        /* scores, then the scale (attention.rs:366-372, 398) */
        oxo_gemm_mt(qj, kj, sc, S, S, dq, 0, 1, rounding, 1.0f, 0.0f);
        for (size_t i = 0; i < S * S; ++i) sc[i] *= scale;
        if (causal) oxo_causal_mask(sc, S, S, S);
        oxo_softmax_rows(sc, S, S, 1.0f, 0);
        float* aj = falloc(S * dv);
        oxo_gemm_mt(sc, vj, aj, S, dv, S, 0, 0, rounding, 1.0f, 0.0f);
        scatter_cols(aj, att, S, Hv, j * dv, dv);
        free(qj); free(kj); free(vj); free(aj);
        if (!p_keep) free(sc);
    }
}

/* Backward of the core (Attention::backward_self, attention.rs:297-308),
 * head by head: dP = dR·Vᵀ, dV = Pᵀ·dR, dS = softmax'(P, dP)·scale,
 * dQ = dS·K, dK = dSᵀ·Q, each in its head's columns. dr: [S, Hv]. */
void oxo_attention_backward_heads(const float* q, const float* k, const float* v,
                                  const float* p, const float* dr, float* dq, float* dk,
                                  float* dv, size_t S, size_t D, size_t Hv, size_t heads,
                                  int rounding) {
    const size_t hq = D / heads, hv = Hv / heads;
    const float scale = 1.0f / sqrtf((float)hq);
    for (size_t j = 0; j < heads; ++j) {
        float* qj = gather_cols(q, S, D, j * hq, hq);
        float* kj = gather_cols(k, S, D, j * hq, hq);
        float* vj = gather_cols(v, S, Hv, j * hv, hv);
        float* drj = gather_cols(dr, S, Hv, j * hv, hv);
        const float* pj = p + j * S * S;
        float* dp = falloc(S * S);
        oxo_gemm_mt(drj, vj, dp, S, S, hv, 0, 1, rounding, 1.0f, 0.0f);  /* dR·Vᵀ */
        float* dvj = falloc(S * hv);
        oxo_gemm_mt(pj, drj, dvj, S, hv, S, 1, 0, rounding, 1.0f, 0.0f); /* Pᵀ·dR */
        float* ds = falloc(S * S);
        oxo_softmax_backward(pj, dp, ds, S, S, 1.0f);
        for (size_t i = 0; i < S * S; ++i) ds[i] *= scale; /* attention.rs:304 */
        float* dqj = falloc(S * hq);
        oxo_gemm_mt(ds, kj, dqj, S, hq, S, 0, 0, rounding, 1.0f, 0.0f);  /* dS·K */
        float* dkj = falloc(S * hq);
        oxo_gemm_mt(ds, qj, dkj, S, hq, S, 1, 0, rounding, 1.0f, 0.0f);  /* dSᵀ·Q */
        scatter_cols(dqj, dq, S, D, j * hq, hq);
        scatter_cols(dkj, dk, S, D, j * hq, hq);
        scatter_cols(dvj, dv, S, Hv, j * hv, hv);
        free(qj); free(kj); free(vj); free(drj); free(dp); free(dvj); free(ds); free(dqj);
        free(dkj);
    }
}

/* InferenceBlock::forward / forward_mask (inference.rs:76-109) with
 * Attention::forward (attention.rs:221-253, 336-387). */
void oxo_transformer_forward_heads(const oxo_transformer* t, const float* x, float* y,
                                   int causal, int rounding, int heads) {
    const size_t S = t->seq, H = t->hidden;
    float* pos = falloc(S * H);
    oxo_binary(x, t->position, pos, S * H, OXO_ADD);
    float* q = falloc(S * t->q.out);
    float* k = falloc(S * t->k.out);
    float* v = falloc(S * t->v.out);
    oxo_linear_forward(&t->q, pos, NULL, q, NULL, S, rounding);
    oxo_linear_forward(&t->k, pos, NULL, k, NULL, S, rounding);
    oxo_linear_forward(&t->v, pos, NULL, v, NULL, S, rounding);
    const size_t D = t->q.out;
    /* softmax(Q·Kᵀ / sqrt(query.cols))·V per head (attention.rs:359-401) */
    float* att = falloc(S * t->v.out);
    oxo_attention_forward_heads(q, k, v, NULL, att, S, D, t->v.out, (size_t)heads, causal,
                                rounding);
    float* h1 = falloc(S * H);
    oxo_binary(pos, att, h1, S * H, OXO_ADD); /* attention.rs:249 */
    norm_forward(t->norm, h1, S, H);
    size_t F = t->ffn.layers[t->ffn.n_layers - 1].out;
    float* ffn = falloc(S * F);
    oxo_mlp_forward(&t->ffn, h1, ffn, NULL, S, rounding);
    float* h2 = falloc(S * H);
    oxo_binary(h1, ffn, h2, S * H, OXO_ADD); /* inference.rs:99 */
    norm_forward(t->norm, h2, S, H);
    oxo_linear_forward(&t->o, h2, NULL, y, NULL, S, rounding);
    free(pos); free(q); free(k); free(v); free(att); free(h1); free(ffn); free(h2);
}

void oxo_transformer_forward(const oxo_transformer* t, const float* x, float* y, int causal,
                             int rounding) {
    oxo_transformer_forward_heads(t, x, y, causal, rounding, 1);
}

size_t oxo_transformer_param_count(const oxo_transformer* t) {
    size_t n = 0;
    const oxo_linear* qkv[3] = {&t->q, &t->k, &t->v};
    for (int i = 0; i < 3; ++i) n += qkv[i]->in * qkv[i]->out + (qkv[i]->b ? qkv[i]->out : 0);
    n += t->seq * t->hidden;
    for (size_t i = 0; i < t->ffn.n_layers; ++i)
        n += t->ffn.layers[i].in * t->ffn.layers[i].out +
             (t->ffn.layers[i].b ? t->ffn.layers[i].out : 0);
    n += t->o.in * t->o.out + (t->o.b ? t->o.out : 0);
    return n;
}

/* TrainingTransformer::forward + backward, encoder.rs:114-186, with
 * Attention::forward_self_training / backward_self (attention.rs:258-321)
 * and QkvProjection::backward_self (attention.rs:104-144). */
void oxo_transformer_train_step_heads(oxo_transformer* t, const float* x, const float* target,
                                      float* y, float* row_loss, float* dx, float lr,
                                      float* grads, int rounding, int heads) {
    const size_t S = t->seq, H = t->hidden, D = t->q.out, O = t->o.out;
    const size_t nh = (size_t)heads;
    /* gradient slots in cursor order */
    float *g_q = NULL, *g_qb = NULL, *g_k = NULL, *g_kb = NULL, *g_v = NULL, *g_vb = NULL;
    float *g_pos = NULL, *g_o = NULL, *g_ob = NULL;
    float** g_fw = (float**)calloc(t->ffn.n_layers, sizeof(float*));
    float** g_fb = (float**)calloc(t->ffn.n_layers, sizeof(float*));
    if (grads) {
        float* p = grads;
        g_q = p; p += t->q.in * t->q.out; if (t->q.b) { g_qb = p; p += t->q.out; }
        g_k = p; p += t->k.in * t->k.out; if (t->k.b) { g_kb = p; p += t->k.out; }
        g_v = p; p += t->v.in * t->v.out; if (t->v.b) { g_vb = p; p += t->v.out; }
        g_pos = p; p += S * H;
        for (size_t i = 0; i < t->ffn.n_layers; ++i) {
            g_fw[i] = p; p += t->ffn.layers[i].in * t->ffn.layers[i].out;
            if (t->ffn.layers[i].b) { g_fb[i] = p; p += t->ffn.layers[i].out; }
        }
        g_o = p; p += t->o.in * t->o.out; if (t->o.b) { g_ob = p; p += t->o.out; }
    }

    /* ---- forward ---- */
    float* pos = falloc(S * H);
    oxo_binary(x, t->position, pos, S * H, OXO_ADD);
    float* q = falloc(S * D);
    float* k = falloc(S * t->k.out);
    float* v = falloc(S * t->v.out);
    float* q_pre = falloc(S * D);
    float* k_pre = falloc(S * t->k.out);
    float* v_pre = falloc(S * t->v.out);
    oxo_linear_forward(&t->q, pos, NULL, q, q_pre, S, rounding);
    oxo_linear_forward(&t->k, pos, NULL, k, k_pre, S, rounding);
    oxo_linear_forward(&t->v, pos, NULL, v, v_pre, S, rounding);
    float* p = falloc(nh * S * S); /* kept for backward (attention.rs:183-190) */
    float* att = falloc(S * t->v.out);
    oxo_attention_forward_heads(q, k, v, p, att, S, D, t->v.out, nh, 0, rounding);
    float* pre_norm = falloc(S * H);
    oxo_binary(pos, att, pre_norm, S * H, OXO_ADD);
    float* h1 = fdup(pre_norm, S * H);
    norm_forward(t->norm, h1, S, H);
    /* TrainingMlp::forward keeps layer inputs */
    size_t L = t->ffn.n_layers;
    float** tape = (float**)calloc(L, sizeof(float*));
    for (size_t i = 0; i < L; ++i) tape[i] = falloc(S * t->ffn.layers[i].in);
    size_t F = t->ffn.layers[L - 1].out;
    float* ffn = falloc(S * F);
    oxo_mlp_forward(&t->ffn, h1, ffn, tape, S, rounding);
    float* pre2 = falloc(S * H);
    oxo_binary(h1, ffn, pre2, S * H, OXO_ADD); /* encoder.rs:120-123 */
    float* enc = fdup(pre2, S * H);
    norm_forward(t->norm, enc, S, H);
    float* o_pre = falloc(S * O);
    oxo_linear_forward(&t->o, enc, NULL, y, o_pre, S, rounding);
    if (row_loss) oxo_loss_rows(y, target, row_loss, S, O);

    /* ---- backward ---- */
    float* dy = falloc(S * O);
    oxo_mse_grad(y, target, dy, S, O);
    float* g_out = falloc(S * O);
    float* d_enc = falloc(S * H);
    linear_backward(&t->o, enc, o_pre, dy, g_out, d_enc, S, lr, g_o, g_ob, rounding);
    float* d2 = falloc(S * H);
    norm_backward(t->norm, pre2, d_enc, d2, S, H);
    float* d_ffn_in = falloc(S * H);
    mlp_backward_impl(&t->ffn, tape, d2, d_ffn_in, S, lr, grads ? g_fw : NULL,
                      grads ? g_fb : NULL, rounding);
    float* d1 = fdup(d2, S * H);
    oxo_binary_assign(d1, d_ffn_in, S * H, OXO_ADD); /* encoder.rs:144-146 */
    /* Attention::backward_self */
    float* dr = falloc(S * H);
    norm_backward(t->norm, pre_norm, d1, dr, S, H);
    float* dq = falloc(S * D);
    float* dk = falloc(S * t->k.out);
    float* dv = falloc(S * t->v.out);
    oxo_attention_backward_heads(q, k, v, p, dr, dq, dk, dv, S, D, t->v.out, nh, rounding);
    float* dpos = fdup(dr, S * H);
    {
        oxo_linear* ls[3] = {&t->q, &t->k, &t->v};
        const float* dps[3] = {dq, dk, dv};
        const float* pres[3] = {q_pre, k_pre, v_pre};
        float* gws[3] = {g_q, g_k, g_v};
        float* gbs[3] = {g_qb, g_kb, g_vb};
        float* din = falloc(S * H);
        for (int j = 0; j < 3; ++j) {
            float* g = falloc(S * ls[j]->out);
            linear_backward(ls[j], pos, pres[j], dps[j], g, din, S, lr, gws[j], gbs[j], rounding);
            oxo_binary_assign(dpos, din, S * H, OXO_ADD); /* attention.rs:127-131, 318-319 */
            free(g);
        }
        free(din);
    }
    if (dx) memcpy(dx, dpos, S * H * sizeof(float));
    if (g_pos)
        for (size_t i = 0; i < S * H; ++i) g_pos[i] += dpos[i];
    if (lr != 0.0f)
        for (size_t i = 0; i < S * H; ++i) t->position[i] -= dpos[i] * lr; /* encoder.rs:180-184 */

    for (size_t i = 0; i < L; ++i) free(tape[i]);
    free(tape); free(g_fw); free(g_fb);
    free(pos); free(q); free(k); free(v); free(q_pre); free(k_pre); free(v_pre); free(p);
    free(att); free(pre_norm); free(h1); free(ffn); free(pre2); free(enc); free(o_pre); free(dy);
    free(g_out); free(d_enc); free(d2); free(d_ffn_in); free(d1); free(dr); free(dv);
    free(dq); free(dk); free(dpos);
}

void oxo_transformer_train_step(oxo_transformer* t, const float* x, const float* target,
                                float* y, float* row_loss, float* dx, float lr, float* grads,
                                int rounding) {
    oxo_transformer_train_step_heads(t, x, target, y, row_loss, dx, lr, grads, rounding, 1);
}
