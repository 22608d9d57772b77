/*
 * oxf_oracle.h — CPU oracle for the OxideForge compute hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is a scalar C restatement of the reference
 * algorithms (MeccBai/oxide-forge, Rust + cuda-oxide). Only tests/, the
 * smoke() check in __graft_entry__.py and bench.py's CPU-baseline / reference
 * arm may load it, and only as the checker or the timed CPU baseline. The
 * product path (liboxf.so) never links or calls it.
 *
 * PARITY UNPINNED: the reference has no tests, golden vectors or fixtures,
 * and it cannot be built or run here (Rust/cuda-oxide toolchain absent). The
 * oracle is pinned instead by hand-derived known-answer cases and by golden
 * fixtures from an independent numpy f64 restatement (tests/golden/).
 *
 * Every function cites the reference file:line whose arithmetic it restates.
 * All matrices are contiguous row-major f32 (the reference's only layout,
 * docs/api.md "Conventions").
 */
#ifndef OXF_ORACLE_H
#define OXF_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* BinaryOp, src/cuda.rs:3-10 (repr(u8): Add, Sub, Mul, Div). */
enum { OXO_ADD = 0, OXO_SUB = 1, OXO_MUL = 2, OXO_DIV = 3 };
/* Activation, src/net/linear.rs:14-19. */
enum { OXO_IDENTITY = 0, OXO_GELU = 1, OXO_RELU = 2, OXO_SILU = 3 };
/* NormType, src/net/transformer.rs:7-13. */
enum { OXO_NORM_RMS = 0, OXO_NORM_LAYER = 1 };
/* GEMM operand rounding: exact f32 products, TF32 round-to-nearest-away
 * (cvt.rna.tf32.f32, gemm.rs:286-347), or TF32 truncation (tensor cores that
 * read raw f32 and drop the low 13 mantissa bits). */
enum { OXO_GEMM_F32 = 0, OXO_GEMM_TF32_RNA = 1, OXO_GEMM_TF32_RZ = 2 };

/* Number of worker threads used by the threaded entry points (0 = all
 * online cores). Returns the count now in effect. */
int oxo_set_threads(int n);
int oxo_get_threads(void);

float oxo_tf32_rna(float x);
float oxo_tf32_rz(float x);

/* C[M,N] = alpha * op(A)·op(B) (+ beta*C).  a_trans: A stored as [K,M]
 * (A = stored^T); b_trans: B stored as [N,K].  Row-major, f32 accumulation in
 * ascending k.  matrix_multiply_device, gemm.rs:202-373 (reference only has
 * the NN form; Xᵀ·G and G·Wᵀ go through matrix_transpose, convert.rs:17-63). */
void oxo_gemm(const float* A, const float* B, float* C, size_t M, size_t N, size_t K,
              int a_trans, int b_trans, int rounding, float alpha, float beta);
/* Same arithmetic, threaded over rows of C. */
void oxo_gemm_mt(const float* A, const float* B, float* C, size_t M, size_t N, size_t K,
                 int a_trans, int b_trans, int rounding, float alpha, float beta);
/* f64 reference product of f32 inputs (tolerance budgeting). */
void oxo_gemm_f64(const float* A, const float* B, double* C, size_t M, size_t N, size_t K,
                  int a_trans, int b_trans);

/* Elementwise, src/cuda/device/elementwise.rs:5-13,45-68. */
float oxo_apply_binary(float lhs, float rhs, int op);
void oxo_binary(const float* lhs, const float* rhs, float* out, size_t n, int op);
void oxo_binary_assign(float* target, const float* rhs, size_t n, int op);
/* row.rs:179-191: M[i,j] op= v[j]. */
void oxo_binary_assign_by_rows(float* m, const float* row, size_t rows, size_t cols, int op);

/* Activation::forward / derivative, linear.rs:21-70. */
float oxo_act_forward(int act, float x);
float oxo_act_derivative(int act, float x);
void oxo_activate(float* x, size_t n, int act);

/* Fills, elementwise.rs:15-43: slice_set, slice_set_seq (element i = i, or
 * len - i), slice_set_random (hash of seed + i, common.rs:3-9, scaled by
 * 1 / (float)UINT32_MAX). */
void oxo_fill(float* out, size_t n, float value);
void oxo_fill_seq(float* out, size_t n, int dir);
void oxo_fill_random(float* out, size_t n, uint32_t seed);
/* The closures the reference passes to slice_for_each / slice_map_sum, as
 * the enumerated oxf_unary_op set: 0 x*p, 1 x+p, 2 act(x) (p = activation),
 * 3 act'(x), 4 0.5*x*x. */
float oxo_unary(int op, float x, float p);
/* slice_map_sum, reduction.rs:44-80: sum of f(x_i) (pairwise). */
float oxo_map_sum(const float* x, size_t n, int op, float p);
/* Vector::dot, vector.rs:109-115: the elementwise product, then its sum
 * (pairwise, as oxo_map_sum). */
float oxo_dot(const float* x, const float* y, size_t n);
/* matrix_slice, layout.rs:58-86: output element l belongs to tile l / (tr*tc)
 * (tile row = tile / tiles_per_row, tile column = tile % tiles_per_row) at
 * local row (l % (tr*tc)) / tc, local column (l % (tr*tc)) % tc. */
void oxo_matrix_slice(const float* in, float* out, size_t out_len, size_t input_cols,
                      size_t tile_rows, size_t tile_cols, size_t tiles_per_row);

/* The data-parallel update over `world` ranks' arenas (the per-rank update
 * is Linear::learn's W -= lr * dW, linear.rs:373-391; the reference itself
 * is single-GPU): for i in [offset, offset + count),
 *   p_i = p_i - lr * (g0_i + g1_i + ... + g{world-1}_i)
 * with the gradients summed left to right in f32 and the update rounded
 * once (fmaf), then written to every rank's parameters. The source value
 * is params[0][i] (all ranks hold equal parameters before the step). */
void oxo_exchange_sgd(float* const* params, const float* const* grads, int world, size_t offset,
                      size_t count, float lr);

/* row.rs:16-53 (per-row sum). */
void oxo_sum_rows(const float* m, float* out, size_t rows, size_t cols);
/* Column sum = sum_rows(transpose(G)), linear.rs:267-270. */
void oxo_sum_cols(const float* m, float* out, size_t rows, size_t cols);
/* layout.rs:9-55. out[cols,rows] = in[rows,cols]^T. */
void oxo_transpose(const float* in, float* out, size_t rows, size_t cols);
/* row.rs:5-14: M[i,j] = -inf for j > i; rows counted modulo `period`
 * (period = rows gives the reference's single-matrix behaviour). */
void oxo_causal_mask(float* m, size_t rows, size_t cols, size_t period);

/* In-place row softmax, row.rs:55-113; `scale` multiplies the row first
 * (attention.rs:372 applies 1/sqrt(d) before softmax); causal_period != 0
 * masks j > (row % causal_period) first (attention.rs:347-357). */
void oxo_softmax_rows(float* m, size_t rows, size_t cols, float scale, size_t causal_period);
/* row.rs:115-177 (eps = 1e-5 at norm.rs:45). Optional gamma/beta (may be NULL). */
void oxo_layer_norm_rows(float* m, size_t rows, size_t cols, float eps, const float* gamma,
                         const float* beta);
/* row.rs:349-396. Optional gamma. */
void oxo_rms_norm_rows(float* m, size_t rows, size_t cols, float eps, const float* gamma);
/* row.rs:193-237: dx = p*(dy - sum(p*dy)); `scale` multiplies dx afterwards
 * (attention.rs:302-304). */
void oxo_softmax_backward(const float* p, const float* dy, float* dx, size_t rows, size_t cols,
                          float scale);
/* row.rs:239-347. */
void oxo_layer_norm_backward(const float* x, const float* dy, float* dx, size_t rows, size_t cols,
                             float eps);
/* row.rs:398-468. */
void oxo_rms_norm_backward(const float* x, const float* dy, float* dx, size_t rows, size_t cols,
                           float eps);

/* Linear::loss_rows, linear.rs:325-333: per row mean_j 0.5*(y-t)^2. */
void oxo_loss_rows(const float* y, const float* t, float* row_loss, size_t rows, size_t cols);
/* Gradient of sum_rows(loss_rows) w.r.t. y: (y - t)/cols. (No reference
 * counterpart; defined to match loss_rows.) */
void oxo_mse_grad(const float* y, const float* t, float* g, size_t rows, size_t cols);

/* ---- Executors (single sequence, reference semantics) ------------------- */

/* One Linear layer: W [in,out] row-major, optional bias [out]. */
typedef struct {
    float* w;
    float* b; /* NULL = no bias */
    size_t in, out;
    int act;
} oxo_linear;

/* Linear::forward, linear.rs:116-206: Y = act(X·W + b + R). If `pre` is not
 * NULL the pre-activation X·W + b + R is stored there too. `rounding` selects
 * the GEMM operand rounding. */
void oxo_linear_forward(const oxo_linear* l, const float* x, const float* residual, float* y,
                        float* pre, size_t rows, int rounding);

/* MLP (MlpExecutor, mlp.rs:14-168). res_start/res_end < 0: no residual. */
typedef struct {
    oxo_linear* layers;
    size_t n_layers;
    int res_start, res_end;
} oxo_mlp;

/* mlp.rs:53-85. `tape` (may be NULL) receives layer inputs: tape[i] is an
 * [rows, layers[i].in] buffer the caller owns, tape[0] = input copy. */
void oxo_mlp_forward(const oxo_mlp* m, const float* x, float* y, float** tape, size_t rows,
                     int rounding);
/* mlp.rs:121-168: backward with immediate SGD per layer (linear.rs:373-391).
 * Writes dX to dx. */
void oxo_mlp_backward(oxo_mlp* m, float* const* tape, const float* dy, float* dx, size_t rows,
                      float lr, int rounding);

/* Single-head, single-block Post-Norm transformer
 * (encoder.rs:94-187, inference.rs:76-109, attention.rs:221-321). */
typedef struct {
    size_t seq, hidden, out;
    int norm;     /* OXO_NORM_* */
    oxo_linear q, k, v;
    float* position; /* [seq, hidden] */
    oxo_mlp ffn;
    oxo_linear o;
} oxo_transformer;

/* Inference forward (InferenceTransformer::forward; causal != 0 gives the
 * decoder's forward_mask, decoder.rs:50-52). y: [seq, out]. */
void oxo_transformer_forward(const oxo_transformer* t, const float* x, float* y, int causal,
                             int rounding);

/* Training step on one sequence: TrainingTransformer::forward followed by
 * backward(dL/dy, lr) with the reference's immediate per-layer SGD
 * (encoder.rs:114-186). dL/dy = oxo_mse_grad(y, target). Writes y (output),
 * row_loss [seq] (may be NULL) and dx (input gradient, may be NULL).
 * If `grads` is not NULL and lr == 0, the parameter gradients are ADDED
 * into it in checkpoint cursor order (q, k, v, position, ffn layers, out;
 * weight then bias per Linear) instead of being applied. */
void oxo_transformer_train_step(oxo_transformer* t, const float* x, const float* target,
                                float* y, float* row_loss, float* dx, float lr, float* grads,
                                int rounding);

/* Number of f32 parameters in cursor order (inference.rs:52-66). */
size_t oxo_transformer_param_count(const oxo_transformer* t);

/* Attention core with `heads` heads (heads = 1: the reference's
 * attention.rs:359-401; see oxf_oracle.c). q, k: [S, D]; v, att, dr, dv:
 * [S, Hv]; p: [heads, S, S]; D and Hv divisible by heads. */
void oxo_attention_forward_heads(const float* q, const float* k, const float* v, float* p_keep,
                                 float* att, size_t S, size_t D, size_t Hv, size_t heads,
                                 int causal, int rounding);
void oxo_attention_backward_heads(const float* q, const float* k, const float* v,
                                  const float* p, const float* dr, float* dq, float* dk,
                                  float* dv, size_t S, size_t D, size_t Hv, size_t heads,
                                  int rounding);
/* oxo_transformer_forward / _train_step with multi-head attention. */
void oxo_transformer_forward_heads(const oxo_transformer* t, const float* x, float* y,
                                   int causal, int rounding, int heads);
void oxo_transformer_train_step_heads(oxo_transformer* t, const float* x, const float* target,
                                      float* y, float* row_loss, float* dx, float lr,
                                      float* grads, int rounding, int heads);

#ifdef __cplusplus
}
#endif
#endif
