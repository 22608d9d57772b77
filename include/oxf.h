/*
 * oxf.h — C ABI of the B200 (sm_100a) kernels that replace OxideForge's
 * cuda-oxide kernel module.
 *
 * The reference's device boundary is `#[cuda_module] mod kernels`
 * (src/cuda/device/module.rs:5-263): 24 `#[kernel]` entry points taking
 * `#[repr(C)]` slice descriptors {ptr,len} by value (src/cuda/span.rs:7-10,
 * 45-48), usize/f32 scalars and `BinaryOp` as repr(u8) (src/cuda.rs:3-10).
 * Each function below names the reference entry point it replaces.
 *
 * Conventions
 *  - All matrices are contiguous row-major f32 in device memory, owned by
 *    the caller. No entry point allocates device memory; the only scratch
 *    any of them needs (3xTF32 operand splits) is caller-provided.
 *  - Every call is asynchronous on the given stream (NULL = legacy default
 *    stream) and acts on the calling thread's current CUDA device.
 *  - Every call returns an oxf_status. On error, oxf_last_error_string()
 *    describes it (thread-local). No entry point aborts the process.
 *  - Where the reference asserts a shape (`assert!` in the src/cuda/container files),
 *    the same check returns OXF_ERR_INVALID_ARG. The reference's caps
 *    (cols <= 1024 for row kernels, M/N/K % 16 for the GEMM) are lifted.
 */
#ifndef OXF_H
#define OXF_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* oxf_stream; /* == cudaStream_t */

typedef enum {
  OXF_OK = 0,
  OXF_ERR_INVALID_ARG = 1,
  OXF_ERR_UNSUPPORTED_SHAPE = 2,
  OXF_ERR_CUDA = 3,
  OXF_ERR_TIMEOUT = 4,
  OXF_ERR_DEVICE_CHECK = 5,
  OXF_ERR_IO = 6,
  OXF_ERR_STATE = 7
} oxf_status;

/* DeviceSliceDescriptor<f32> (span.rs:7-10) and
 * DeviceSliceMutDescriptor<f32> (span.rs:45-48). */
typedef struct { const float* ptr; size_t len; } oxf_cslice;
typedef struct { float* ptr; size_t len; } oxf_slice;

/* BinaryOp, src/cuda.rs:3-10. */
typedef enum { OXF_ADD = 0, OXF_SUB = 1, OXF_MUL = 2, OXF_DIV = 3 } oxf_binary_op;

/* Activation, src/net/linear.rs:14-19. */
typedef enum { OXF_ACT_IDENTITY = 0, OXF_ACT_GELU = 1, OXF_ACT_RELU = 2, OXF_ACT_SILU = 3 }
    oxf_activation;

/* The closures the reference passes to slice_for_each (module.rs:59-67)
 * cannot cross a C ABI; these are the ones its callers use:
 *   SCALE        x * p             (Matrix::scale, matrix.rs:30; linear.rs:383)
 *   ADD_SCALAR   x + p             (matrix.rs:34)
 *   ACT_FORWARD  act(x)            (linear.rs:225-230), act = (int)p
 *   ACT_DERIV    act'(x)           (linear.rs:262), act = (int)p
 *   HALF_SQUARE  0.5 * x * x       (linear.rs:327)                      */
typedef enum {
  OXF_UNARY_SCALE = 0,
  OXF_UNARY_ADD_SCALAR = 1,
  OXF_UNARY_ACT_FORWARD = 2,
  OXF_UNARY_ACT_DERIV = 3,
  OXF_UNARY_HALF_SQUARE = 4
} oxf_unary_op;

/* NormType, src/net/transformer.rs:7-13 (Rms = 0, Layer = 1). */
typedef enum { OXF_NORM_RMS = 0, OXF_NORM_LAYER = 1 } oxf_norm_type;

/* ---------------------------------------------------------------- status */
const char* oxf_last_error_string(void);
/* Reads and clears the device error word that bounded in-kernel waits set
 * (0 = none). Synchronises the current device. Codes: 0x101-0x107 GEMM
 * pipeline waits, 0x108 the fused multi-head attention's waits, 0x1FF the self-test below, OXF_DEVERR_EXCHANGE_START / _END
 * the exchange barriers, OXF_DEVERR_ROW_PARAMS a norm kernel's gamma / beta
 * copy into shared memory. */
oxf_status oxf_device_error(uint32_t* code);
#define OXF_DEVERR_ROW_PARAMS 0x301u
/* Failure-detection self-test: a one-thread kernel waits on an mbarrier
 * that nothing completes, bounded by limit_us (1..1e6), exactly as every
 * pipeline wait in this library is bounded. On expiry it writes 1 to the
 * device int *expired, records 0x1FF in the device error word and returns:
 * no hang, no fault, the context stays usable. No counterpart in the
 * reference (its waits are unbounded). */
oxf_status oxf_wait_timeout_selftest(uint32_t limit_us, int* expired, oxf_stream stream);
/* Library version string. */
const char* oxf_version(void);
/* Kernels this library has launched in this process (all devices). */
unsigned long long oxf_kernel_launches(void);

/* ---------------------------------------------------------------- elementwise */
/* slice_binary (module.rs:36-43): out = lhs op rhs over min(len). */
oxf_status oxf_slice_binary(oxf_cslice lhs, oxf_cslice rhs, oxf_slice out, oxf_binary_op op,
                            oxf_stream stream);
/* slice_binary_assign (module.rs:48-54): target op= rhs. */
oxf_status oxf_slice_binary_assign(oxf_slice target, oxf_cslice rhs, oxf_binary_op op,
                                   oxf_stream stream);
/* slice_for_each (module.rs:59-64) for the enumerated closures above. */
oxf_status oxf_slice_unary(oxf_slice span, oxf_unary_op op, float param, oxf_stream stream);
/* target = target - lr * grad (Linear::learn's scale + Sub, linear.rs:383-390,
 * fused). */
oxf_status oxf_sgd_update(oxf_slice target, oxf_cslice grad, float lr, oxf_stream stream);
/* out = (y - t) * (1/cols): gradient of sum(loss_rows) (no reference
 * counterpart; loss_rows is linear.rs:325-333). */
oxf_status oxf_mse_grad(oxf_cslice y, oxf_cslice target, oxf_slice out, size_t cols,
                        oxf_stream stream);
/* loss_rows and its gradient in one pass: row_loss[r] = mean_j 0.5(y-t)^2
 * and dy = (y - t)/cols. */
oxf_status oxf_mse_loss_grad(oxf_cslice y, oxf_cslice target, oxf_slice row_loss, oxf_slice dy,
                             size_t cols, oxf_stream stream);
/* Linear::loss_rows (linear.rs:325-333) fused: row_loss[r] = mean_j 0.5(y-t)^2. */
oxf_status oxf_loss_rows(oxf_cslice y, oxf_cslice target, oxf_slice row_loss, size_t cols,
                         oxf_stream stream);

/* ---------------------------------------------------------------- reductions */
/* slice_sum + host re-launch loop (module.rs:69-74, span.rs:301-385) as one
 * launch: *result = sum(span). result is a device pointer to one float. */
oxf_status oxf_slice_sum(oxf_cslice span, float* result, oxf_stream stream);
/* slice_max (module.rs:92-97, span.rs:318-333); empty -> f32::MIN. */
oxf_status oxf_slice_max(oxf_cslice span, float* result, oxf_stream stream);
/* slice_map_sum (module.rs:79-90, reduction.rs:44-80, span.rs:335-359):
 * *result = sum_i f(span[i]), the closure given as an oxf_unary_op with
 * its parameter (as oxf_slice_unary). */
oxf_status oxf_slice_map_sum(oxf_cslice span, oxf_unary_op op, float param, float* result,
                             oxf_stream stream);
/* Vector::dot (vector.rs:109-115: an elementwise product into a temporary
 * vector, then its sum) as one reduction launch with no temporary:
 * *result = sum_i lhs[i] * rhs[i]. Lengths must match (vector.rs:110). */
oxf_status oxf_slice_dot(oxf_cslice lhs, oxf_cslice rhs, float* result, oxf_stream stream);

/* ---------------------------------------------------------------- fills */
/* slice_set (module.rs:15-20): every element = value. */
oxf_status oxf_slice_set(oxf_slice target, float value, oxf_stream stream);
/* slice_set_seq (module.rs:22-27, elementwise.rs:24-35): element i = i
 * (dir != 0) or len - i, as f32. */
oxf_status oxf_slice_set_seq(oxf_slice target, int dir, oxf_stream stream);
/* slice_set_random (module.rs:29-34, elementwise.rs:37-43): element i =
 * h(seed + i) / (float)UINT32_MAX with the reference's hash h
 * (common.rs:3-9: x += x<<13; x -= x>>17; x *= x<<5, wrapping 32-bit), so
 * the same seed fills the same values as the reference. */
oxf_status oxf_slice_set_random(oxf_slice target, uint32_t seed, oxf_stream stream);
/* matrix_sum_rows (module.rs:102-108): result[r] = sum_j M[r,j]. */
oxf_status oxf_matrix_sum_rows(oxf_cslice matrix, oxf_slice result, size_t cols,
                               oxf_stream stream);
/* Column sums: result[j] = sum_r M[r,j]; replaces the reference's bias
 * gradient sum_rows(transpose(G)) (linear.rs:267-270). If accumulate != 0
 * the sums are added to result. */
oxf_status oxf_matrix_sum_cols(oxf_cslice matrix, oxf_slice result, size_t cols, int accumulate,
                               oxf_stream stream);

/* ---------------------------------------------------------------- row kernels */
/* matrix_softmax_rows (module.rs:111-116) with matrix_causal_mask
 * (module.rs:245-250) and the attention scale (attention.rs:372) folded in:
 * row r of `cols` entries becomes softmax(scale * x) with entries
 * j > (r % causal_period) masked to -inf first when causal_period != 0. */
oxf_status oxf_matrix_softmax_rows(oxf_slice matrix, size_t cols, float scale,
                                   size_t causal_period, oxf_stream stream);
/* matrix_layer_norm_rows (module.rs:118-127), in place. gamma/beta may be
 * NULL (the reference is non-affine). */
oxf_status oxf_matrix_layer_norm_rows(oxf_slice matrix, size_t cols, float epsilon,
                                      const float* gamma, const float* beta, oxf_stream stream);
/* rms_norm_assign (module.rs:226-231), in place; gamma may be NULL. */
oxf_status oxf_rms_norm_assign(oxf_slice matrix, size_t cols, float epsilon, const float* gamma,
                               oxf_stream stream);
/* Normalization::forward (attention.rs:157-162) out of place: output =
 * LayerNorm or RMSNorm of input by rows (input == output is allowed). */
oxf_status oxf_norm_rows(oxf_cslice input, oxf_slice output, size_t cols, int norm_type,
                         float epsilon, const float* gamma, const float* beta, oxf_stream stream);
/* Normalization::backward (attention.rs:164-174). */
oxf_status oxf_norm_rows_backward(oxf_cslice input, oxf_cslice output_gradient, oxf_slice result,
                                  size_t cols, int norm_type, float epsilon, oxf_stream stream);
/* out[i] = lhs[i] op rhs[i % rhs.len]: the position table added to every
 * sequence of a batch (inference.rs:78, encoder.rs:117). */
oxf_status oxf_slice_binary_broadcast(oxf_cslice lhs, oxf_cslice rhs, oxf_slice out,
                                      oxf_binary_op op, oxf_stream stream);
/* gradient[i] *= act'(pre_activation[i]): Linear::backward's clone +
 * derivative + multiply (linear.rs:254-265) in one pass. */
oxf_status oxf_slice_mul_act_derivative(oxf_slice gradient, oxf_cslice pre_activation,
                                        oxf_activation act, oxf_stream stream);
/* softmax_rows_backward (module.rs:141-151): dx = scale * p*(dy - sum(p*dy)). */
oxf_status oxf_softmax_rows_backward(oxf_cslice probabilities, oxf_cslice output_gradient,
                                     oxf_slice result, size_t cols, float scale,
                                     oxf_stream stream);
/* layer_norm_backward (module.rs:153-163), non-affine. */
oxf_status oxf_layer_norm_backward(oxf_cslice input, oxf_cslice output_gradient,
                                   oxf_slice result, size_t cols, float epsilon,
                                   oxf_stream stream);
/* matrix_rms_norm_backward (module.rs:252-262), non-affine. */
oxf_status oxf_matrix_rms_norm_backward(oxf_cslice input, oxf_cslice output_gradient,
                                        oxf_slice result, size_t cols, float epsilon,
                                        oxf_stream stream);
/* matrix_binary_assign_by_rows (module.rs:129-139): M[i,j] op= row[j]. */
oxf_status oxf_matrix_binary_assign_by_rows(oxf_slice matrix, oxf_cslice row, size_t cols,
                                            oxf_binary_op op, oxf_stream stream);
/* matrix_causal_mask (module.rs:245-250): M[i,j] = -inf for j > i. */
oxf_status oxf_matrix_causal_mask(oxf_slice matrix, size_t cols, oxf_stream stream);
/* matrix_slice (module.rs:208-227, layout.rs:58-86, container/convert.rs:
 * 105-130): cuts a matrix with input_cols columns into tile_rows x
 * tile_cols tiles, tiles_per_row of them per row of tiles, and writes them
 * one after another (each row-major) into output; output.len / (tile_rows *
 * tile_cols) tiles are taken. Tiles reaching past the input are refused. */
oxf_status oxf_matrix_slice(oxf_cslice input, oxf_slice output, size_t input_cols,
                            size_t tile_rows, size_t tile_cols, size_t tiles_per_row,
                            oxf_stream stream);
/* matrix_transpose (module.rs:193-203): out[cols,rows] = in[rows,cols]^T. */
oxf_status oxf_matrix_transpose(oxf_cslice input, oxf_slice result, size_t rows, size_t cols,
                                oxf_stream stream);

/* ---------------------------------------------------------------- GEMM */
/* TF32: tensor cores, TF32 operands. TF32X3: tensor cores, hi+lo splits (f32-faithful).
 * F32: CUDA cores, f32 products and sums (the reference's matrix_multiply_fp32). */
typedef enum { OXF_PREC_TF32 = 0, OXF_PREC_TF32X3 = 1, OXF_PREC_F32 = 2 } oxf_precision;

/* One (batched) GEMM with a fused epilogue:
 *   acc = alpha * op(A)·op(B)                         [M,N] per batch item
 *   acc += beta * C          (beta != 0, not with accumulate)
 *   acc += bias[n]           (bias != NULL)
 *   acc += R[m,n]            (residual != NULL)
 *   P[m,n] = acc             (pre_out != NULL: pre-activation store)
 *   acc *= act'(X[m,n])      (grad_act != IDENTITY, X = aux)
 *   acc = act(acc)           (act != IDENTITY)
 *   C = acc, or C += acc atomically (accumulate != 0; allows split_k > 1)
 * A is [M,K] (a_trans = 0) or stored as [K,M] (a_trans = 1, A = storedᵀ).
 * B is [K,N] (b_trans = 0) or stored as [N,K] (b_trans = 1).
 * Leading dimensions are in elements; *_stride are batch strides in
 * elements (0 = the operand is shared by every batch item). The order
 * GEMM -> bias -> residual -> activation is Linear::affine_on + activate_on
 * (linear.rs:185-230). The TF32 path truncates operands to TF32 in the
 * tensor core; OXF_PREC_TF32X3 splits each operand into hi+lo TF32 parts
 * (needs `workspace`, see oxf_gemm_workspace_size). */
typedef struct {
  int M, N, K, batch;
  int a_trans, b_trans;
  const float* A; long long lda; long long stride_a;
  const float* B; long long ldb; long long stride_b;
  float* C; long long ldc; long long stride_c;
  float alpha, beta;
  const float* bias;
  const float* residual; long long ldr; long long stride_r;
  float* pre_out; long long ldp; long long stride_p;
  const float* aux; long long ldx; long long stride_x;
  int act;        /* oxf_activation applied last */
  int grad_act;   /* oxf_activation whose derivative at aux multiplies acc */
  int accumulate; /* 1: C += result with atomics */
  int split_k;    /* 0/1 = none; >1 requires accumulate */
  int precision;  /* oxf_precision */
  void* workspace; size_t workspace_bytes;
  int reduce_batch; /* 1: C = sum over the batch of op(A_b)·op(B_b) (one output,
                       output strides 0); K then runs over batch x K */
  int variant;      /* kernel choice: 0 automatic, 1 one CTA per 128-row tile,
                       2 a CTA pair per 256 x 256 tile (tcgen05 cta_group::2),
                       3 a CTA pair per 256 x 512 tile (TF32 only) */
} oxf_gemm_desc;

/* Fills a descriptor with defaults (batch 1, alpha 1, tight leading dims
 * for the given shape/transposes, everything else off). */
void oxf_gemm_desc_init(oxf_gemm_desc* d, int M, int N, int K, int a_trans, int b_trans,
                        const float* A, const float* B, float* C);
/* Bytes of workspace the descriptor needs (0 for plain TF32). */
size_t oxf_gemm_workspace_size(const oxf_gemm_desc* d);
oxf_status oxf_gemm(const oxf_gemm_desc* d, oxf_stream stream);

/* Which kernel oxf_gemm runs a descriptor on, with what tile, K splits and
 * raster: the library's own choice, reported for integrators tuning their
 * shapes and for tests of that choice. No counterpart in the reference,
 * whose GEMM has one 32 x 32 tiling (gemm.rs:202-373). Nothing is launched
 * and the operand pointers are only checked for alignment. sm_count <= 0
 * asks the current device (a GPU is then needed); > 0 plans for that many
 * SMs (148 on B200). Invalid descriptors get oxf_gemm's errors. */
typedef enum {
  OXF_GEMM_PATH_NONE = 0,     /* M or N is 0: nothing runs */
  OXF_GEMM_PATH_SIMT = 1,     /* operands TMA cannot read, K = 0, or OXF_PREC_F32 */
  OXF_GEMM_PATH_TINY = 2,     /* a tiny TF32 product on the CUDA cores */
  OXF_GEMM_PATH_ONE_CTA = 3,  /* tcgen05, one CTA per 128-row tile */
  OXF_GEMM_PATH_CTA_PAIR = 4  /* tcgen05 cta_group::2, a CTA pair per 256-row tile */
} oxf_gemm_path;
typedef struct {
  int path;        /* oxf_gemm_path */
  int tile_m;      /* output tile rows (per CTA pair on the pair path) */
  int tile_n;      /* output tile columns */
  int stages;      /* operand ring stages (tensor-core paths) */
  int staging;     /* epilogue staging tiles per warp */
  int splits;      /* K splits (1: none) */
  int group_m;     /* tile rows per raster group (1: N fastest) */
  int zero_c;      /* 1: C is zeroed first and the K splits add into it */
  long long units; /* work units: tiles x splits (tiles for SIMT and tiny) */
} oxf_gemm_plan_info;
oxf_status oxf_gemm_plan(const oxf_gemm_desc* d, int sm_count, oxf_gemm_plan_info* out);

/* oxf_gemm in 3xTF32 precision without any allocation, for callers that
 * cannot call cudaMalloc: plugin hosts that own the device memory budget
 * through their own allocator, and latency-critical paths that must not
 * pay for cudaMalloc's implicit synchronisation. No counterpart in the
 * reference (it has no 3xTF32 mode and no scratch memory).
 * The hi/lo operand splits live in a 16 MiB static device array that every
 * GPU loading the library holds until exit; shapes needing more
 * (oxf_gemm_workspace_size > 16 MiB) return OXF_ERR_UNSUPPORTED_SHAPE.
 * Descriptors oxf_gemm would refuse get oxf_gemm's error; operands the
 * tensor cores cannot read (misaligned, K = 0) run on the CUDA cores with no
 * splits and no size limit. The descriptor's precision and workspace fields
 * are ignored. The first call on a device, and the first after a device
 * reset, looks up the array's device address; such a call made inside a
 * stream capture returns OXF_ERR_INVALID_ARG, so make one call before
 * capturing. All calls on a device share that device's array, which keeps
 * the last call's contents: calls that can overlap on the GPU (issued on
 * different streams of one device) race, so serialise them. */
oxf_status oxf_gemm_tf32x3_noalloc(const oxf_gemm_desc* desc, oxf_stream stream);

/* Scaled dot-product attention of Attention::forward
 * (src/net/transformer/attention.rs:243-253, 359-401) for `batch` independent
 * sequences, with the row softmax fused into its two products:
 *   out = residual + softmax(scale * Q·Kᵀ) · V
 * with the decoder's causal mask (key j of row i kept for j <= i) when causal
 * is 1. q, k: [batch][seq][d_qk]; v, residual (may be NULL), out:
 * [batch][seq][d_v]; all row-major device arrays. scores: caller workspace of
 * batch*seq*seq floats; stats: caller workspace of
 * oxf_attention_stats_floats(batch, seq) floats (8-byte aligned). No
 * allocation. Two forms compute the same result:
 *  - three launches (the default): scores = scale·Q·Kᵀ, the row softmax in
 *    place, then P·V + residual; scores then holds the probabilities.
 *  - fused (environment OXF_ATTENTION=fused, read at every call; rows must
 *    be 16-byte aligned, else the three launches run): the score product's
 *    epilogue stores, for each 32-column chunk of a row, exp(logit - chunk
 *    maximum) into scores (0 where masked) and (chunk maximum, chunk sum)
 *    into stats; the P·V product reads those values as its A operand and
 *    scales each tile in shared memory by exp(chunk maximum - row maximum)
 *    / row sum before the tensor cores read it, so the probabilities are
 *    never written and no softmax pass runs. On B200 at 64 sequences of
 *    [2048, 1024] it took 3.5 ms against 2.2 ms for the three launches. */
size_t oxf_attention_stats_floats(int batch, int seq);
oxf_status oxf_attention_forward(const float* q, const float* k, const float* v,
                                 const float* residual, float* out, float* scores, float* stats,
                                 int batch, int seq, int d_qk, int d_v, float scale, int causal,
                                 oxf_stream stream);
/* Multi-head attention in one fused kernel: for every head j and sequence,
 *   out[:, j*w .. (j+1)*w) = residual + softmax(Q_j·K_jᵀ / sqrt(w)) · V_j
 * where Q_j, K_j, V_j are columns [j*w, (j+1)*w) of q, k, v and
 * w = d_qk/heads (the head split docs/api.md:440-442 anticipates;
 * heads = 1 is Attention::forward with query width w). q, k:
 * [batch][seq][d_qk]; v, residual (may be NULL), out: [batch][seq][d_v].
 * Each CTA keeps a 128-row query tile's scores in TMEM and runs the softmax
 * online, so the seq x seq scores are never written: no workspace, no
 * allocation. heads must divide d_qk and d_v (else INVALID_ARG). Needs
 * d_qk = d_v, w = 32 or 64, seq a multiple of 128 and 16-byte aligned
 * matrices; otherwise OXF_ERR_UNSUPPORTED_SHAPE and nothing runs. A stalled
 * pipeline wait records 0x108 in the device error word. */
oxf_status oxf_attention_heads_forward(const float* q, const float* k, const float* v,
                                       const float* residual, float* out, int batch, int seq,
                                       int d_qk, int d_v, int heads, int causal,
                                       oxf_stream stream);

/* matrix_multiply (module.rs:179-191) with the reference's argument order:
 * result[rows,cols] = lhs[rows,len] · rhs[len,cols], TF32 operands, f32
 * accumulation. The reference asserts rows, cols, len % 16 == 0
 * (matrix.rs:147-149); this entry point accepts any sizes. */
oxf_status oxf_matrix_multiply(oxf_cslice lhs, oxf_cslice rhs, oxf_slice result, size_t len,
                               size_t rows, size_t cols, oxf_stream stream);

/* matrix_multiply_fp32 (module.rs:165-177, gemm.rs:16-113): the same
 * product with f32 operands and f32 fused multiply-adds on the CUDA cores
 * (no TF32 rounding), tiled 32 x 32 as the reference does. Any sizes. */
oxf_status oxf_matrix_multiply_fp32(oxf_cslice lhs, oxf_cslice rhs, oxf_slice result, size_t len,
                                    size_t rows, size_t cols, oxf_stream stream);

/* Reference-algorithm restatement, for measurement only: the reference's
 * 32x32-tile, 128-thread, mma.sync.m16n8k8 TF32, 2-stage cp.async GEMM
 * (gemm.rs:202-373) written in CUDA C++. Same contract and asserts as
 * matrix_multiply (rows, cols, len % 16 == 0). */
oxf_status oxf_matrix_multiply_refalgo(oxf_cslice lhs, oxf_cslice rhs, oxf_slice result,
                                       size_t len, size_t rows, size_t cols, oxf_stream stream);

/* ---------------------------------------------------------------- peer exchange
 * Data-parallel SGD over the GPUs of one node in one kernel per rank, over
 * NVLink peer memory instead of a library all-reduce followed by an update.
 * No reference counterpart: the reference trains on one GPU
 * (src/cuda/runtime.rs:34-45) and its update is Linear::learn's
 * W -= lr * dW (src/net/linear.rs:373-391).
 *
 * Every process maps every other rank's parameter arena, gradient arena and
 * signal pad (CUDA IPC handles, exchanged by the caller). One call of
 * oxf_exchange_sgd on every rank, with the same offset, count, lr, epoch and
 * blocks, computes for each element i of [offset, offset + count)
 *     p_i = p_i - lr * (g0_i + g1_i + ... + g{world-1}_i)
 * (rank order, left to right) with each rank owning 1/world of the range:
 * it reads that shard's gradients from every rank, updates its own copy of
 * the parameters and stores the result into every rank's parameter arena.
 * All ranks therefore hold bit-identical parameters afterwards; with
 * world == 1 the result equals oxf_sgd_update bit for bit.
 *
 * Two cross-GPU barriers per CTA bracket the data movement: the start barrier
 * (every rank's kernel has begun, so the gradients its stream produced
 * before it are complete) and the end barrier (every rank has finished
 * reading this rank's gradients and writing its parameters). Each barrier
 * wait is bounded by timeout_us; on expiry the kernel records
 * OXF_DEVERR_EXCHANGE_START / _END in the device error word (read by
 * oxf_device_error), skips the rest of its work and returns. */
#define OXF_EXCHANGE_MAX_RANKS 8
#define OXF_EXCHANGE_MAX_BLOCKS 1024
/* Bytes of one rank's signal pad; zero it once before the first call. */
#define OXF_EXCHANGE_SIGNAL_BYTES (2u * OXF_EXCHANGE_MAX_BLOCKS * OXF_EXCHANGE_MAX_RANKS * 4u)
#define OXF_DEVERR_EXCHANGE_START 0x201u
#define OXF_DEVERR_EXCHANGE_END 0x202u

typedef struct {
  int rank;  /* this process's rank, 0 <= rank < world */
  int world; /* 1..OXF_EXCHANGE_MAX_RANKS */
  /* Indexed by rank, each as mapped into this process (its own entry is
   * local memory). All 16-byte aligned. */
  float* params[OXF_EXCHANGE_MAX_RANKS];
  const float* grads[OXF_EXCHANGE_MAX_RANKS];
  uint32_t* signals[OXF_EXCHANGE_MAX_RANKS];
  uint32_t epoch;      /* nonzero, larger than every earlier call's on these pads */
  int blocks;          /* CTAs per rank, equal on all ranks; 0 = one per SM */
  uint32_t timeout_us; /* bound of each barrier wait; 0 = 4 s */
} oxf_exchange_desc;

oxf_status oxf_exchange_sgd(const oxf_exchange_desc* desc, size_t offset, size_t count, float lr,
                            oxf_stream stream);

/* CUDA IPC for the exchange: a handle names the cudaMalloc allocation that
 * holds `ptr` plus ptr's offset inside it. oxf_ipc_open maps another
 * process's allocation (peer access over NVLink) and returns the pointer at
 * the same offset; oxf_ipc_close unmaps it. A process does not open its own
 * handles. */
typedef struct {
  unsigned char handle[64]; /* cudaIpcMemHandle_t */
  uint64_t offset;
} oxf_ipc_handle;

oxf_status oxf_ipc_export(const void* ptr, oxf_ipc_handle* out);
oxf_status oxf_ipc_open(const oxf_ipc_handle* handle, void** ptr);
oxf_status oxf_ipc_close(const oxf_ipc_handle* handle, void* ptr);

#ifdef __cplusplus
}
#endif
#endif
