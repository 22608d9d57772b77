// abi.cu — the extern "C" entry points declared in include/oxf.h.
//
// Each function validates its arguments the way the reference's launchers
// assert them (src/cuda/container/*.rs), minus the caps this build lifts,
// then forwards to the kernels in rows.cu / gemm.cu on the caller's stream.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "../../include/oxf.h"
#include "status.cuh"

namespace oxf {

// rows.cu
oxf_status rows_read_device_error(uint32_t*);
// attention.cu
oxf_status attention_read_device_error(uint32_t*);
oxf_status rows_softmax(float*, long long, long long, float, long long, cudaStream_t);
oxf_status rows_softmax_bwd(const float*, const float*, float*, long long, long long, float,
                            cudaStream_t);
oxf_status rows_layernorm(const float*, float*, long long, long long, float, const float*,
                          const float*, cudaStream_t);
oxf_status rows_layernorm_bwd(const float*, const float*, float*, long long, long long, float,
                              cudaStream_t);
oxf_status rows_rmsnorm(const float*, float*, long long, long long, float, const float*,
                        cudaStream_t);
oxf_status ew_binary_bcast(const float*, const float*, float*, long long, long long, int,
                           cudaStream_t);
oxf_status ew_mul_act_deriv(float*, const float*, long long, int, cudaStream_t);
oxf_status rows_rmsnorm_bwd(const float*, const float*, float*, long long, long long, float,
                            cudaStream_t);
oxf_status rows_sum(const float*, float*, long long, long long, cudaStream_t);
oxf_status rows_loss(const float*, const float*, float*, long long, long long, cudaStream_t);
oxf_status rows_loss_grad(const float*, const float*, float*, float*, long long, long long,
                          cudaStream_t);
oxf_status ew_binary(const float*, const float*, float*, long long, int, cudaStream_t);
oxf_status ew_binary_assign(float*, const float*, long long, int, cudaStream_t);
oxf_status ew_unary(float*, long long, int, float, cudaStream_t);
oxf_status ew_sgd(float*, const float*, long long, float, cudaStream_t);
oxf_status ew_mse_grad(const float*, const float*, float*, long long, long long, cudaStream_t);
oxf_status ew_by_rows(float*, const float*, long long, long long, int, cudaStream_t);
oxf_status causal_mask(float*, long long, long long, cudaStream_t);
oxf_status cols_sum(const float*, float*, long long, long long, int, cudaStream_t);
oxf_status transpose(const float*, float*, long long, long long, cudaStream_t);
oxf_status slice_reduce(const float*, long long, float*, int, cudaStream_t, int map_op = -1,
                        float map_p = 0.f, const float* y = nullptr);
oxf_status fill_slice(float*, long long, int, float, int, uint32_t, cudaStream_t);
oxf_status matrix_slice(const float*, float*, long long, long long, long long, long long,
                        long long, cudaStream_t);
// gemm.cu
oxf_status gemm_run(const oxf_gemm_desc*, cudaStream_t);
size_t gemm_workspace_bytes(const oxf_gemm_desc*);
oxf_status gemm_refalgo(const float*, const float*, float*, size_t, size_t, size_t,
                        cudaStream_t);
oxf_status gemm_read_device_error(uint32_t*);
oxf_status wait_selftest(unsigned long long, int*, cudaStream_t);
oxf_status gemm_tf32x3_noalloc(const oxf_gemm_desc*, cudaStream_t);
oxf_status gemm_plan_report(const oxf_gemm_desc*, int, oxf_gemm_plan_info*);
long long attention_stats_parts(long long);
oxf_status attention_forward(const float*, const float*, const float*, const float*, float*,
                             float*, float*, int, int, int, int, float, int, cudaStream_t);
oxf_status attention_heads_forward(const float*, const float*, const float*, const float*, float*,
                                   int, int, int, int, int, int, cudaStream_t);
// exchange.cu
oxf_status exchange_sgd(const oxf_exchange_desc*, size_t, size_t, float, cudaStream_t);
oxf_status exchange_read_device_error(uint32_t*);
oxf_status ipc_export(const void*, oxf_ipc_handle*);
oxf_status ipc_open(const oxf_ipc_handle*, void**);
oxf_status ipc_close(const oxf_ipc_handle*, void*);

namespace {
thread_local char g_last_error[512] = "";
std::atomic<unsigned long long> g_launches{0};
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

oxf_status set_error(oxf_status st, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return st;
}

}  // namespace oxf

using namespace oxf;

namespace {

inline cudaStream_t S(oxf_stream s) { return reinterpret_cast<cudaStream_t>(s); }

oxf_status need(bool cond, const char* what) {
  return cond ? OXF_OK : set_error(OXF_ERR_INVALID_ARG, "%s", what);
}

#define OXF_TRY(x)                   \
  do {                               \
    oxf_status _st = (x);            \
    if (_st != OXF_OK) return _st;   \
  } while (0)

bool valid_op(int op) { return op >= OXF_ADD && op <= OXF_DIV; }
bool valid_act(int a) { return a >= OXF_ACT_IDENTITY && a <= OXF_ACT_SILU; }

// rows = len / cols with the reference's shape checks: a row kernel needs
// cols > 0 and a whole number of rows (norm.rs:12,30,54; rows.rs:73).
oxf_status rows_of(size_t len, size_t cols, long long* rows, const char* who) {
  if (len == 0) {
    *rows = 0;
    return OXF_OK;
  }
  if (cols == 0) return set_error(OXF_ERR_INVALID_ARG, "%s: cols must be > 0", who);
  if (len % cols) return set_error(OXF_ERR_INVALID_ARG, "%s: len %% cols != 0", who);
  *rows = static_cast<long long>(len / cols);
  return OXF_OK;
}

}  // namespace

extern "C" {

const char* oxf_last_error_string(void) { return g_last_error; }

const char* oxf_version(void) { return "oxf-b200 0.1 (sm_100a)"; }

unsigned long long oxf_kernel_launches(void) { return g_launches.load(); }

oxf_status oxf_device_error(uint32_t* code) {
  if (!code) return set_error(OXF_ERR_INVALID_ARG, "oxf_device_error: null code");
  OXF_TRY(check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize"));
  // Each translation unit with bounded waits has its own word; report the
  // first nonzero one and clear them all.
  uint32_t g = 0, x = 0, r = 0, a = 0;
  OXF_TRY(gemm_read_device_error(&g));
  OXF_TRY(exchange_read_device_error(&x));
  OXF_TRY(rows_read_device_error(&r));
  OXF_TRY(attention_read_device_error(&a));
  *code = g ? g : (x ? x : (r ? r : a));
  return OXF_OK;
}

oxf_status oxf_exchange_sgd(const oxf_exchange_desc* desc, size_t offset, size_t count, float lr,
                            oxf_stream stream) {
  return exchange_sgd(desc, offset, count, lr, S(stream));
}

oxf_status oxf_ipc_export(const void* ptr, oxf_ipc_handle* out) { return ipc_export(ptr, out); }
oxf_status oxf_ipc_open(const oxf_ipc_handle* handle, void** ptr) { return ipc_open(handle, ptr); }
oxf_status oxf_ipc_close(const oxf_ipc_handle* handle, void* ptr) {
  return ipc_close(handle, ptr);
}

oxf_status oxf_wait_timeout_selftest(uint32_t limit_us, int* expired, oxf_stream stream) {
  if (!expired) return set_error(OXF_ERR_INVALID_ARG, "oxf_wait_timeout_selftest: null flag");
  if (limit_us == 0 || limit_us > 1000000)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_wait_timeout_selftest: limit must be 1..1e6 us");
  return wait_selftest(static_cast<unsigned long long>(limit_us) * 1000ull, expired, S(stream));
}

// ---------------------------------------------------------------- elementwise
oxf_status oxf_slice_binary(oxf_cslice lhs, oxf_cslice rhs, oxf_slice out, oxf_binary_op op,
                            oxf_stream stream) {
  OXF_TRY(need(valid_op(op), "oxf_slice_binary: bad op"));
  size_t n = out.len < lhs.len ? out.len : lhs.len;
  n = n < rhs.len ? n : rhs.len;  // elementwise.rs:53 bounds all three
  if (n && (!lhs.ptr || !rhs.ptr || !out.ptr))
    return set_error(OXF_ERR_INVALID_ARG, "oxf_slice_binary: null pointer");
  return ew_binary(lhs.ptr, rhs.ptr, out.ptr, static_cast<long long>(n), op, S(stream));
}

oxf_status oxf_slice_binary_assign(oxf_slice target, oxf_cslice rhs, oxf_binary_op op,
                                   oxf_stream stream) {
  OXF_TRY(need(valid_op(op), "oxf_slice_binary_assign: bad op"));
  const size_t n = target.len < rhs.len ? target.len : rhs.len;  // elementwise.rs:65
  if (n && (!target.ptr || !rhs.ptr))
    return set_error(OXF_ERR_INVALID_ARG, "oxf_slice_binary_assign: null pointer");
  return ew_binary_assign(target.ptr, rhs.ptr, static_cast<long long>(n), op, S(stream));
}

oxf_status oxf_slice_unary(oxf_slice span, oxf_unary_op op, float param, oxf_stream stream) {
  if (op < OXF_UNARY_SCALE || op > OXF_UNARY_HALF_SQUARE)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_slice_unary: bad op");
  if ((op == OXF_UNARY_ACT_FORWARD || op == OXF_UNARY_ACT_DERIV) &&
      !valid_act(static_cast<int>(param)))
    return set_error(OXF_ERR_INVALID_ARG, "oxf_slice_unary: bad activation");
  if (span.len && !span.ptr) return set_error(OXF_ERR_INVALID_ARG, "oxf_slice_unary: null");
  return ew_unary(span.ptr, static_cast<long long>(span.len), op, param, S(stream));
}

oxf_status oxf_sgd_update(oxf_slice target, oxf_cslice grad, float lr, oxf_stream stream) {
  OXF_TRY(need(target.len == grad.len, "oxf_sgd_update: length mismatch"));
  if (target.len && (!target.ptr || !grad.ptr))
    return set_error(OXF_ERR_INVALID_ARG, "oxf_sgd_update: null pointer");
  return ew_sgd(target.ptr, grad.ptr, static_cast<long long>(target.len), lr, S(stream));
}

oxf_status oxf_mse_grad(oxf_cslice y, oxf_cslice target, oxf_slice out, size_t cols,
                        oxf_stream stream) {
  OXF_TRY(need(y.len == target.len && y.len == out.len, "oxf_mse_grad: length mismatch"));
  long long rows = 0;
  OXF_TRY(rows_of(y.len, cols, &rows, "oxf_mse_grad"));
  return ew_mse_grad(y.ptr, target.ptr, out.ptr, static_cast<long long>(y.len),
                     static_cast<long long>(cols ? cols : 1), S(stream));
}

oxf_status oxf_loss_rows(oxf_cslice y, oxf_cslice target, oxf_slice row_loss, size_t cols,
                         oxf_stream stream) {
  OXF_TRY(need(y.len == target.len, "oxf_loss_rows: length mismatch"));
  long long rows = 0;
  OXF_TRY(rows_of(y.len, cols, &rows, "oxf_loss_rows"));
  OXF_TRY(need(row_loss.len >= static_cast<size_t>(rows), "oxf_loss_rows: result too short"));
  return rows_loss(y.ptr, target.ptr, row_loss.ptr, rows, static_cast<long long>(cols),
                   S(stream));
}

oxf_status oxf_mse_loss_grad(oxf_cslice y, oxf_cslice target, oxf_slice row_loss, oxf_slice dy,
                             size_t cols, oxf_stream stream) {
  OXF_TRY(need(y.len == target.len && y.len == dy.len, "oxf_mse_loss_grad: length mismatch"));
  long long rows = 0;
  OXF_TRY(rows_of(y.len, cols, &rows, "oxf_mse_loss_grad"));
  OXF_TRY(need(row_loss.len >= static_cast<size_t>(rows), "oxf_mse_loss_grad: result too short"));
  if (rows == 0) return OXF_OK;
  return rows_loss_grad(y.ptr, target.ptr, row_loss.ptr, dy.ptr, rows,
                        static_cast<long long>(cols), S(stream));
}

// ---------------------------------------------------------------- reductions
oxf_status oxf_slice_sum(oxf_cslice span, float* result, oxf_stream stream) {
  OXF_TRY(need(result != nullptr, "oxf_slice_sum: null result"));
  return slice_reduce(span.ptr, static_cast<long long>(span.len), result, 0, S(stream));
}

oxf_status oxf_slice_max(oxf_cslice span, float* result, oxf_stream stream) {
  OXF_TRY(need(result != nullptr, "oxf_slice_max: null result"));
  return slice_reduce(span.ptr, static_cast<long long>(span.len), result, 1, S(stream));
}

oxf_status oxf_slice_map_sum(oxf_cslice span, oxf_unary_op op, float param, float* result,
                             oxf_stream stream) {
  OXF_TRY(need(result != nullptr, "oxf_slice_map_sum: null result"));
  if (op < OXF_UNARY_SCALE || op > OXF_UNARY_HALF_SQUARE)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_slice_map_sum: bad op");
  if ((op == OXF_UNARY_ACT_FORWARD || op == OXF_UNARY_ACT_DERIV) &&
      !valid_act(static_cast<int>(param)))
    return set_error(OXF_ERR_INVALID_ARG, "oxf_slice_map_sum: bad activation");
  if (span.len && !span.ptr) return set_error(OXF_ERR_INVALID_ARG, "oxf_slice_map_sum: null");
  return slice_reduce(span.ptr, static_cast<long long>(span.len), result, 0, S(stream),
                      static_cast<int>(op), param);
}

oxf_status oxf_slice_dot(oxf_cslice lhs, oxf_cslice rhs, float* result, oxf_stream stream) {
  OXF_TRY(need(result != nullptr, "oxf_slice_dot: null result"));
  OXF_TRY(need(lhs.len == rhs.len, "oxf_slice_dot: length mismatch"));  // vector.rs:110
  if (lhs.len && (!lhs.ptr || !rhs.ptr))
    return set_error(OXF_ERR_INVALID_ARG, "oxf_slice_dot: null operand");
  return slice_reduce(lhs.ptr, static_cast<long long>(lhs.len), result, 0, S(stream), -1, 0.f,
                      rhs.ptr);
}

oxf_status oxf_slice_set(oxf_slice target, float value, oxf_stream stream) {
  if (target.len && !target.ptr) return set_error(OXF_ERR_INVALID_ARG, "oxf_slice_set: null");
  return fill_slice(target.ptr, static_cast<long long>(target.len), 0, value, 0, 0, S(stream));
}

oxf_status oxf_slice_set_seq(oxf_slice target, int dir, oxf_stream stream) {
  if (target.len && !target.ptr) return set_error(OXF_ERR_INVALID_ARG, "oxf_slice_set_seq: null");
  return fill_slice(target.ptr, static_cast<long long>(target.len), 1, 0.f, dir != 0, 0,
                    S(stream));
}

oxf_status oxf_slice_set_random(oxf_slice target, uint32_t seed, oxf_stream stream) {
  if (target.len && !target.ptr)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_slice_set_random: null");
  return fill_slice(target.ptr, static_cast<long long>(target.len), 2, 0.f, 0, seed, S(stream));
}

oxf_status oxf_matrix_sum_rows(oxf_cslice matrix, oxf_slice result, size_t cols,
                               oxf_stream stream) {
  long long rows = 0;
  OXF_TRY(rows_of(matrix.len, cols, &rows, "oxf_matrix_sum_rows"));
  OXF_TRY(need(result.len >= static_cast<size_t>(rows), "oxf_matrix_sum_rows: result too short"));
  return rows_sum(matrix.ptr, result.ptr, rows, static_cast<long long>(cols), S(stream));
}

oxf_status oxf_matrix_sum_cols(oxf_cslice matrix, oxf_slice result, size_t cols, int accumulate,
                               oxf_stream stream) {
  long long rows = 0;
  OXF_TRY(rows_of(matrix.len, cols, &rows, "oxf_matrix_sum_cols"));
  OXF_TRY(need(result.len >= cols, "oxf_matrix_sum_cols: result too short"));
  return cols_sum(matrix.ptr, result.ptr, rows, static_cast<long long>(cols), accumulate,
                  S(stream));
}

// ---------------------------------------------------------------- row kernels
oxf_status oxf_matrix_softmax_rows(oxf_slice matrix, size_t cols, float scale,
                                   size_t causal_period, oxf_stream stream) {
  long long rows = 0;
  OXF_TRY(rows_of(matrix.len, cols, &rows, "oxf_matrix_softmax_rows"));
  return rows_softmax(matrix.ptr, rows, static_cast<long long>(cols), scale,
                      static_cast<long long>(causal_period), S(stream));
}

oxf_status oxf_matrix_layer_norm_rows(oxf_slice matrix, size_t cols, float epsilon,
                                      const float* gamma, const float* beta, oxf_stream stream) {
  long long rows = 0;
  OXF_TRY(rows_of(matrix.len, cols, &rows, "oxf_matrix_layer_norm_rows"));
  return rows_layernorm(matrix.ptr, matrix.ptr, rows, static_cast<long long>(cols), epsilon,
                        gamma, beta, S(stream));
}

oxf_status oxf_rms_norm_assign(oxf_slice matrix, size_t cols, float epsilon, const float* gamma,
                               oxf_stream stream) {
  long long rows = 0;
  OXF_TRY(rows_of(matrix.len, cols, &rows, "oxf_rms_norm_assign"));
  return rows_rmsnorm(matrix.ptr, matrix.ptr, rows, static_cast<long long>(cols), epsilon, gamma,
                      S(stream));
}

oxf_status oxf_norm_rows(oxf_cslice input, oxf_slice output, size_t cols, int norm_type,
                         float epsilon, const float* gamma, const float* beta,
                         oxf_stream stream) {
  OXF_TRY(need(input.len == output.len, "oxf_norm_rows: length mismatch"));
  OXF_TRY(need(norm_type == OXF_NORM_RMS || norm_type == OXF_NORM_LAYER,
               "oxf_norm_rows: bad norm type"));
  long long rows = 0;
  OXF_TRY(rows_of(input.len, cols, &rows, "oxf_norm_rows"));
  if (norm_type == OXF_NORM_LAYER)
    return rows_layernorm(input.ptr, output.ptr, rows, static_cast<long long>(cols), epsilon,
                          gamma, beta, S(stream));
  OXF_TRY(need(beta == nullptr, "oxf_norm_rows: RMS norm takes no beta"));
  return rows_rmsnorm(input.ptr, output.ptr, rows, static_cast<long long>(cols), epsilon, gamma,
                      S(stream));
}

oxf_status oxf_norm_rows_backward(oxf_cslice input, oxf_cslice output_gradient, oxf_slice result,
                                  size_t cols, int norm_type, float epsilon, oxf_stream stream) {
  if (norm_type == OXF_NORM_LAYER)
    return oxf_layer_norm_backward(input, output_gradient, result, cols, epsilon, stream);
  if (norm_type == OXF_NORM_RMS)
    return oxf_matrix_rms_norm_backward(input, output_gradient, result, cols, epsilon, stream);
  return set_error(OXF_ERR_INVALID_ARG, "oxf_norm_rows_backward: bad norm type");
}

oxf_status oxf_slice_binary_broadcast(oxf_cslice lhs, oxf_cslice rhs, oxf_slice out,
                                      oxf_binary_op op, oxf_stream stream) {
  OXF_TRY(need(valid_op(op), "oxf_slice_binary_broadcast: bad op"));
  OXF_TRY(need(lhs.len == out.len, "oxf_slice_binary_broadcast: lhs/out length mismatch"));
  if (lhs.len == 0) return OXF_OK;
  OXF_TRY(need(rhs.len > 0 && lhs.len % rhs.len == 0,
               "oxf_slice_binary_broadcast: rhs length must divide lhs length"));
  return ew_binary_bcast(lhs.ptr, rhs.ptr, out.ptr, static_cast<long long>(lhs.len),
                         static_cast<long long>(rhs.len), op, S(stream));
}

oxf_status oxf_slice_mul_act_derivative(oxf_slice gradient, oxf_cslice pre_activation,
                                        oxf_activation act, oxf_stream stream) {
  OXF_TRY(need(valid_act(act), "oxf_slice_mul_act_derivative: bad activation"));
  OXF_TRY(need(gradient.len == pre_activation.len,
               "oxf_slice_mul_act_derivative: length mismatch"));
  return ew_mul_act_deriv(gradient.ptr, pre_activation.ptr,
                          static_cast<long long>(gradient.len), act, S(stream));
}

oxf_status oxf_softmax_rows_backward(oxf_cslice probabilities, oxf_cslice output_gradient,
                                     oxf_slice result, size_t cols, float scale,
                                     oxf_stream stream) {
  OXF_TRY(need(probabilities.len == output_gradient.len && probabilities.len == result.len,
               "oxf_softmax_rows_backward: shape mismatch"));  // norm.rs:78-80
  long long rows = 0;
  OXF_TRY(rows_of(result.len, cols, &rows, "oxf_softmax_rows_backward"));
  return rows_softmax_bwd(probabilities.ptr, output_gradient.ptr, result.ptr, rows,
                          static_cast<long long>(cols), scale, S(stream));
}

oxf_status oxf_layer_norm_backward(oxf_cslice input, oxf_cslice output_gradient,
                                   oxf_slice result, size_t cols, float epsilon,
                                   oxf_stream stream) {
  OXF_TRY(need(input.len == output_gradient.len && input.len == result.len,
               "oxf_layer_norm_backward: shape mismatch"));  // norm.rs:104-106
  long long rows = 0;
  OXF_TRY(rows_of(result.len, cols, &rows, "oxf_layer_norm_backward"));
  return rows_layernorm_bwd(input.ptr, output_gradient.ptr, result.ptr, rows,
                            static_cast<long long>(cols), epsilon, S(stream));
}

oxf_status oxf_matrix_rms_norm_backward(oxf_cslice input, oxf_cslice output_gradient,
                                        oxf_slice result, size_t cols, float epsilon,
                                        oxf_stream stream) {
  OXF_TRY(need(input.len == output_gradient.len && input.len == result.len,
               "oxf_matrix_rms_norm_backward: shape mismatch"));  // norm.rs:130-132
  long long rows = 0;
  OXF_TRY(rows_of(result.len, cols, &rows, "oxf_matrix_rms_norm_backward"));
  return rows_rmsnorm_bwd(input.ptr, output_gradient.ptr, result.ptr, rows,
                          static_cast<long long>(cols), epsilon, S(stream));
}

oxf_status oxf_matrix_binary_assign_by_rows(oxf_slice matrix, oxf_cslice row, size_t cols,
                                            oxf_binary_op op, oxf_stream stream) {
  OXF_TRY(need(valid_op(op), "oxf_matrix_binary_assign_by_rows: bad op"));
  OXF_TRY(need(row.len == cols, "oxf_matrix_binary_assign_by_rows: cols != row.len"));  // rows.rs:18
  long long rows = 0;
  OXF_TRY(rows_of(matrix.len, cols, &rows, "oxf_matrix_binary_assign_by_rows"));
  return ew_by_rows(matrix.ptr, row.ptr, static_cast<long long>(matrix.len),
                    static_cast<long long>(cols ? cols : 1), op, S(stream));
}

oxf_status oxf_matrix_causal_mask(oxf_slice matrix, size_t cols, oxf_stream stream) {
  long long rows = 0;
  OXF_TRY(rows_of(matrix.len, cols, &rows, "oxf_matrix_causal_mask"));
  return causal_mask(matrix.ptr, rows, static_cast<long long>(cols), S(stream));
}

oxf_status oxf_matrix_slice(oxf_cslice input, oxf_slice output, size_t input_cols,
                            size_t tile_rows, size_t tile_cols, size_t tiles_per_row,
                            oxf_stream stream) {
  OXF_TRY(need(tile_rows > 0 && tile_cols > 0 && tiles_per_row > 0,
               "oxf_matrix_slice: tile sizes must be positive"));
  const size_t tile = tile_rows * tile_cols;
  OXF_TRY(need(output.len % tile == 0, "oxf_matrix_slice: output is not a whole number of tiles"));
  OXF_TRY(need(tiles_per_row * tile_cols <= input_cols,
               "oxf_matrix_slice: tiles_per_row * tile_cols exceeds input_cols"));
  if (output.len) {
    const size_t tiles = output.len / tile;
    const size_t last_row = ((tiles - 1) / tiles_per_row + 1) * tile_rows - 1;
    OXF_TRY(need((last_row + 1) * input_cols <= input.len,
                 "oxf_matrix_slice: tiles reach past the input matrix"));
    if (!input.ptr || !output.ptr) return set_error(OXF_ERR_INVALID_ARG, "oxf_matrix_slice: null");
  }
  return matrix_slice(input.ptr, output.ptr, static_cast<long long>(output.len),
                      static_cast<long long>(input_cols), static_cast<long long>(tile_rows),
                      static_cast<long long>(tile_cols), static_cast<long long>(tiles_per_row),
                      S(stream));
}

oxf_status oxf_matrix_transpose(oxf_cslice input, oxf_slice result, size_t rows, size_t cols,
                                oxf_stream stream) {
  OXF_TRY(need(input.len == rows * cols && result.len == rows * cols,
               "oxf_matrix_transpose: shape mismatch"));
  return transpose(input.ptr, result.ptr, static_cast<long long>(rows),
                   static_cast<long long>(cols), S(stream));
}

// ---------------------------------------------------------------- GEMM
void oxf_gemm_desc_init(oxf_gemm_desc* d, int M, int N, int K, int a_trans, int b_trans,
                        const float* A, const float* B, float* C) {
  std::memset(d, 0, sizeof(*d));
  d->M = M; d->N = N; d->K = K; d->batch = 1;
  d->a_trans = a_trans; d->b_trans = b_trans;
  d->A = A; d->lda = a_trans ? M : K;
  d->B = B; d->ldb = b_trans ? K : N;
  d->C = C; d->ldc = N;
  d->alpha = 1.0f;
  d->ldr = d->ldp = d->ldx = N;
  d->act = d->grad_act = OXF_ACT_IDENTITY;
  d->precision = OXF_PREC_TF32;
}

size_t oxf_gemm_workspace_size(const oxf_gemm_desc* d) { return gemm_workspace_bytes(d); }

oxf_status oxf_gemm(const oxf_gemm_desc* d, oxf_stream stream) {
  if (d && (!valid_act(d->act) || !valid_act(d->grad_act)))
    return set_error(OXF_ERR_INVALID_ARG, "oxf_gemm: bad activation");
  return gemm_run(d, S(stream));
}

oxf_status oxf_gemm_plan(const oxf_gemm_desc* d, int sm_count, oxf_gemm_plan_info* out) {
  if (d && (!valid_act(d->act) || !valid_act(d->grad_act)))
    return set_error(OXF_ERR_INVALID_ARG, "oxf_gemm_plan: bad activation");
  return gemm_plan_report(d, sm_count, out);
}

oxf_status oxf_gemm_tf32x3_noalloc(const oxf_gemm_desc* d, oxf_stream stream) {
  if (d && (!valid_act(d->act) || !valid_act(d->grad_act)))
    return set_error(OXF_ERR_INVALID_ARG, "oxf_gemm_tf32x3_noalloc: bad activation");
  return gemm_tf32x3_noalloc(d, S(stream));
}

size_t oxf_attention_stats_floats(int batch, int seq) {
  if (batch <= 0 || seq <= 0) return 0;
  return static_cast<size_t>(batch) * static_cast<size_t>(seq) *
         static_cast<size_t>(attention_stats_parts(seq)) * 2;
}

oxf_status oxf_attention_forward(const float* q, const float* k, const float* v,
                                 const float* residual, float* out, float* scores, float* stats,
                                 int batch, int seq, int d_qk, int d_v, float scale, int causal,
                                 oxf_stream stream) {
  return attention_forward(q, k, v, residual, out, scores, stats, batch, seq, d_qk, d_v, scale,
                           causal, S(stream));
}

oxf_status oxf_attention_heads_forward(const float* q, const float* k, const float* v,
                                       const float* residual, float* out, int batch, int seq,
                                       int d_qk, int d_v, int heads, int causal,
                                       oxf_stream stream) {
  return attention_heads_forward(q, k, v, residual, out, batch, seq, d_qk, d_v, heads, causal,
                                 S(stream));
}

oxf_status oxf_matrix_multiply(oxf_cslice lhs, oxf_cslice rhs, oxf_slice result, size_t len,
                               size_t rows, size_t cols, oxf_stream stream) {
  OXF_TRY(need(lhs.len >= rows * len && rhs.len >= len * cols && result.len >= rows * cols,
               "oxf_matrix_multiply: slice shorter than its shape"));
  if (rows > 0x7fffffffu || cols > 0x7fffffffu || len > 0x7fffffffu)
    return set_error(OXF_ERR_UNSUPPORTED_SHAPE, "oxf_matrix_multiply: dimension too large");
  oxf_gemm_desc d;
  oxf_gemm_desc_init(&d, static_cast<int>(rows), static_cast<int>(cols), static_cast<int>(len), 0,
                     0, lhs.ptr, rhs.ptr, result.ptr);
  return gemm_run(&d, S(stream));
}

oxf_status oxf_matrix_multiply_fp32(oxf_cslice lhs, oxf_cslice rhs, oxf_slice result,
                                    size_t len, size_t rows, size_t cols, oxf_stream stream) {
  OXF_TRY(need(lhs.len >= rows * len && rhs.len >= len * cols && result.len >= rows * cols,
               "oxf_matrix_multiply_fp32: slice shorter than its shape"));
  if (rows > 0x7fffffffu || cols > 0x7fffffffu || len > 0x7fffffffu)
    return set_error(OXF_ERR_UNSUPPORTED_SHAPE, "oxf_matrix_multiply_fp32: dimension too large");
  oxf_gemm_desc d;
  oxf_gemm_desc_init(&d, static_cast<int>(rows), static_cast<int>(cols), static_cast<int>(len), 0,
                     0, lhs.ptr, rhs.ptr, result.ptr);
  d.precision = OXF_PREC_F32;
  return gemm_run(&d, S(stream));
}

oxf_status oxf_matrix_multiply_refalgo(oxf_cslice lhs, oxf_cslice rhs, oxf_slice result,
                                       size_t len, size_t rows, size_t cols, oxf_stream stream) {
  OXF_TRY(need(lhs.len >= rows * len && rhs.len >= len * cols && result.len >= rows * cols,
               "oxf_matrix_multiply_refalgo: slice shorter than its shape"));
  return gemm_refalgo(lhs.ptr, rhs.ptr, result.ptr, len, rows, cols, S(stream));
}

}  // extern "C"
