// oxf_ffi.rs — the complete Rust FFI module for include/oxf.h and
// include/oxf_host.h, as a maintainer of the Rust reference would add it at
// src/cuda/oxf_ffi.rs. Every function of both headers and every structure they
// pass, in header order; the structures copy the C member order.
//
// Not compiled here: the image has no Rust toolchain. tests/test_abi.py keeps
// it in step with the headers (function names and parameter counts) and with
// the C structure layouts.
#![allow(non_camel_case_types, non_snake_case)]
use core::ffi::{c_char, c_int, c_void};

pub type oxf_status = c_int;      // OXF_OK = 0, OXF_ERR_* = 1..7
pub type oxf_stream = *mut c_void; // CUstream
pub type oxf_binary_op = c_int;   // OXF_ADD, OXF_SUB, OXF_MUL, OXF_DIV
pub type oxf_unary_op = c_int;    // OXF_UNARY_*
pub type oxf_activation = c_int;  // OXF_ACT_IDENTITY, _GELU, _RELU, _SILU
pub const OXF_EXCHANGE_MAX_RANKS: usize = 8;
pub const OXF_MAX_LAYERS: usize = 16;

#[repr(C)] #[derive(Clone, Copy)] pub struct oxf_cslice { pub ptr: *const f32, pub len: usize }
#[repr(C)] #[derive(Clone, Copy)] pub struct oxf_slice  { pub ptr: *mut f32,   pub len: usize }

#[repr(C)] #[derive(Clone, Copy)]
pub struct oxf_gemm_desc {
    pub M: c_int, pub N: c_int, pub K: c_int, pub batch: c_int,
    pub a_trans: c_int, pub b_trans: c_int,
    pub A: *const f32, pub lda: i64, pub stride_a: i64,
    pub B: *const f32, pub ldb: i64, pub stride_b: i64,
    pub C: *mut f32, pub ldc: i64, pub stride_c: i64,
    pub alpha: f32, pub beta: f32,
    pub bias: *const f32,
    pub residual: *const f32, pub ldr: i64, pub stride_r: i64,
    pub pre_out: *mut f32, pub ldp: i64, pub stride_p: i64,
    pub aux: *const f32, pub ldx: i64, pub stride_x: i64,
    pub act: c_int, pub grad_act: c_int, pub accumulate: c_int,
    pub split_k: c_int, pub precision: c_int,
    pub workspace: *mut c_void, pub workspace_bytes: usize,
    pub reduce_batch: c_int, pub variant: c_int,
}

#[repr(C)] #[derive(Clone, Copy)]
pub struct oxf_exchange_desc {
    pub rank: c_int, pub world: c_int,
    pub params: [*mut f32; OXF_EXCHANGE_MAX_RANKS],
    pub grads: [*const f32; OXF_EXCHANGE_MAX_RANKS],
    pub signals: [*mut u32; OXF_EXCHANGE_MAX_RANKS],
    pub epoch: u32, pub blocks: c_int, pub timeout_us: u32,
}

#[repr(C)] #[derive(Clone, Copy)] pub struct oxf_ipc_handle { pub handle: [u8; 64], pub offset: u64 }

pub const OXF_GEMM_PATH_NONE: c_int = 0;
pub const OXF_GEMM_PATH_SIMT: c_int = 1;
pub const OXF_GEMM_PATH_TINY: c_int = 2;
pub const OXF_GEMM_PATH_ONE_CTA: c_int = 3;
pub const OXF_GEMM_PATH_CTA_PAIR: c_int = 4;

#[repr(C)] #[derive(Clone, Copy)]
pub struct oxf_gemm_plan_info {
    pub path: c_int, pub tile_m: c_int, pub tile_n: c_int, pub stages: c_int,
    pub staging: c_int, pub splits: c_int, pub group_m: c_int, pub zero_c: c_int,
    pub units: i64,
}

#[repr(C)] #[derive(Clone, Copy)]
pub struct oxf_layer_spec { pub in_: c_int, pub out: c_int, pub act: c_int, pub bias: c_int }
#[repr(C)] #[derive(Clone, Copy)]
pub struct oxf_mlp_spec {
    pub n_layers: c_int, pub layers: [oxf_layer_spec; OXF_MAX_LAYERS],
    pub res_start: c_int, pub res_end: c_int,
}
#[repr(C)] #[derive(Clone, Copy)]
pub struct oxf_transformer_spec {
    pub seq: c_int, pub hidden: c_int, pub norm: c_int,
    pub q: oxf_layer_spec, pub k: oxf_layer_spec, pub v: oxf_layer_spec,
    pub ffn: oxf_mlp_spec, pub out: oxf_layer_spec,
}

// Engine and exchange handles (oxf_transformer, oxf_mlp, oxf_exchange) are opaque pointers.
#[link(name = "oxf")]
extern "C" {
    // include/oxf.h
    pub fn oxf_last_error_string() -> *const c_char;
    pub fn oxf_device_error(code: *mut u32) -> oxf_status;
    pub fn oxf_wait_timeout_selftest(limit_us: u32, expired: *mut c_int,
                                     stream: oxf_stream) -> oxf_status;
    pub fn oxf_version() -> *const c_char;
    pub fn oxf_kernel_launches() -> u64;
    pub fn oxf_slice_binary(lhs: oxf_cslice, rhs: oxf_cslice, out: oxf_slice, op: oxf_binary_op,
                            stream: oxf_stream) -> oxf_status;
    pub fn oxf_slice_binary_assign(target: oxf_slice, rhs: oxf_cslice, op: oxf_binary_op,
                                   stream: oxf_stream) -> oxf_status;
    pub fn oxf_slice_unary(span: oxf_slice, op: oxf_unary_op, param: f32,
                           stream: oxf_stream) -> oxf_status;
    pub fn oxf_sgd_update(target: oxf_slice, grad: oxf_cslice, lr: f32,
                          stream: oxf_stream) -> oxf_status;
    pub fn oxf_mse_grad(y: oxf_cslice, target: oxf_cslice, out: oxf_slice, cols: usize,
                        stream: oxf_stream) -> oxf_status;
    pub fn oxf_mse_loss_grad(y: oxf_cslice, target: oxf_cslice, row_loss: oxf_slice,
                             dy: oxf_slice, cols: usize, stream: oxf_stream) -> oxf_status;
    pub fn oxf_loss_rows(y: oxf_cslice, target: oxf_cslice, row_loss: oxf_slice, cols: usize,
                         stream: oxf_stream) -> oxf_status;
    pub fn oxf_slice_sum(span: oxf_cslice, result: *mut f32, stream: oxf_stream) -> oxf_status;
    pub fn oxf_slice_max(span: oxf_cslice, result: *mut f32, stream: oxf_stream) -> oxf_status;
    pub fn oxf_slice_map_sum(span: oxf_cslice, op: oxf_unary_op, param: f32, result: *mut f32,
                             stream: oxf_stream) -> oxf_status;
    pub fn oxf_slice_dot(lhs: oxf_cslice, rhs: oxf_cslice, result: *mut f32,
                         stream: oxf_stream) -> oxf_status;
    pub fn oxf_slice_set(target: oxf_slice, value: f32, stream: oxf_stream) -> oxf_status;
    pub fn oxf_slice_set_seq(target: oxf_slice, dir: c_int, stream: oxf_stream) -> oxf_status;
    pub fn oxf_slice_set_random(target: oxf_slice, seed: u32, stream: oxf_stream) -> oxf_status;
    pub fn oxf_matrix_sum_rows(matrix: oxf_cslice, result: oxf_slice, cols: usize,
                               stream: oxf_stream) -> oxf_status;
    pub fn oxf_matrix_sum_cols(matrix: oxf_cslice, result: oxf_slice, cols: usize,
                               accumulate: c_int, stream: oxf_stream) -> oxf_status;
    pub fn oxf_matrix_softmax_rows(matrix: oxf_slice, cols: usize, scale: f32,
                                   causal_period: usize, stream: oxf_stream) -> oxf_status;
    pub fn oxf_matrix_layer_norm_rows(matrix: oxf_slice, cols: usize, epsilon: f32,
                                      gamma: *const f32, beta: *const f32,
                                      stream: oxf_stream) -> oxf_status;
    pub fn oxf_rms_norm_assign(matrix: oxf_slice, cols: usize, epsilon: f32, gamma: *const f32,
                               stream: oxf_stream) -> oxf_status;
    pub fn oxf_norm_rows(input: oxf_cslice, output: oxf_slice, cols: usize, norm_type: c_int,
                         epsilon: f32, gamma: *const f32, beta: *const f32,
                         stream: oxf_stream) -> oxf_status;
    pub fn oxf_norm_rows_backward(input: oxf_cslice, output_gradient: oxf_cslice,
                                  result: oxf_slice, cols: usize, norm_type: c_int, epsilon: f32,
                                  stream: oxf_stream) -> oxf_status;
    pub fn oxf_slice_binary_broadcast(lhs: oxf_cslice, rhs: oxf_cslice, out: oxf_slice,
                                      op: oxf_binary_op, stream: oxf_stream) -> oxf_status;
    pub fn oxf_slice_mul_act_derivative(gradient: oxf_slice, pre_activation: oxf_cslice,
                                        act: oxf_activation, stream: oxf_stream) -> oxf_status;
    pub fn oxf_softmax_rows_backward(probabilities: oxf_cslice, output_gradient: oxf_cslice,
                                     result: oxf_slice, cols: usize, scale: f32,
                                     stream: oxf_stream) -> oxf_status;
    pub fn oxf_layer_norm_backward(input: oxf_cslice, output_gradient: oxf_cslice,
                                   result: oxf_slice, cols: usize, epsilon: f32,
                                   stream: oxf_stream) -> oxf_status;
    pub fn oxf_matrix_rms_norm_backward(input: oxf_cslice, output_gradient: oxf_cslice,
                                        result: oxf_slice, cols: usize, epsilon: f32,
                                        stream: oxf_stream) -> oxf_status;
    pub fn oxf_matrix_binary_assign_by_rows(matrix: oxf_slice, row: oxf_cslice, cols: usize,
                                            op: oxf_binary_op, stream: oxf_stream) -> oxf_status;
    pub fn oxf_matrix_causal_mask(matrix: oxf_slice, cols: usize, stream: oxf_stream) -> oxf_status;
    pub fn oxf_matrix_slice(input: oxf_cslice, output: oxf_slice, input_cols: usize,
                            tile_rows: usize, tile_cols: usize, tiles_per_row: usize,
                            stream: oxf_stream) -> oxf_status;
    pub fn oxf_matrix_transpose(input: oxf_cslice, result: oxf_slice, rows: usize, cols: usize,
                                stream: oxf_stream) -> oxf_status;
    pub fn oxf_gemm_desc_init(d: *mut oxf_gemm_desc, M: c_int, N: c_int, K: c_int,
                              a_trans: c_int, b_trans: c_int, A: *const f32, B: *const f32,
                              C: *mut f32);
    pub fn oxf_gemm_workspace_size(d: *const oxf_gemm_desc) -> usize;
    pub fn oxf_gemm(d: *const oxf_gemm_desc, stream: oxf_stream) -> oxf_status;
    pub fn oxf_gemm_plan(d: *const oxf_gemm_desc, sm_count: c_int,
                         out: *mut oxf_gemm_plan_info) -> oxf_status;
    pub fn oxf_gemm_tf32x3_noalloc(desc: *const oxf_gemm_desc, stream: oxf_stream) -> oxf_status;
    pub fn oxf_attention_stats_floats(batch: c_int, seq: c_int) -> usize;
    pub fn oxf_attention_forward(q: *const f32, k: *const f32, v: *const f32,
                                 residual: *const f32, out: *mut f32, scores: *mut f32,
                                 stats: *mut f32, batch: c_int, seq: c_int, d_qk: c_int,
                                 d_v: c_int, scale: f32, causal: c_int, stream: oxf_stream)
                                 -> oxf_status;
    pub fn oxf_attention_heads_forward(q: *const f32, k: *const f32, v: *const f32,
                                       residual: *const f32, out: *mut f32, batch: c_int,
                                       seq: c_int, d_qk: c_int, d_v: c_int, heads: c_int,
                                       causal: c_int, stream: oxf_stream) -> oxf_status;
    pub fn oxf_matrix_multiply(lhs: oxf_cslice, rhs: oxf_cslice, result: oxf_slice, len: usize,
                               rows: usize, cols: usize, stream: oxf_stream) -> oxf_status;
    pub fn oxf_matrix_multiply_fp32(lhs: oxf_cslice, rhs: oxf_cslice, result: oxf_slice,
                                    len: usize, rows: usize, cols: usize,
                                    stream: oxf_stream) -> oxf_status;
    pub fn oxf_matrix_multiply_refalgo(lhs: oxf_cslice, rhs: oxf_cslice, result: oxf_slice,
                                       len: usize, rows: usize, cols: usize,
                                       stream: oxf_stream) -> oxf_status;
    pub fn oxf_exchange_sgd(desc: *const oxf_exchange_desc, offset: usize, count: usize, lr: f32,
                            stream: oxf_stream) -> oxf_status;
    pub fn oxf_ipc_export(ptr: *const c_void, out: *mut oxf_ipc_handle) -> oxf_status;
    pub fn oxf_ipc_open(handle: *const oxf_ipc_handle, ptr: *mut *mut c_void) -> oxf_status;
    pub fn oxf_ipc_close(handle: *const oxf_ipc_handle, ptr: *mut c_void) -> oxf_status;
    // include/oxf_host.h
    pub fn oxf_transformer_create(spec: *const oxf_transformer_spec, max_batch: c_int,
                                  stream: oxf_stream, out: *mut *mut c_void) -> oxf_status;
    pub fn oxf_transformer_destroy(t: *mut c_void) -> oxf_status;
    pub fn oxf_transformer_param_count(t: *mut c_void) -> usize;
    pub fn oxf_transformer_params(t: *mut c_void) -> *mut f32;
    pub fn oxf_transformer_grads(t: *mut c_void) -> *mut f32;
    pub fn oxf_transformer_stream(t: *mut c_void) -> oxf_stream;
    pub fn oxf_transformer_set_params_host(t: *mut c_void, params_host: *const f32) -> oxf_status;
    pub fn oxf_transformer_get_params_host(t: *mut c_void, params_host: *mut f32) -> oxf_status;
    pub fn oxf_transformer_forward(t: *mut c_void, x: *const f32, batch: c_int, causal: c_int,
                                   y: *mut f32) -> oxf_status;
    pub fn oxf_transformer_train_forward(t: *mut c_void, x: *const f32, batch: c_int) -> oxf_status;
    pub fn oxf_transformer_set_target(t: *mut c_void, target: *const f32) -> oxf_status;
    pub fn oxf_transformer_set_output_gradient(t: *mut c_void, dy: *const f32) -> oxf_status;
    pub fn oxf_transformer_backward_stage(t: *mut c_void, stage: c_int) -> oxf_status;
    pub fn oxf_transformer_bucket(t: *mut c_void, stage: c_int, offset: *mut usize,
                                  count: *mut usize) -> oxf_status;
    pub fn oxf_transformer_zero_grads(t: *mut c_void) -> oxf_status;
    pub fn oxf_transformer_sgd(t: *mut c_void, lr: f32) -> oxf_status;
    pub fn oxf_transformer_set_heads(t: *mut c_void, heads: c_int) -> oxf_status;
    pub fn oxf_transformer_heads(t: *mut c_void) -> c_int;
    pub fn oxf_transformer_output(t: *mut c_void, y: *mut *const f32, row_loss: *mut *const f32,
                                  input_gradient: *mut *const f32) -> oxf_status;
    pub fn oxf_transformer_set_timing(t: *mut c_void, on: c_int) -> oxf_status;
    pub fn oxf_transformer_read_timing(t: *mut c_void, gemm_ms: *mut f64, gemm_flops: *mut f64,
                                       launches: *mut c_int) -> oxf_status;
    pub fn oxf_transformer_train_step_host(t: *mut c_void, x_host: *const f32,
                                           target_host: *const f32, batch: c_int, lr: f32,
                                           mean_loss_host: *mut f32) -> oxf_status;
    pub fn oxf_mlp_create(spec: *const oxf_mlp_spec, max_rows: usize, stream: oxf_stream,
                          out: *mut *mut c_void) -> oxf_status;
    pub fn oxf_mlp_destroy(m: *mut c_void) -> oxf_status;
    pub fn oxf_mlp_param_count(m: *mut c_void) -> usize;
    pub fn oxf_mlp_params(m: *mut c_void) -> *mut f32;
    pub fn oxf_mlp_grads(m: *mut c_void) -> *mut f32;
    pub fn oxf_mlp_forward(m: *mut c_void, x: *const f32, y: *mut f32, rows: usize) -> oxf_status;
    pub fn oxf_mlp_backward(m: *mut c_void, dy: *const f32, dx: *mut f32,
                            rows: usize) -> oxf_status;
    pub fn oxf_mlp_zero_grads(m: *mut c_void) -> oxf_status;
    pub fn oxf_mlp_sgd(m: *mut c_void, lr: f32) -> oxf_status;
    pub fn oxf_runtime_create(device: c_int, stream: oxf_stream, out: *mut *mut c_void)
                              -> oxf_status;
    pub fn oxf_runtime_destroy(rt: *mut c_void) -> oxf_status;
    pub fn oxf_runtime_stream(rt: *mut c_void) -> oxf_stream;
    pub fn oxf_runtime_sync(rt: *mut c_void) -> oxf_status;
    pub fn oxf_runtime_reserve_buffers(rt: *mut c_void, len: usize, count: usize) -> oxf_status;
    pub fn oxf_runtime_pooled_buffers(rt: *mut c_void, count: *mut usize) -> oxf_status;
    pub fn oxf_linear_create(rt: *mut c_void, spec: *const oxf_layer_spec,
                             weights_host: *const f32, bias_host: *const f32,
                             out: *mut *mut c_void) -> oxf_status;
    pub fn oxf_linear_destroy(l: *mut c_void) -> oxf_status;
    pub fn oxf_linear_params(l: *mut c_void, weights: *mut *mut f32, bias: *mut *mut f32)
                             -> oxf_status;
    pub fn oxf_linear_forward(l: *mut c_void, x: *const f32, rows: usize, residual: *const f32,
                              y: *mut f32, pre_activation: *mut f32, stream: oxf_stream)
                              -> oxf_status;
    pub fn oxf_linear_backward(l: *mut c_void, pre_activation: *const f32,
                               output_gradient: *const f32, residual_gradient: *const f32,
                               rows: usize, gradient: *mut f32, bias_gradient: *mut f32,
                               stream: oxf_stream) -> oxf_status;
    pub fn oxf_linear_learn(l: *mut c_void, x: *const f32, gradient: *const f32,
                            bias_gradient: *const f32, rows: usize, learning_rate: f32,
                            stream: oxf_stream) -> oxf_status;
    pub fn oxf_linear_input_gradient(l: *mut c_void, gradient: *const f32, rows: usize,
                                     dx: *mut f32, stream: oxf_stream) -> oxf_status;
    pub fn oxf_checkpoint_write_linear(path: *const c_char, spec: *const oxf_layer_spec,
                                       params_host: *const f32, count: usize) -> oxf_status;
    pub fn oxf_checkpoint_write_mlp(path: *const c_char, spec: *const oxf_mlp_spec,
                                    params_host: *const f32, count: usize) -> oxf_status;
    pub fn oxf_checkpoint_write_transformer(path: *const c_char,
                                            spec: *const oxf_transformer_spec,
                                            params_host: *const f32, count: usize) -> oxf_status;
    pub fn oxf_checkpoint_read_linear(path: *const c_char, spec: *mut oxf_layer_spec,
                                      params_host: *mut f32, capacity: usize,
                                      count: *mut usize) -> oxf_status;
    pub fn oxf_checkpoint_read_mlp(path: *const c_char, spec: *mut oxf_mlp_spec,
                                   params_host: *mut f32, capacity: usize,
                                   count: *mut usize) -> oxf_status;
    pub fn oxf_checkpoint_read_transformer(path: *const c_char, spec: *mut oxf_transformer_spec,
                                           params_host: *mut f32, capacity: usize,
                                           count: *mut usize) -> oxf_status;
    pub fn oxf_transformer_dump(t: *mut c_void, path: *const c_char) -> oxf_status;
    pub fn oxf_transformer_load(path: *const c_char, max_batch: c_int, stream: oxf_stream,
                                out: *mut *mut c_void) -> oxf_status;
    pub fn oxf_mlp_dump(m: *mut c_void, path: *const c_char) -> oxf_status;
    pub fn oxf_mlp_load(path: *const c_char, max_rows: usize, stream: oxf_stream,
                        out: *mut *mut c_void) -> oxf_status;
    pub fn oxf_exchange_create(rank: c_int, world: c_int, params: *mut f32, grads: *mut f32,
                               count: usize, out: *mut *mut c_void) -> oxf_status;
    pub fn oxf_exchange_handles(ex: *mut c_void, out: *mut oxf_ipc_handle) -> oxf_status;
    pub fn oxf_exchange_connect(ex: *mut c_void, all: *const oxf_ipc_handle) -> oxf_status;
    pub fn oxf_exchange_step(ex: *mut c_void, offset: usize, count: usize, lr: f32,
                             blocks: c_int, stream: oxf_stream) -> oxf_status;
    pub fn oxf_exchange_set_timeout(ex: *mut c_void, timeout_us: u32) -> oxf_status;
    pub fn oxf_exchange_destroy(ex: *mut c_void) -> oxf_status;
}
