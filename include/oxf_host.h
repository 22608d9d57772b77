/*
 * oxf_host.h — C ABI of the host executors (the batched MLP and transformer
 * engines of oxide-forge_b200/host/engine.hpp).
 *
 * These replace the reference's executor layer for the hot path:
 *   InferenceTransformer / TrainingTransformer (src/net/transformer/
 *   encoder.rs:37-187, decoder.rs:7-53, inference.rs:76-109),
 *   Attention (src/net/transformer/attention.rs:177-402),
 *   MlpExecutor / InferenceMLP / TrainingMlp (src/net/mlp.rs:14-269),
 *   Linear (src/net/linear.rs:72-533).
 * The reference drives one [seq, hidden] sequence per call; these drive
 * `batch` independent sequences (or rows) per call with the same
 * arithmetic. Parameters and gradients are flat f32 device arenas in
 * checkpoint cursor order (inference.rs:52-66, metadata.rs:21-68): per
 * Linear the weight [in, out] row-major, then its bias; for the transformer
 * q, k, v, position [seq, hidden], the feed-forward layers, the output.
 * Device pointers unless a name ends in _host. Same error conventions as
 * oxf.h.
 */
#ifndef OXF_HOST_H
#define OXF_HOST_H

#include "oxf.h"

#ifdef __cplusplus
extern "C" {
#endif

/* One Linear layer (linear.rs:72-86): weights [in,out], optional bias. */
typedef struct {
  int in, out;
  int act;  /* oxf_activation */
  int bias; /* 0/1 */
} oxf_layer_spec;

#define OXF_MAX_LAYERS 16

/* MlpExecutor (mlp.rs:14-19). res_start/res_end = -1: no residual. */
typedef struct {
  int n_layers;
  oxf_layer_spec layers[OXF_MAX_LAYERS];
  int res_start, res_end;
} oxf_mlp_spec;

/* Single-block Post-Norm transformer (TransformerMetadata,
 * inference.rs:12-24). */
typedef struct {
  int seq, hidden;
  int norm; /* oxf_norm_type */
  oxf_layer_spec q, k, v;
  oxf_mlp_spec ffn;
  oxf_layer_spec out;
} oxf_transformer_spec;

typedef struct oxf_transformer_s* oxf_transformer;
typedef struct oxf_mlp_s* oxf_mlp;

/* ---------------------------------------------------------------- transformer */
/* Builds an engine for up to max_batch sequences on the current device;
 * all its work runs on `stream` (NULL: the legacy default stream).
 * Parameters start at zero. */
oxf_status oxf_transformer_create(const oxf_transformer_spec* spec, int max_batch,
                                  oxf_stream stream, oxf_transformer* out);
oxf_status oxf_transformer_destroy(oxf_transformer t);
size_t oxf_transformer_param_count(oxf_transformer t);
/* Device arenas (param_count floats each), cursor order. */
float* oxf_transformer_params(oxf_transformer t);
float* oxf_transformer_grads(oxf_transformer t);
oxf_stream oxf_transformer_stream(oxf_transformer t);
/* Host <-> device copies of the parameter arena (synchronous). */
oxf_status oxf_transformer_set_params_host(oxf_transformer t, const float* params_host);
oxf_status oxf_transformer_get_params_host(oxf_transformer t, float* params_host);

/* InferenceTransformer::forward (encoder.rs:55-57) or the decoder's masked
 * forward (decoder.rs:50-52, causal = 1): x [batch*seq, hidden] ->
 * y [batch*seq, out] (y may be NULL: read it with oxf_transformer_output). */
oxf_status oxf_transformer_forward(oxf_transformer t, const float* x, int batch, int causal,
                                   float* y);
/* TrainingTransformer::forward (encoder.rs:114-133). */
oxf_status oxf_transformer_train_forward(oxf_transformer t, const float* x, int batch);
/* Per-row loss (Linear::loss_rows, linear.rs:325-333) and dL/dy =
 * (y - target)/out against `target` [batch*seq, out]. */
oxf_status oxf_transformer_set_target(oxf_transformer t, const float* target);
/* Or a caller-computed dL/dy [batch*seq, out]. */
oxf_status oxf_transformer_set_output_gradient(oxf_transformer t, const float* dy);
/* TrainingTransformer::backward (encoder.rs:135-186) in stages 0 (output
 * Linear), 1 (feed-forward), 2 (attention, Q/K/V, position). Parameter
 * gradients ACCUMULATE into the gradient arena; nothing is updated. Needs
 * oxf_transformer_train_forward as the last forward: the inference forward
 * keeps neither probabilities nor pre-activations (OXF_ERR_INVALID_ARG). */
oxf_status oxf_transformer_backward_stage(oxf_transformer t, int stage);
/* [offset, offset+count) of the gradient arena that stage writes. */
oxf_status oxf_transformer_bucket(oxf_transformer t, int stage, size_t* offset, size_t* count);
oxf_status oxf_transformer_zero_grads(oxf_transformer t);
/* params -= lr * grads (the reference's per-Linear SGD, linear.rs:373-391,
 * and position update, encoder.rs:180-184, applied once). */
oxf_status oxf_transformer_sgd(oxf_transformer t, float lr);
/* Attention heads (default 1: the reference's single-head attention,
 * attention.rs:359-401). Head j attends over columns [j*D/h, (j+1)*D/h) of Q
 * and K and [j*H/h, (j+1)*H/h) of V with scale 1/sqrt(D/h) and writes those
 * columns of the attention output; the projections and all other layers
 * are unchanged (the multi-head path docs/api.md:440-442 anticipates). h
 * must divide the query width D and hidden H (INVALID_ARG otherwise). Takes
 * effect from the next forward. Inference runs the fused kernel
 * (oxf_attention_heads_forward) where it applies and keeps no scores; the
 * first training step, or inference the kernel cannot take, allocates score
 * buffers of h per sequence (after synchronising the engine's stream).
 * The checkpoint format has no head count: a loaded engine has one head. */
oxf_status oxf_transformer_set_heads(oxf_transformer t, int heads);
int oxf_transformer_heads(oxf_transformer t);
/* Device views of the last output [batch*seq, out], per-row loss
 * [batch*seq] and input gradient [batch*seq, hidden]. */
oxf_status oxf_transformer_output(oxf_transformer t, const float** y, const float** row_loss,
                                  const float** input_gradient);
/* GEMM timing: while on, CUDA events bracket every GEMM the engine
 * launches; read returns the summed device time (ms), summed algorithmic
 * flops (2*M*N*K per product) and launch count since the last read, and
 * resets them. Synchronises on the recorded events. */
oxf_status oxf_transformer_set_timing(oxf_transformer t, int on);
oxf_status oxf_transformer_read_timing(oxf_transformer t, double* gemm_ms, double* gemm_flops,
                                       int* launches);
/* One data-parallel-free training step through host memory: copies x and
 * target from the host, runs forward, loss, backward, and SGD on the mean
 * gradient (lr / batch), and returns the mean row loss. */
oxf_status oxf_transformer_train_step_host(oxf_transformer t, const float* x_host,
                                           const float* target_host, int batch, float lr,
                                           float* mean_loss_host);

/* ---------------------------------------------------------------- MLP */
oxf_status oxf_mlp_create(const oxf_mlp_spec* spec, size_t max_rows, oxf_stream stream,
                          oxf_mlp* out);
oxf_status oxf_mlp_destroy(oxf_mlp m);
size_t oxf_mlp_param_count(oxf_mlp m);
float* oxf_mlp_params(oxf_mlp m);
float* oxf_mlp_grads(oxf_mlp m);
/* MlpExecutor::forward (mlp.rs:53-85): y [rows, out] = MLP(x [rows, in]).
 * x must stay valid until oxf_mlp_backward. */
oxf_status oxf_mlp_forward(oxf_mlp m, const float* x, float* y, size_t rows);
/* MlpExecutor::backward (mlp.rs:121-168) without the update: accumulates
 * parameter gradients, writes dx [rows, in] (may be NULL). */
oxf_status oxf_mlp_backward(oxf_mlp m, const float* dy, float* dx, size_t rows);
oxf_status oxf_mlp_zero_grads(oxf_mlp m);
oxf_status oxf_mlp_sgd(oxf_mlp m, float lr);

/* ---------------------------------------------------------------- runtime + Linear */
/* CudaRuntime (src/cuda/runtime.rs:24-212): a device, its primary stream
 * and an exact-size pool of device buffers (runtime.rs:47-110) from which
 * the Linear below takes its parameters. stream NULL: the runtime creates
 * its own non-blocking primary stream (the reference creates one per
 * runtime, runtime.rs:34-45); otherwise it borrows `stream`. */
typedef struct oxf_runtime_s* oxf_runtime;
oxf_status oxf_runtime_create(int device, oxf_stream stream, oxf_runtime* out);
/* Synchronises, then frees the pool and the streams the runtime created. */
oxf_status oxf_runtime_destroy(oxf_runtime rt);
oxf_stream oxf_runtime_stream(oxf_runtime rt);
/* CudaRuntime::sync (runtime.rs:112-114). */
oxf_status oxf_runtime_sync(oxf_runtime rt);
/* CudaRuntime::reserve_buffers (runtime.rs:75-91): at least `count` free
 * pooled buffers of `len` floats. */
oxf_status oxf_runtime_reserve_buffers(oxf_runtime rt, size_t len, size_t count);
/* Free buffers held by the pool, all lengths. */
oxf_status oxf_runtime_pooled_buffers(oxf_runtime rt, size_t* count);

/* Linear (src/net/linear.rs:72-533): weights [in, out] row-major, a bias
 * [out] when spec->bias, spec->act. The parameters live in the runtime's
 * pool buffers, copied from host memory at creation (Linear::new,
 * linear.rs:89-95, after matrix_from_host). The layer belongs to the
 * runtime: destroy it before the runtime. Every call takes device pointers
 * of rows x (in or out) matrices and runs on `stream`: NULL is the
 * runtime's primary stream; another stream first waits for the primary
 * stream (the reference's stream.join(runtime.stream())). */
typedef struct oxf_linear_s* oxf_linear;
oxf_status oxf_linear_create(oxf_runtime rt, const oxf_layer_spec* spec, const float* weights_host,
                             const float* bias_host, oxf_linear* out);
oxf_status oxf_linear_destroy(oxf_linear l);
/* Device pointers of the weights [in, out] and the bias [out] (NULL without
 * a bias); updated in place by oxf_linear_learn. */
oxf_status oxf_linear_params(oxf_linear l, float** weights, float** bias);
/* Linear::forward (linear.rs:116-132, 185-230): y = act(x·W + b +
 * residual), in that order, as one GEMM with a fused epilogue. residual
 * (rows x out) may be NULL; pre_activation (rows x out, may be NULL)
 * receives x·W + b + residual, which Linear::backward needs. */
oxf_status oxf_linear_forward(oxf_linear l, const float* x, size_t rows, const float* residual,
                              float* y, float* pre_activation, oxf_stream stream);
/* Linear::backward / backward_with_res (linear.rs:232-306, 446-533):
 * gradient = (output_gradient [+ residual_gradient]) ⊙ act'(pre_activation)
 * and, for a biased layer, bias_gradient = its column sums (NULL
 * pre_activation only for Identity; residual_gradient may be NULL). */
oxf_status oxf_linear_backward(oxf_linear l, const float* pre_activation,
                               const float* output_gradient, const float* residual_gradient,
                               size_t rows, float* gradient, float* bias_gradient,
                               oxf_stream stream);
/* Linear::learn (linear.rs:350-415): W -= lr·xᵀ·gradient, b -= lr·bias_gradient
 * (bias_gradient required for a biased layer). */
oxf_status oxf_linear_learn(oxf_linear l, const float* x, const float* gradient,
                            const float* bias_gradient, size_t rows, float learning_rate,
                            oxf_stream stream);
/* Linear::input_gradient (linear.rs:417-446): dx [rows, in] = gradient·Wᵀ. */
oxf_status oxf_linear_input_gradient(oxf_linear l, const float* gradient, size_t rows,
                                     float* dx, oxf_stream stream);

/* ---------------------------------------------------------------- checkpoints (v1) */
/* The reference's checkpoint format (src/net/checkpoint/model.rs:17-21,
 * io.rs:14-181): <name>.toml holds format_version = 1, model_type
 * ("linear" | "mlp" | "transformer"), scalar_type = "f32_le", data_file,
 * data_bytes and the model's metadata (Linear neuron counts, activation,
 * weight/bias shapes and [byte_start, byte_end) ranges; MLP layer_count,
 * loss, residual; transformer block_count, residual flags, normalization,
 * position); <name>.bin holds the parameters as little-endian f32 in cursor
 * order. `path` without an extension gets ".toml"; any extension other
 * than .toml is refused (io.rs:20-29). Loading validates what the
 * reference validates (model.rs:350-537): version, model type, scalar
 * encoding, contiguous ranges, shapes, Linear connectivity, residual and
 * transformer dimensions, and the data file's size.
 *
 * Host-array forms (no GPU needed); parameters in cursor order: */
/* dump_linear / dump_mlp / dump_transformer with the parameters given. */
oxf_status oxf_checkpoint_write_linear(const char* path, const oxf_layer_spec* spec,
                                       const float* params_host, size_t count);
oxf_status oxf_checkpoint_write_mlp(const char* path, const oxf_mlp_spec* spec,
                                    const float* params_host, size_t count);
oxf_status oxf_checkpoint_write_transformer(const char* path, const oxf_transformer_spec* spec,
                                            const float* params_host, size_t count);
/* load_*: validates, fills *spec (may be NULL) and *count, and copies the
 * parameters when params_host != NULL (capacity >= *count). */
oxf_status oxf_checkpoint_read_linear(const char* path, oxf_layer_spec* spec, float* params_host,
                                      size_t capacity, size_t* count);
oxf_status oxf_checkpoint_read_mlp(const char* path, oxf_mlp_spec* spec, float* params_host,
                                   size_t capacity, size_t* count);
oxf_status oxf_checkpoint_read_transformer(const char* path, oxf_transformer_spec* spec,
                                           float* params_host, size_t capacity, size_t* count);
/* Engine forms: dump_transformer / load_transformer and dump_mlp / load_mlp
 * (model.rs:78-208) on an engine's parameter arena. Loading creates the
 * engine (as oxf_*_create) with the checkpoint's parameters. */
oxf_status oxf_transformer_dump(oxf_transformer t, const char* path);
oxf_status oxf_transformer_load(const char* path, int max_batch, oxf_stream stream,
                                oxf_transformer* out);
oxf_status oxf_mlp_dump(oxf_mlp m, const char* path);
oxf_status oxf_mlp_load(const char* path, size_t max_rows, oxf_stream stream, oxf_mlp* out);

/* ---------------------------------------------------------------- peer exchange */
/* One rank's side of the fused gradient exchange + SGD (oxf_exchange_sgd in
 * oxf.h) over a parameter and a gradient arena of `count` floats each,
 * e.g. oxf_transformer_params / _grads. Usage, on every rank of one node
 * (one process per GPU): create; send the three handles of
 * oxf_exchange_handles to every rank (any host transport); connect with all
 * ranks' handles; then oxf_exchange_step once per gradient bucket, in the
 * same order on every rank. No reference counterpart (single-GPU
 * reference, src/cuda/runtime.rs:34-45). */
typedef struct oxf_exchange_s* oxf_exchange;

/* Allocates and zeroes this rank's signal pad on the current device. */
oxf_status oxf_exchange_create(int rank, int world, float* params, float* grads, size_t count,
                               oxf_exchange* out);
/* This rank's handles: out[0] params, out[1] grads, out[2] signal pad. */
oxf_status oxf_exchange_handles(oxf_exchange ex, oxf_ipc_handle out[3]);
/* Maps every other rank's memory: all[3*q + 0..2] are rank q's handles
 * (this rank's entries are not opened). Once per exchange. */
oxf_status oxf_exchange_connect(oxf_exchange ex, const oxf_ipc_handle* all);
/* oxf_exchange_sgd over [offset, offset + count) of the arenas with the
 * next epoch; blocks = CTAs per rank (0: one per SM), equal on all ranks. */
oxf_status oxf_exchange_step(oxf_exchange ex, size_t offset, size_t count, float lr, int blocks,
                             oxf_stream stream);
/* Bound of each barrier wait in later steps (0: 4 s). */
oxf_status oxf_exchange_set_timeout(oxf_exchange ex, uint32_t timeout_us);
/* Unmaps the peers' memory and frees the pad. Every rank must have finished
 * its last step first (synchronise, then a host barrier). */
oxf_status oxf_exchange_destroy(oxf_exchange ex);

#ifdef __cplusplus
}
#endif
#endif
