// host_abi.cpp — extern "C" entry points of include/oxf_host.h over the
// C++ engines (engine.hpp). Exceptions never cross the ABI: they become an
// oxf_status plus oxf_last_error_string().
#include <cuda_runtime.h>

#include <algorithm>
#include <exception>
#include <new>
#include <vector>

#include "checkpoint.hpp"
#include "engine.hpp"
#include "errors.hpp"
#include "linear.hpp"
#include "oxf_host.h"

struct oxf_transformer_s {
  oxf_transformer_spec spec{};  // as created (checkpoint metadata)
  oxf::TransformerEngine* engine = nullptr;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  float* x_dev = nullptr;  // staging for the host-memory training step
  float* t_dev = nullptr;
  float* loss_dev = nullptr;
};

struct oxf_runtime_s {
  oxf::CudaRuntime* rt = nullptr;
};

struct oxf_linear_s {
  oxf::CudaRuntime* rt = nullptr;
  oxf::Linear* layer = nullptr;
};

struct oxf_mlp_s {
  oxf_mlp_spec spec{};  // as created (checkpoint metadata)
  oxf::MlpEngine* engine = nullptr;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  float* params = nullptr;
  float* grads = nullptr;
  size_t nparams = 0;
};

namespace {

template <typename F>
oxf_status guard(F&& f) {
  try {
    f();
    return OXF_OK;
  } catch (const oxf::Error& e) {
    return oxf::set_error(e.status, "%s", e.what());
  } catch (const std::bad_alloc&) {
    return oxf::set_error(OXF_ERR_CUDA, "out of host memory");
  } catch (const std::exception& e) {
    return oxf::set_error(OXF_ERR_STATE, "%s", e.what());
  }
}

oxf::LayerSpec layer(const oxf_layer_spec& l) {
  oxf::LayerSpec s;
  s.in = l.in;
  s.out = l.out;
  s.act = l.act;
  s.bias = l.bias != 0;
  oxf::require(l.in > 0 && l.out > 0, "layer widths must be positive");
  oxf::require(l.act >= OXF_ACT_IDENTITY && l.act <= OXF_ACT_SILU, "bad activation");
  return s;
}

oxf::MlpSpec mlp_spec(const oxf_mlp_spec& m) {
  oxf::require(m.n_layers >= 1 && m.n_layers <= OXF_MAX_LAYERS, "MLP layer count");
  oxf::MlpSpec s;
  for (int i = 0; i < m.n_layers; ++i) s.layers.push_back(layer(m.layers[i]));
  s.res_start = m.res_start;
  s.res_end = m.res_end;
  return s;
}

// NULL selects the legacy default stream, as everywhere in oxf.h; the
// engines never create streams of their own.
cudaStream_t make_stream(oxf_stream given, bool* own) {
  *own = false;
  return reinterpret_cast<cudaStream_t>(given);
}

}  // namespace

// Checkpoint entry points: copy between a checkpoint and host arrays.
namespace {

template <typename Spec>
oxf_status write_ckpt(const char* path, oxf::ckpt::ModelType type, const Spec* spec,
                      const float* params_host, size_t count,
                      void (*put)(oxf::ckpt::Model&, const Spec&)) {
  if (!path || !spec || (!params_host && count)) {
    return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  }
  return guard([&] {
    oxf::ckpt::Model m;
    m.type = type;
    put(m, *spec);
    m.params.assign(params_host, params_host + count);
    oxf::ckpt::write(path, m);
  });
}

template <typename Spec>
oxf_status read_ckpt(const char* path, oxf::ckpt::ModelType type, Spec* spec, float* params_host,
                     size_t capacity, size_t* count, Spec (*get)(const oxf::ckpt::Model&)) {
  if (!path || !count) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] {
    const oxf::ckpt::Model m = oxf::ckpt::read(path, type);
    *count = m.params.size();
    if (spec) *spec = get(m);
    if (params_host) {
      oxf::require(capacity >= m.params.size(), "parameter buffer smaller than the checkpoint");
      std::copy(m.params.begin(), m.params.end(), params_host);
    }
  });
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------- transformer
oxf_status oxf_transformer_create(const oxf_transformer_spec* spec, int max_batch,
                                  oxf_stream stream, oxf_transformer* out) {
  if (!spec || !out) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  return guard([&] {
    oxf::TransformerSpec s;
    s.seq = spec->seq;
    s.hidden = spec->hidden;
    s.norm = spec->norm;
    s.q = layer(spec->q);
    s.k = layer(spec->k);
    s.v = layer(spec->v);
    s.ffn = mlp_spec(spec->ffn);
    s.o = layer(spec->out);
    auto* h = new oxf_transformer_s();
    h->spec = *spec;
    try {
      h->stream = make_stream(stream, &h->own_stream);
      h->engine = new oxf::TransformerEngine(s, max_batch, h->stream);
    } catch (...) {
      if (h->own_stream) cudaStreamDestroy(h->stream);
      delete h;
      throw;
    }
    *out = h;
  });
}

oxf_status oxf_transformer_destroy(oxf_transformer t) {
  if (!t) return OXF_OK;
  cudaStreamSynchronize(t->stream);
  delete t->engine;
  cudaFree(t->x_dev);
  cudaFree(t->t_dev);
  cudaFree(t->loss_dev);
  if (t->own_stream) cudaStreamDestroy(t->stream);
  delete t;
  return OXF_OK;
}

size_t oxf_transformer_param_count(oxf_transformer t) { return t ? t->engine->param_count() : 0; }
float* oxf_transformer_params(oxf_transformer t) { return t ? t->engine->params() : nullptr; }
float* oxf_transformer_grads(oxf_transformer t) { return t ? t->engine->grads() : nullptr; }
oxf_stream oxf_transformer_stream(oxf_transformer t) {
  return t ? reinterpret_cast<oxf_stream>(t->stream) : nullptr;
}

oxf_status oxf_transformer_set_params_host(oxf_transformer t, const float* params_host) {
  if (!t || !params_host) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] {
    oxf::check_cuda_call(cudaMemcpyAsync(t->engine->params(), params_host,
                                         t->engine->param_count() * 4, cudaMemcpyHostToDevice,
                                         t->stream),
                         "H2D params");
    oxf::check_cuda_call(cudaStreamSynchronize(t->stream), "sync");
  });
}

oxf_status oxf_transformer_get_params_host(oxf_transformer t, float* params_host) {
  if (!t || !params_host) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] {
    oxf::check_cuda_call(cudaMemcpyAsync(params_host, t->engine->params(),
                                         t->engine->param_count() * 4, cudaMemcpyDeviceToHost,
                                         t->stream),
                         "D2H params");
    oxf::check_cuda_call(cudaStreamSynchronize(t->stream), "sync");
  });
}

oxf_status oxf_transformer_forward(oxf_transformer t, const float* x, int batch, int causal,
                                   float* y) {
  if (!t || !x) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] {
    t->engine->forward(x, batch, causal != 0);
    if (y) {
      const auto& s = t->engine->spec();
      const size_t n = static_cast<size_t>(batch) * s.seq * s.o.out;
      oxf::check_cuda_call(cudaMemcpyAsync(y, t->engine->output(), n * 4,
                                           cudaMemcpyDeviceToDevice, t->stream),
                           "D2D output");
    }
  });
}

oxf_status oxf_transformer_train_forward(oxf_transformer t, const float* x, int batch) {
  if (!t || !x) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] { t->engine->train_forward(x, batch); });
}

oxf_status oxf_transformer_set_target(oxf_transformer t, const float* target) {
  if (!t || !target) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] { t->engine->set_target(target); });
}

oxf_status oxf_transformer_set_output_gradient(oxf_transformer t, const float* dy) {
  if (!t || !dy) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] { t->engine->set_output_gradient(dy); });
}

oxf_status oxf_transformer_backward_stage(oxf_transformer t, int stage) {
  if (!t) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  if (stage < 0 || stage > 2) return oxf::set_error(OXF_ERR_INVALID_ARG, "stage must be 0..2");
  return guard([&] { t->engine->backward_stage(stage); });
}

oxf_status oxf_transformer_bucket(oxf_transformer t, int stage, size_t* offset, size_t* count) {
  if (!t || !offset || !count) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  if (stage < 0 || stage > 2) return oxf::set_error(OXF_ERR_INVALID_ARG, "stage must be 0..2");
  t->engine->bucket(stage, offset, count);
  return OXF_OK;
}

oxf_status oxf_transformer_zero_grads(oxf_transformer t) {
  if (!t) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] { t->engine->zero_grads(); });
}

oxf_status oxf_transformer_sgd(oxf_transformer t, float lr) {
  if (!t) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] { t->engine->sgd(lr); });
}

oxf_status oxf_transformer_set_heads(oxf_transformer t, int heads) {
  if (!t) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] { t->engine->set_heads(heads); });
}

int oxf_transformer_heads(oxf_transformer t) { return t ? t->engine->heads() : 0; }

oxf_status oxf_transformer_output(oxf_transformer t, const float** y, const float** row_loss,
                                  const float** input_gradient) {
  if (!t) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  if (y) *y = t->engine->output();
  if (row_loss) *row_loss = t->engine->row_loss();
  if (input_gradient) *input_gradient = t->engine->input_gradient();
  return OXF_OK;
}

oxf_status oxf_transformer_set_timing(oxf_transformer t, int on) {
  if (!t) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  t->engine->set_timing(on != 0);
  return OXF_OK;
}

oxf_status oxf_transformer_read_timing(oxf_transformer t, double* gemm_ms, double* gemm_flops,
                                       int* launches) {
  if (!t) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] { t->engine->read_timing(gemm_ms, gemm_flops, launches); });
}

oxf_status oxf_transformer_train_step_host(oxf_transformer t, const float* x_host,
                                           const float* target_host, int batch, float lr,
                                           float* mean_loss_host) {
  if (!t || !x_host || !target_host) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] {
    oxf::TransformerEngine& e = *t->engine;
    const auto& s = e.spec();
    oxf::require(batch >= 1 && batch <= e.max_batch(), "batch outside [1, max_batch]");
    const size_t rows = static_cast<size_t>(batch) * s.seq;
    const size_t nx = rows * s.hidden, nt = rows * s.o.out;
    const size_t cap_x = static_cast<size_t>(e.max_batch()) * s.seq * s.hidden;
    const size_t cap_t = static_cast<size_t>(e.max_batch()) * s.seq * s.o.out;
    if (!t->x_dev) oxf::check_cuda_call(cudaMalloc(&t->x_dev, cap_x * 4), "cudaMalloc");
    if (!t->t_dev) oxf::check_cuda_call(cudaMalloc(&t->t_dev, cap_t * 4), "cudaMalloc");
    if (!t->loss_dev) oxf::check_cuda_call(cudaMalloc(&t->loss_dev, 4), "cudaMalloc");
    oxf::check_cuda_call(cudaMemcpyAsync(t->x_dev, x_host, nx * 4, cudaMemcpyHostToDevice,
                                         t->stream), "H2D x");
    oxf::check_cuda_call(cudaMemcpyAsync(t->t_dev, target_host, nt * 4, cudaMemcpyHostToDevice,
                                         t->stream), "H2D target");
    e.zero_grads();
    e.train_forward(t->x_dev, batch);
    e.set_target(t->t_dev);
    for (int st = 0; st < 3; ++st) e.backward_stage(st);
    e.sgd(lr / static_cast<float>(batch));
    oxf::check(oxf_slice_sum({e.row_loss(), rows}, t->loss_dev,
                             reinterpret_cast<oxf_stream>(t->stream)));
    float sum = 0.f;
    oxf::check_cuda_call(cudaMemcpyAsync(&sum, t->loss_dev, 4, cudaMemcpyDeviceToHost, t->stream),
                         "D2H loss");
    oxf::check_cuda_call(cudaStreamSynchronize(t->stream), "sync");
    if (mean_loss_host) *mean_loss_host = sum / static_cast<float>(rows);
  });
}

// ---------------------------------------------------------------- MLP
oxf_status oxf_mlp_create(const oxf_mlp_spec* spec, size_t max_rows, oxf_stream stream,
                          oxf_mlp* out) {
  if (!spec || !out) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  return guard([&] {
    oxf::MlpSpec s = mlp_spec(*spec);
    auto* h = new oxf_mlp_s();
    h->spec = *spec;
    try {
      h->stream = make_stream(stream, &h->own_stream);
      h->engine = new oxf::MlpEngine(s, max_rows);
      h->nparams = s.param_count();
      oxf::check_cuda_call(cudaMalloc(&h->params, h->nparams * 4), "cudaMalloc");
      oxf::check_cuda_call(cudaMalloc(&h->grads, h->nparams * 4), "cudaMalloc");
      cudaMemsetAsync(h->params, 0, h->nparams * 4, h->stream);
      cudaMemsetAsync(h->grads, 0, h->nparams * 4, h->stream);
      h->engine->bind(h->params, h->grads);
    } catch (...) {
      delete h->engine;
      cudaFree(h->params);
      cudaFree(h->grads);
      if (h->own_stream) cudaStreamDestroy(h->stream);
      delete h;
      throw;
    }
    *out = h;
  });
}

oxf_status oxf_mlp_destroy(oxf_mlp m) {
  if (!m) return OXF_OK;
  cudaStreamSynchronize(m->stream);
  delete m->engine;
  cudaFree(m->params);
  cudaFree(m->grads);
  if (m->own_stream) cudaStreamDestroy(m->stream);
  delete m;
  return OXF_OK;
}

size_t oxf_mlp_param_count(oxf_mlp m) { return m ? m->nparams : 0; }
float* oxf_mlp_params(oxf_mlp m) { return m ? m->params : nullptr; }
float* oxf_mlp_grads(oxf_mlp m) { return m ? m->grads : nullptr; }

oxf_status oxf_mlp_forward(oxf_mlp m, const float* x, float* y, size_t rows) {
  if (!m || !x || !y) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] { m->engine->forward(x, y, rows, nullptr, m->stream); });
}

oxf_status oxf_mlp_backward(oxf_mlp m, const float* dy, float* dx, size_t rows) {
  if (!m || !dy) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] {
    float* out = dx;
    float* tmp = nullptr;
    if (!out) {
      const size_t n = rows * static_cast<size_t>(m->engine->spec().layers.front().in);
      oxf::check_cuda_call(cudaMallocAsync(reinterpret_cast<void**>(&tmp), n * 4, m->stream),
                           "cudaMallocAsync");
      out = tmp;
    }
    m->engine->backward(dy, out, rows, nullptr, m->stream);
    if (tmp) cudaFreeAsync(tmp, m->stream);
  });
}

oxf_status oxf_mlp_zero_grads(oxf_mlp m) {
  if (!m) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] {
    oxf::check_cuda_call(cudaMemsetAsync(m->grads, 0, m->nparams * 4, m->stream), "memset");
  });
}

oxf_status oxf_mlp_sgd(oxf_mlp m, float lr) {
  if (!m) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] {
    oxf::check(oxf_sgd_update({m->params, m->nparams}, {m->grads, m->nparams}, lr,
                              reinterpret_cast<oxf_stream>(m->stream)));
  });
}

// ---------------------------------------------------------------- checkpoints (v1)
// ================================================================ runtime + Linear
oxf_status oxf_runtime_create(int device, oxf_stream stream, oxf_runtime* out) {
  if (!out) return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_runtime_create: null out");
  *out = nullptr;
  return guard([&] {
    auto* r = new oxf_runtime_s;
    try {
      r->rt = new oxf::CudaRuntime(device, reinterpret_cast<cudaStream_t>(stream));
    } catch (...) {
      delete r;
      throw;
    }
    *out = r;
  });
}

oxf_status oxf_runtime_destroy(oxf_runtime r) {
  if (!r) return OXF_OK;
  delete r->rt;
  delete r;
  return OXF_OK;
}

oxf_stream oxf_runtime_stream(oxf_runtime r) {
  return r ? reinterpret_cast<oxf_stream>(r->rt->stream()) : nullptr;
}

oxf_status oxf_runtime_sync(oxf_runtime r) {
  if (!r) return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_runtime_sync: null runtime");
  return guard([&] { r->rt->sync(); });
}

oxf_status oxf_runtime_reserve_buffers(oxf_runtime r, size_t len, size_t count) {
  if (!r) return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_runtime_reserve_buffers: null runtime");
  return guard([&] { r->rt->reserve_buffers(len, count); });
}

oxf_status oxf_runtime_pooled_buffers(oxf_runtime r, size_t* count) {
  if (!r || !count)
    return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_runtime_pooled_buffers: null argument");
  *count = r->rt->pooled_buffers();
  return OXF_OK;
}

oxf_status oxf_linear_create(oxf_runtime r, const oxf_layer_spec* spec, const float* weights_host,
                             const float* bias_host, oxf_linear* out) {
  if (!r || !spec || !weights_host || !out)
    return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_linear_create: null argument");
  *out = nullptr;
  return guard([&] {
    const oxf::LayerSpec s = layer(*spec);
    oxf::require(!s.bias || bias_host != nullptr, "oxf_linear_create: a biased layer needs bias_host");
    oxf::CudaRuntime& rt = *r->rt;
    oxf::Matrix w = rt.matrix_from_host(weights_host, static_cast<size_t>(s.in),
                                        static_cast<size_t>(s.out));
    std::optional<oxf::Vector> b;
    if (s.bias) b.emplace(rt.vector_from_host(bias_host, static_cast<size_t>(s.out)));
    auto* l = new oxf_linear_s;
    l->rt = r->rt;
    try {
      l->layer = new oxf::Linear(std::move(w), std::move(b), static_cast<oxf::Activation>(s.act));
    } catch (...) {
      delete l;
      throw;
    }
    rt.sync();  // the host arrays may be released on return
    *out = l;
  });
}

oxf_status oxf_linear_destroy(oxf_linear l) {
  if (!l) return OXF_OK;
  delete l->layer;  // its buffers go back to the runtime's pool
  delete l;
  return OXF_OK;
}

oxf_status oxf_linear_params(oxf_linear l, float** weights, float** bias) {
  if (!l) return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_linear_params: null layer");
  if (weights) *weights = l->layer->weights().data();
  if (bias) *bias = l->layer->bias() ? l->layer->bias()->data() : nullptr;
  return OXF_OK;
}

namespace {

// A borrowed rows x cols view of caller-owned device memory. Views of null
// optional arguments are built but never passed on.
oxf::Matrix view(const float* p, size_t rows, size_t cols) {
  return oxf::Matrix::view(const_cast<float*>(p), rows, cols);
}

}  // namespace

oxf_status oxf_linear_forward(oxf_linear l, const float* x, size_t rows, const float* residual,
                              float* y, float* pre_activation, oxf_stream stream) {
  if (!l) return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_linear_forward: null layer");
  return guard([&] {
    const oxf::Linear& L = *l->layer;
    oxf::require(rows == 0 || (x && y), "oxf_linear_forward: null x or y");
    const oxf::Matrix xm = view(x, rows, L.input_neurons());
    oxf::Matrix ym = view(y, rows, L.output_neurons());
    const oxf::Matrix rm = view(residual, rows, L.output_neurons());
    oxf::Matrix pm = view(pre_activation, rows, L.output_neurons());
    L.forward_into(xm, residual ? &rm : nullptr, ym, pre_activation ? &pm : nullptr, *l->rt,
                   reinterpret_cast<cudaStream_t>(stream));
  });
}

oxf_status oxf_linear_backward(oxf_linear l, const float* pre_activation,
                               const float* output_gradient, const float* residual_gradient,
                               size_t rows, float* gradient, float* bias_gradient,
                               oxf_stream stream) {
  if (!l) return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_linear_backward: null layer");
  return guard([&] {
    const oxf::Linear& L = *l->layer;
    const size_t o = L.output_neurons();
    oxf::require(rows == 0 || (output_gradient && gradient),
                 "oxf_linear_backward: null output_gradient or gradient");
    const oxf::Matrix zm = view(pre_activation, rows, o);
    const oxf::Matrix dym = view(output_gradient, rows, o);
    const oxf::Matrix drm = view(residual_gradient, rows, o);
    oxf::Matrix gm = view(gradient, rows, o);
    oxf::Vector bg = oxf::Vector::view(bias_gradient, bias_gradient ? o : 0);
    L.backward_into(pre_activation ? &zm : nullptr, dym, residual_gradient ? &drm : nullptr, gm,
                    bias_gradient ? &bg : nullptr, *l->rt, reinterpret_cast<cudaStream_t>(stream));
  });
}

oxf_status oxf_linear_learn(oxf_linear l, const float* x, const float* gradient,
                            const float* bias_gradient, size_t rows, float learning_rate,
                            oxf_stream stream) {
  if (!l) return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_linear_learn: null layer");
  return guard([&] {
    oxf::Linear& L = *l->layer;
    oxf::require(rows == 0 || (x && gradient), "oxf_linear_learn: null x or gradient");
    const oxf::Matrix xm = view(x, rows, L.input_neurons());
    const oxf::Matrix gm = view(gradient, rows, L.output_neurons());
    const oxf::Vector bg =
        oxf::Vector::view(const_cast<float*>(bias_gradient), bias_gradient ? L.output_neurons() : 0);
    L.learn(xm, gm, bias_gradient ? &bg : nullptr, learning_rate, *l->rt,
            reinterpret_cast<cudaStream_t>(stream));
  });
}

oxf_status oxf_linear_input_gradient(oxf_linear l, const float* gradient, size_t rows, float* dx,
                                     oxf_stream stream) {
  if (!l) return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_linear_input_gradient: null layer");
  return guard([&] {
    const oxf::Linear& L = *l->layer;
    oxf::require(rows == 0 || (gradient && dx), "oxf_linear_input_gradient: null gradient or dx");
    const oxf::Matrix gm = view(gradient, rows, L.output_neurons());
    oxf::Matrix dxm = view(dx, rows, L.input_neurons());
    L.input_gradient_into(gm, dxm, *l->rt, reinterpret_cast<cudaStream_t>(stream));
  });
}

oxf_status oxf_checkpoint_write_linear(const char* path, const oxf_layer_spec* spec,
                                       const float* params_host, size_t count) {
  return write_ckpt<oxf_layer_spec>(
      path, oxf::ckpt::ModelType::Linear, spec, params_host, count,
      [](oxf::ckpt::Model& m, const oxf_layer_spec& s) { m.linear = s; });
}

oxf_status oxf_checkpoint_write_mlp(const char* path, const oxf_mlp_spec* spec,
                                    const float* params_host, size_t count) {
  return write_ckpt<oxf_mlp_spec>(path, oxf::ckpt::ModelType::Mlp, spec, params_host, count,
                                  [](oxf::ckpt::Model& m, const oxf_mlp_spec& s) { m.mlp = s; });
}

oxf_status oxf_checkpoint_write_transformer(const char* path, const oxf_transformer_spec* spec,
                                            const float* params_host, size_t count) {
  return write_ckpt<oxf_transformer_spec>(
      path, oxf::ckpt::ModelType::Transformer, spec, params_host, count,
      [](oxf::ckpt::Model& m, const oxf_transformer_spec& s) { m.transformer = s; });
}

oxf_status oxf_checkpoint_read_linear(const char* path, oxf_layer_spec* spec, float* params_host,
                                      size_t capacity, size_t* count) {
  return read_ckpt<oxf_layer_spec>(path, oxf::ckpt::ModelType::Linear, spec, params_host,
                                   capacity, count,
                                   [](const oxf::ckpt::Model& m) { return m.linear; });
}

oxf_status oxf_checkpoint_read_mlp(const char* path, oxf_mlp_spec* spec, float* params_host,
                                   size_t capacity, size_t* count) {
  return read_ckpt<oxf_mlp_spec>(path, oxf::ckpt::ModelType::Mlp, spec, params_host, capacity,
                                 count, [](const oxf::ckpt::Model& m) { return m.mlp; });
}

oxf_status oxf_checkpoint_read_transformer(const char* path, oxf_transformer_spec* spec,
                                           float* params_host, size_t capacity, size_t* count) {
  return read_ckpt<oxf_transformer_spec>(
      path, oxf::ckpt::ModelType::Transformer, spec, params_host, capacity, count,
      [](const oxf::ckpt::Model& m) { return m.transformer; });
}

oxf_status oxf_transformer_dump(oxf_transformer t, const char* path) {
  if (!t || !path) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] {
    oxf::ckpt::Model m;
    m.type = oxf::ckpt::ModelType::Transformer;
    m.transformer = t->spec;
    m.params.resize(t->engine->param_count());
    oxf::check(oxf_transformer_get_params_host(t, m.params.data()));
    oxf::ckpt::write(path, m);
  });
}

oxf_status oxf_transformer_load(const char* path, int max_batch, oxf_stream stream,
                                oxf_transformer* out) {
  if (!path || !out) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  return guard([&] {
    const oxf::ckpt::Model m = oxf::ckpt::read(path, oxf::ckpt::ModelType::Transformer);
    oxf_transformer t = nullptr;
    oxf::check(oxf_transformer_create(&m.transformer, max_batch, stream, &t));
    const oxf_status st = oxf_transformer_set_params_host(t, m.params.data());
    if (st != OXF_OK) {
      oxf_transformer_destroy(t);
      oxf::check(st);
    }
    *out = t;
  });
}

oxf_status oxf_mlp_dump(oxf_mlp m, const char* path) {
  if (!m || !path) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  return guard([&] {
    oxf::ckpt::Model c;
    c.type = oxf::ckpt::ModelType::Mlp;
    c.mlp = m->spec;
    c.params.resize(m->nparams);
    oxf::check_cuda_call(cudaMemcpyAsync(c.params.data(), m->params, m->nparams * 4,
                                         cudaMemcpyDeviceToHost, m->stream),
                         "D2H params");
    oxf::check_cuda_call(cudaStreamSynchronize(m->stream), "sync");
    oxf::ckpt::write(path, c);
  });
}

oxf_status oxf_mlp_load(const char* path, size_t max_rows, oxf_stream stream, oxf_mlp* out) {
  if (!path || !out) return oxf::set_error(OXF_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  return guard([&] {
    const oxf::ckpt::Model c = oxf::ckpt::read(path, oxf::ckpt::ModelType::Mlp);
    oxf_mlp m = nullptr;
    oxf::check(oxf_mlp_create(&c.mlp, max_rows, stream, &m));
    cudaError_t e = cudaMemcpyAsync(m->params, c.params.data(), c.params.size() * 4,
                                    cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) {
      oxf_mlp_destroy(m);
      oxf::check_cuda_call(e, "H2D params");
    }
    *out = m;
  });
}

}  // extern "C"
