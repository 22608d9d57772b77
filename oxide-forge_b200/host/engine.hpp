// engine.hpp — batched executors for the MLP and the single-block
// Post-Norm transformer: the throughput path behind the reference API.
//
// The reference runs one [seq, hidden] sequence per call through Linear /
// MlpExecutor / Attention / TrainingTransformer (src/net/*), with one kernel
// launch per operation and materialised transposes. These engines run B
// independent sequences per call as [B*seq, hidden] row blocks:
//   - every Linear is one GEMM over all B*seq rows, with bias, residual,
//     activation and pre-activation store fused into the epilogue;
//   - QKᵀ and P·V are batched GEMMs over the B sequences; the 1/sqrt(d)
//     scale is the GEMM alpha; Q/K/V projections are one batched launch;
//   - backward products read operands in their stored layout (no
//     transposes); activation derivatives and residual gradients are fused
//     into the epilogues of the dX GEMMs; weight gradients accumulate
//     atomically into a flat gradient arena (split-K where K = B*seq).
// With B = 1 the arithmetic is the reference's (tests check it against the
// oracle). Parameters and gradients live in flat arenas in checkpoint
// cursor order (src/net/transformer/inference.rs:52-66,
// src/net/metadata.rs:21-68): per Linear the weight [in,out] then the bias.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <vector>

#include "runtime.hpp"

namespace oxf {

struct LayerSpec {
  int in = 0, out = 0;
  int act = OXF_ACT_IDENTITY;
  bool bias = false;
  size_t param_count() const { return static_cast<size_t>(in) * out + (bias ? out : 0); }
};

// MlpExecutor layers plus the optional residual range (mlp.rs:14-19):
// the input of layer res_start is added to the output of layer res_end-1.
struct MlpSpec {
  std::vector<LayerSpec> layers;
  int res_start = -1, res_end = -1;
  size_t param_count() const;
  int max_width() const;
};

// Single-block transformer (encoder.rs, inference.rs): Q/K/V/output Linears,
// a position table [seq, hidden], a feed-forward MLP and a NormType.
struct TransformerSpec {
  int seq = 0, hidden = 0;
  int norm = OXF_NORM_LAYER;
  LayerSpec q, k, v;
  MlpSpec ffn;
  LayerSpec o;
  size_t param_count() const;
};

// Records CUDA events around every GEMM an engine launches while enabled,
// so a caller can measure the GEMM share of a step on the device without a
// profiler (flops = 2*M*N*K*batch per launch).
class GemmTimer {
 public:
  ~GemmTimer();
  void begin(cudaStream_t s, double flops);
  void end(cudaStream_t s);
  // Synchronises, returns totals since the last read and resets.
  void read(double* ms, double* flops, int* launches);

 private:
  std::vector<cudaEvent_t> ev_;
  std::vector<double> flops_;
  size_t used_ = 0;
};

// The timer GEMMs on this thread report to (nullptr: off).
GemmTimer*& active_gemm_timer();

// Thin GEMM descriptor builder over oxf_gemm (include/oxf.h).
class Gemm {
 public:
  Gemm(int M, int N, int K, bool a_trans, bool b_trans, const float* A, const float* B, float* C);
  Gemm& batch(int n, long long sa, long long sb, long long sc);
  Gemm& ld(long long lda, long long ldb, long long ldc);
  Gemm& alpha(float a);
  Gemm& beta(float b);
  Gemm& bias(const float* b);
  Gemm& residual(const float* r, long long ldr, long long stride = 0);
  Gemm& pre_out(float* p, long long ldp, long long stride = 0);
  Gemm& grad_act(int act, const float* aux, long long ldx, long long stride = 0);
  Gemm& act(int a);
  Gemm& accumulate();
  Gemm& reduce_batch();
  void run(cudaStream_t s) const;

 private:
  oxf_gemm_desc d_;
};

class MlpEngine {
 public:
  MlpEngine(const MlpSpec& spec, size_t max_rows);
  ~MlpEngine();
  MlpEngine(const MlpEngine&) = delete;
  MlpEngine& operator=(const MlpEngine&) = delete;

  const MlpSpec& spec() const { return spec_; }
  size_t param_count() const { return spec_.param_count(); }
  // Points the layers at slices of a parameter / gradient arena.
  void bind(float* params, float* grads);
  float* weight(int i) const;
  float* bias(int i) const;
  float* weight_grad(int i) const;
  float* bias_grad(int i) const;

  // y = MLP(x) (+ extra_residual added after the last activation).
  // x must stay valid until backward. keep_pre = false (inference) skips
  // storing the pre-activations, which only backward reads.
  void forward(const float* x, float* y, size_t rows, const float* extra_residual,
               cudaStream_t s, bool keep_pre = true);
  // Given dL/dy, accumulates parameter gradients and writes dL/dx
  // (+ extra_dx added to it). Requires the preceding forward.
  void backward(const float* dy, float* dx, size_t rows, const float* extra_dx, cudaStream_t s);

 private:
  MlpSpec spec_;
  size_t max_rows_;
  std::vector<size_t> w_off_, b_off_;
  float* params_ = nullptr;
  float* grads_ = nullptr;
  const float* x_ = nullptr;         // input of layer 0 (caller-owned)
  std::vector<float*> outs_;         // output of layer i (input of i+1), i < L-1
  std::vector<float*> pres_;         // pre-activation of layer i (activated layers)
  float* gbuf_[2] = {nullptr, nullptr};
  float* skip_ = nullptr;
  std::vector<void*> allocs_;
};

class TransformerEngine {
 public:
  TransformerEngine(const TransformerSpec& spec, int max_batch, cudaStream_t stream);
  ~TransformerEngine();
  TransformerEngine(const TransformerEngine&) = delete;
  TransformerEngine& operator=(const TransformerEngine&) = delete;

  const TransformerSpec& spec() const { return spec_; }
  int max_batch() const { return max_batch_; }
  cudaStream_t stream() const { return stream_; }
  size_t param_count() const { return nparams_; }
  float* params() const { return params_; }
  float* grads() const { return grads_; }
  float* output() const { return y_; }              // [batch*seq, out]
  float* input_gradient() const { return dpos_; }   // [batch*seq, hidden] after stage 2
  float* row_loss() const { return loss_; }         // [batch*seq] after set_target

  // Inference forward (InferenceBlock::forward / forward_mask,
  // inference.rs:76-109): y = output(x) for `batch` sequences.
  void forward(const float* x, int batch, bool causal);
  // Training forward (TrainingTransformer::forward, encoder.rs:114-133);
  // keeps what backward needs. x is copied into the engine.
  void train_forward(const float* x, int batch);
  // dL/dy = (y - target)/out and the per-row loss (linear.rs:325-333).
  void set_target(const float* target);
  // Copies a caller-provided dL/dy instead.
  void set_output_gradient(const float* dy);
  // Backward in three stages so gradient buckets can be reduced while the
  // next stage runs: 0 = output Linear, 1 = feed-forward, 2 = attention,
  // Q/K/V and position. Gradients ACCUMULATE into grads().
  void backward_stage(int stage);
  // [offset, count) of the parameters stage `stage` produces gradients for.
  void bucket(int stage, size_t* offset, size_t* count) const;
  void zero_grads();
  // params -= lr * grads (Linear::learn, linear.rs:373-391, applied once).
  void sgd(float lr);
  // Attention heads (1, the reference's single-head attention, by default).
  // Head j attends over columns [j*D/h, (j+1)*D/h) of Q and K and
  // [j*H/h, (j+1)*H/h) of V with scale 1/sqrt(D/h), writing those columns
  // of the attention output; the projections and every other layer are
  // unchanged. h must divide the query width D and hidden H. Takes effect
  // from the next forward; the paths that keep per-head scores (training,
  // and inference the fused kernel cannot take) grow the score buffers to h
  // per sequence on first use.
  void set_heads(int h);
  int heads() const { return heads_; }
  // GEMM event timing (off by default).
  void set_timing(bool on) { timing_ = on; }
  void read_timing(double* ms, double* flops, int* launches) { timer_.read(ms, flops, launches); }
  // Scope guard: GEMMs launched while alive report to this engine's timer.
  struct TimingScope {
    explicit TimingScope(TransformerEngine* e)
        : prev(active_gemm_timer()) { active_gemm_timer() = e->timing_ ? &e->timer_ : nullptr; }
    ~TimingScope() { active_gemm_timer() = prev; }
    GemmTimer* prev;
  };

 private:
  void forward_impl(const float* x, int batch, bool causal, bool training);
  // training: P is kept for backward (three launches); inference: the
  // softmax is fused into the two products (oxf_attention_forward)
  void attention_forward(const float* x, int batch, bool causal, bool training);
  // the core with heads_ > 1: in inference the fused kernel
  // (oxf_attention_heads_forward) where it applies, else per-head batched
  // products over column slices (training keeps P for backward)
  void attention_heads_forward(int batch, bool causal, bool training);
  void attention_heads_backward(int batch);
  void ensure_score_buffers();
  void qkv_project(int batch, bool keep_pre);

  TransformerSpec spec_;
  int max_batch_;
  cudaStream_t stream_;
  size_t nparams_ = 0;
  size_t off_q_ = 0, off_k_ = 0, off_v_ = 0, off_pos_ = 0, off_ffn_ = 0, off_o_ = 0;
  float* params_ = nullptr;
  float* grads_ = nullptr;
  MlpEngine* ffn_ = nullptr;
  int batch_ = 0;
  bool trained_ = false;  // the last forward kept what backward reads
  // activations
  float *x_ = nullptr, *pos_ = nullptr, *qkv_ = nullptr, *qkv_pre_ = nullptr, *p_ = nullptr;
  float* stats_ = nullptr;  // softmax row statistics of the fused inference attention
  float *pre_norm_ = nullptr, *h1_ = nullptr, *pre2_ = nullptr, *enc_ = nullptr;
  float *zo_ = nullptr, *y_ = nullptr, *loss_ = nullptr;
  // gradients
  float *dy_ = nullptr, *denc_ = nullptr, *d2_ = nullptr, *d1_ = nullptr, *dr_ = nullptr;
  float *dp_ = nullptr, *dqkv_ = nullptr, *dpos_ = nullptr;
  int heads_ = 1;
  int score_heads_ = 1;  // heads the p_ / dp_ buffers are sized for
  std::vector<void*> allocs_;
  float* alloc(size_t n);
  void release(float* p);  // frees one of allocs_
  bool timing_ = false;
  GemmTimer timer_;
};

}  // namespace oxf
