// engine.cpp — batched MLP and transformer executors (see engine.hpp).
#include "engine.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace oxf {

// ================================================================ specs
size_t MlpSpec::param_count() const {
  size_t n = 0;
  for (const auto& l : layers) n += l.param_count();
  return n;
}

int MlpSpec::max_width() const {
  int w = 0;
  for (const auto& l : layers) w = std::max({w, l.in, l.out});
  return w;
}

size_t TransformerSpec::param_count() const {
  return q.param_count() + k.param_count() + v.param_count() +
         static_cast<size_t>(seq) * hidden + ffn.param_count() + o.param_count();
}

// ================================================================ Gemm builder
Gemm::Gemm(int M, int N, int K, bool a_trans, bool b_trans, const float* A, const float* B,
           float* C) {
  oxf_gemm_desc_init(&d_, M, N, K, a_trans ? 1 : 0, b_trans ? 1 : 0, A, B, C);
}
Gemm& Gemm::batch(int n, long long sa, long long sb, long long sc) {
  d_.batch = n;
  d_.stride_a = sa;
  d_.stride_b = sb;
  d_.stride_c = sc;
  return *this;
}
Gemm& Gemm::ld(long long lda, long long ldb, long long ldc) {
  d_.lda = lda;
  d_.ldb = ldb;
  d_.ldc = ldc;
  return *this;
}
Gemm& Gemm::alpha(float a) { d_.alpha = a; return *this; }
Gemm& Gemm::beta(float b) { d_.beta = b; return *this; }
Gemm& Gemm::bias(const float* b) { d_.bias = b; return *this; }
Gemm& Gemm::residual(const float* r, long long ldr, long long stride) {
  d_.residual = r;
  d_.ldr = ldr;
  d_.stride_r = stride;
  return *this;
}
Gemm& Gemm::pre_out(float* p, long long ldp, long long stride) {
  d_.pre_out = p;
  d_.ldp = ldp;
  d_.stride_p = stride;
  return *this;
}
Gemm& Gemm::grad_act(int act, const float* aux, long long ldx, long long stride) {
  d_.grad_act = act;
  d_.aux = aux;
  d_.ldx = ldx;
  d_.stride_x = stride;
  return *this;
}
Gemm& Gemm::act(int a) { d_.act = a; return *this; }
Gemm& Gemm::accumulate() { d_.accumulate = 1; return *this; }
Gemm& Gemm::reduce_batch() { d_.reduce_batch = 1; return *this; }
void Gemm::run(cudaStream_t s) const {
  GemmTimer* t = active_gemm_timer();
  if (t) t->begin(s, 2.0 * d_.M * d_.N * static_cast<double>(d_.K) * d_.batch);
  check(oxf_gemm(&d_, ST(s)));
  if (t) t->end(s);
}

GemmTimer*& active_gemm_timer() {
  thread_local GemmTimer* t = nullptr;
  return t;
}

GemmTimer::~GemmTimer() {
  for (cudaEvent_t e : ev_) cudaEventDestroy(e);
}

void GemmTimer::begin(cudaStream_t s, double flops) {
  if (ev_.size() < 2 * (used_ + 1)) {
    for (int i = 0; i < 2; ++i) {
      cudaEvent_t e;
      check_cuda_call(cudaEventCreate(&e), "cudaEventCreate");
      ev_.push_back(e);
    }
    flops_.push_back(0.0);
  }
  flops_[used_] = flops;
  check_cuda_call(cudaEventRecord(ev_[2 * used_], s), "cudaEventRecord");
}

void GemmTimer::end(cudaStream_t s) {
  check_cuda_call(cudaEventRecord(ev_[2 * used_ + 1], s), "cudaEventRecord");
  ++used_;
}

void GemmTimer::read(double* ms, double* flops, int* launches) {
  double tm = 0.0, fl = 0.0;
  for (size_t i = 0; i < used_; ++i) {
    check_cuda_call(cudaEventSynchronize(ev_[2 * i + 1]), "cudaEventSynchronize");
    float e = 0.f;
    check_cuda_call(cudaEventElapsedTime(&e, ev_[2 * i], ev_[2 * i + 1]), "cudaEventElapsedTime");
    tm += e;
    fl += flops_[i];
  }
  if (ms) *ms = tm;
  if (flops) *flops = fl;
  if (launches) *launches = static_cast<int>(used_);
  used_ = 0;
}

namespace {

float* dev_alloc(size_t n, std::vector<void*>& list) {
  if (n == 0) return nullptr;
  void* p = nullptr;
  check_cuda_call(cudaMalloc(&p, n * sizeof(float)), "cudaMalloc");
  list.push_back(p);
  return static_cast<float*>(p);
}

void copy_d2d(float* dst, const float* src, size_t n, cudaStream_t s) {
  if (n)
    check_cuda_call(cudaMemcpyAsync(dst, src, n * sizeof(float), cudaMemcpyDeviceToDevice, s),
                    "cudaMemcpyAsync D2D");
}

oxf_cslice cs(const float* p, size_t n) { return {p, n}; }
oxf_slice ms(float* p, size_t n) { return {p, n}; }

}  // namespace

// ================================================================ MlpEngine
MlpEngine::MlpEngine(const MlpSpec& spec, size_t max_rows) : spec_(spec), max_rows_(max_rows) {
  const int L = static_cast<int>(spec_.layers.size());
  require(L >= 1, "MLP must contain at least one layer");  // mlp.rs:42
  if (spec_.res_start >= 0 || spec_.res_end >= 0)
    require(spec_.res_start >= 0 && spec_.res_start < spec_.res_end && spec_.res_end <= L,
            "invalid residual range");  // mlp.rs:43-45
  for (int i = 0; i + 1 < L; ++i)
    require(spec_.layers[i].out == spec_.layers[i + 1].in, "MLP layer widths do not chain");
  if (spec_.res_end > 0)
    require(spec_.layers[spec_.res_start].in == spec_.layers[spec_.res_end - 1].out,
            "residual range endpoints have different widths");
  size_t off = 0;
  for (const auto& l : spec_.layers) {
    w_off_.push_back(off);
    off += static_cast<size_t>(l.in) * l.out;
    b_off_.push_back(l.bias ? off : static_cast<size_t>(-1));
    if (l.bias) off += l.out;
  }
  std::vector<void*> mine;
  outs_.assign(L, nullptr);
  pres_.assign(L, nullptr);
  for (int i = 0; i < L; ++i) {
    if (i + 1 < L) outs_[i] = dev_alloc(max_rows_ * spec_.layers[i].out, mine);
    if (spec_.layers[i].act != OXF_ACT_IDENTITY)
      pres_[i] = dev_alloc(max_rows_ * spec_.layers[i].out, mine);
  }
  const size_t w = static_cast<size_t>(spec_.max_width());
  gbuf_[0] = dev_alloc(max_rows_ * w, mine);
  gbuf_[1] = dev_alloc(max_rows_ * w, mine);
  if (spec_.res_end > 0) skip_ = dev_alloc(max_rows_ * spec_.layers[spec_.res_end - 1].out, mine);
  allocs_ = mine;
}

MlpEngine::~MlpEngine() {
  for (void* p : allocs_) cudaFree(p);
}

void MlpEngine::bind(float* params, float* grads) {
  params_ = params;
  grads_ = grads;
}

float* MlpEngine::weight(int i) const { return params_ + w_off_[i]; }
float* MlpEngine::bias(int i) const {
  return spec_.layers[i].bias ? params_ + b_off_[i] : nullptr;
}
float* MlpEngine::weight_grad(int i) const { return grads_ + w_off_[i]; }
float* MlpEngine::bias_grad(int i) const {
  return spec_.layers[i].bias ? grads_ + b_off_[i] : nullptr;
}

// MlpExecutor::forward / TrainingMlp::forward (mlp.rs:53-85, 233-254):
// Linear::forward per layer (GEMM, bias, residual, activation) as one GEMM.
void MlpEngine::forward(const float* x, float* y, size_t rows, const float* extra_residual,
                        cudaStream_t s, bool keep_pre) {
  require(rows <= max_rows_, "MlpEngine::forward: more rows than the engine was sized for");
  const int L = static_cast<int>(spec_.layers.size());
  x_ = x;
  const float* in = x;
  for (int i = 0; i < L; ++i) {
    const LayerSpec& l = spec_.layers[i];
    float* out = (i == L - 1) ? y : outs_[i];
    Gemm g(static_cast<int>(rows), l.out, l.in, false, false, in, weight(i), out);
    if (l.bias) g.bias(bias(i));
    bool extra_fused = false;
    if (spec_.res_end - 1 == i) {
      const float* r = spec_.res_start == 0 ? x : outs_[spec_.res_start - 1];
      g.residual(r, l.out);
    } else if (i == L - 1 && extra_residual && l.act == OXF_ACT_IDENTITY) {
      g.residual(extra_residual, l.out);
      extra_fused = true;
    }
    if (l.act != OXF_ACT_IDENTITY) {
      if (keep_pre) g.pre_out(pres_[i], l.out);
      g.act(l.act);
    }
    g.run(s);
    if (i == L - 1 && extra_residual && !extra_fused)
      check(oxf_slice_binary_assign(ms(out, rows * l.out), cs(extra_residual, rows * l.out),
                                    OXF_ADD, ST(s)));
    in = out;
  }
}

// MlpExecutor::backward (mlp.rs:121-168) with the parameter update deferred:
// per layer G = dY ⊙ act'(Z) (fused into the previous dX GEMM), dW += XᵀG,
// db += colsum(G), dX = G·Wᵀ (+ the skip gradient of the residual range).
void MlpEngine::backward(const float* dy, float* dx, size_t rows, const float* extra_dx,
                         cudaStream_t s) {
  const int L = static_cast<int>(spec_.layers.size());
  const float* G = dy;
  int gi = -1;  // which gbuf_ holds G (-1: the caller's dy)
  const LayerSpec& last = spec_.layers[L - 1];
  if (last.act != OXF_ACT_IDENTITY) {
    copy_d2d(gbuf_[0], dy, rows * last.out, s);
    check(oxf_slice_mul_act_derivative(ms(gbuf_[0], rows * last.out),
                                       cs(pres_[L - 1], rows * last.out),
                                       static_cast<oxf_activation>(last.act), ST(s)));
    G = gbuf_[0];
    gi = 0;
  }
  for (int i = L - 1; i >= 0; --i) {
    const LayerSpec& l = spec_.layers[i];
    const float* in = (i == 0) ? x_ : outs_[i - 1];
    // weight and bias gradients
    Gemm(l.in, l.out, static_cast<int>(rows), true, false, in, G, weight_grad(i))
        .accumulate()
        .run(s);
    if (l.bias)
      check(oxf_matrix_sum_cols(cs(G, rows * l.out), ms(bias_grad(i), l.out), l.out, 1, ST(s)));
    // residual range: the gradient at the end layer also reaches the start
    // layer's input (mlp.rs:145-154)
    if (spec_.res_end - 1 == i && spec_.res_start != i) copy_d2d(skip_, G, rows * l.out, s);
    const float* skip_now = nullptr;
    if (spec_.res_start == i) skip_now = (spec_.res_end - 1 == i) ? G : skip_;
    if (i > 0) {
      const int wi = (gi == 0) ? 1 : 0;
      float* out = gbuf_[wi];
      Gemm g(static_cast<int>(rows), l.in, l.out, false, true, G, weight(i), out);
      if (skip_now) g.residual(skip_now, l.in);
      const LayerSpec& prev = spec_.layers[i - 1];
      if (prev.act != OXF_ACT_IDENTITY) g.grad_act(prev.act, pres_[i - 1], l.in);
      g.run(s);
      G = out;
      gi = wi;
    } else {
      Gemm g(static_cast<int>(rows), l.in, l.out, false, true, G, weight(0), dx);
      const float* r1 = skip_now ? skip_now : extra_dx;
      const float* r2 = skip_now ? extra_dx : nullptr;
      if (r1) g.residual(r1, l.in);
      g.run(s);
      if (r2)
        check(oxf_slice_binary_assign(ms(dx, rows * l.in), cs(r2, rows * l.in), OXF_ADD, ST(s)));
    }
  }
}

// ================================================================ TransformerEngine
float* TransformerEngine::alloc(size_t n) { return dev_alloc(n, allocs_); }

void TransformerEngine::release(float* p) {
  if (!p) return;
  for (size_t i = 0; i < allocs_.size(); ++i)
    if (allocs_[i] == p) {
      cudaFree(p);
      allocs_.erase(allocs_.begin() + static_cast<long>(i));
      return;
    }
}

void TransformerEngine::set_heads(int h) {
  const int H = spec_.hidden, D = spec_.q.out;
  require(h >= 1 && D % h == 0 && H % h == 0,
          "transformer: heads must divide the query width and hidden");
  heads_ = h;
}

// The per-head probabilities of every sequence, [heads, batch, S, S], for
// the paths that materialise them (training, and inference the fused kernel
// cannot take); allocated on first use, after the stream drains.
void TransformerEngine::ensure_score_buffers() {
  if (heads_ <= score_heads_) return;
  const int S = spec_.seq;
  check_cuda_call(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
  const size_t n = static_cast<size_t>(heads_) * max_batch_ * S * S;
  float* p = alloc(n);
  float* dp = alloc(n);
  release(p_);
  release(dp_);
  p_ = p;
  dp_ = dp;
  score_heads_ = heads_;
}

TransformerEngine::TransformerEngine(const TransformerSpec& spec, int max_batch,
                                     cudaStream_t stream)
    : spec_(spec), max_batch_(max_batch), stream_(stream) {
  const int S = spec_.seq, H = spec_.hidden;
  require(S > 0 && H > 0 && max_batch > 0, "transformer: empty shape");
  require(spec_.q.in == H && spec_.k.in == H && spec_.v.in == H, "Q/K/V take hidden inputs");
  require(spec_.q.out == spec_.k.out, "query and key widths differ");
  require(spec_.v.out == H, "value width must equal hidden (residual add, attention.rs:249)");
  require(!spec_.ffn.layers.empty() && spec_.ffn.layers.front().in == H &&
              spec_.ffn.layers.back().out == H,
          "feed-forward must map hidden to hidden (inference.rs:99)");
  require(spec_.o.in == H, "output Linear takes hidden inputs");
  require(spec_.norm == OXF_NORM_LAYER || spec_.norm == OXF_NORM_RMS, "bad NormType");

  off_q_ = 0;
  off_k_ = off_q_ + spec_.q.param_count();
  off_v_ = off_k_ + spec_.k.param_count();
  off_pos_ = off_v_ + spec_.v.param_count();
  off_ffn_ = off_pos_ + static_cast<size_t>(S) * H;
  off_o_ = off_ffn_ + spec_.ffn.param_count();
  nparams_ = off_o_ + spec_.o.param_count();
  params_ = alloc(nparams_);
  grads_ = alloc(nparams_);
  check_cuda_call(cudaMemsetAsync(params_, 0, nparams_ * 4, stream_), "memset");
  check_cuda_call(cudaMemsetAsync(grads_, 0, nparams_ * 4, stream_), "memset");

  const size_t T = static_cast<size_t>(max_batch) * S;
  const size_t D = spec_.q.out, O = spec_.o.out;
  const size_t qkvw = 2 * D + H;
  ffn_ = new MlpEngine(spec_.ffn, T);
  ffn_->bind(params_ + off_ffn_, grads_ + off_ffn_);
  pos_ = alloc(T * H);
  qkv_ = alloc(T * qkvw);
  if (spec_.q.act || spec_.k.act || spec_.v.act) qkv_pre_ = alloc(T * qkvw);
  p_ = alloc(static_cast<size_t>(max_batch) * S * S);
  stats_ = alloc(oxf_attention_stats_floats(max_batch, S));
  pre_norm_ = alloc(T * H);
  h1_ = alloc(T * H);
  pre2_ = alloc(T * H);
  enc_ = alloc(T * H);
  if (spec_.o.act) zo_ = alloc(T * O);
  y_ = alloc(T * O);
  loss_ = alloc(T);
  dy_ = alloc(T * O);
  denc_ = alloc(T * H);
  d2_ = alloc(T * H);
  d1_ = alloc(T * H);
  dr_ = alloc(T * H);
  dp_ = alloc(static_cast<size_t>(max_batch) * S * S);
  dqkv_ = alloc(T * qkvw);
  dpos_ = alloc(T * H);
}

TransformerEngine::~TransformerEngine() {
  cudaStreamSynchronize(stream_);
  delete ffn_;
  for (void* p : allocs_) cudaFree(p);
}

// Q, K, V = act(pos·W + b) (QkvProjection::project, attention.rs:65-94): one
// batched GEMM when the three projections share shape, activation and have
// no bias; otherwise three GEMMs.
void TransformerEngine::qkv_project(int batch, bool keep_pre) {
  const int H = spec_.hidden;
  const int T = batch * spec_.seq;
  const int D = spec_.q.out;
  const LayerSpec* ls[3] = {&spec_.q, &spec_.k, &spec_.v};
  const size_t offs[3] = {off_q_, off_k_, off_v_};
  float* outs[3] = {qkv_, qkv_ + static_cast<size_t>(T) * D, qkv_ + 2 * static_cast<size_t>(T) * D};
  const bool uniform = spec_.q.out == spec_.v.out && spec_.q.act == spec_.k.act &&
                       spec_.q.act == spec_.v.act && !spec_.q.bias && !spec_.k.bias &&
                       !spec_.v.bias;
  if (uniform) {
    Gemm g(T, D, H, false, false, pos_, params_ + off_q_, qkv_);
    g.batch(3, 0, static_cast<long long>(spec_.q.param_count()), static_cast<long long>(T) * D);
    if (spec_.q.act) {
      if (keep_pre) g.pre_out(qkv_pre_, D, static_cast<long long>(T) * D);
      g.act(spec_.q.act);
    }
    g.run(stream_);
    return;
  }
  for (int j = 0; j < 3; ++j) {
    const LayerSpec& l = *ls[j];
    Gemm g(T, l.out, H, false, false, pos_, params_ + offs[j], outs[j]);
    if (l.bias) g.bias(params_ + offs[j] + static_cast<size_t>(l.in) * l.out);
    if (l.act) {
      if (keep_pre) g.pre_out(qkv_pre_ + (outs[j] - qkv_), l.out);
      g.act(l.act);
    }
    g.run(stream_);
  }
}

void TransformerEngine::attention_forward(const float* x, int batch, bool causal, bool training) {
  const int S = spec_.seq, H = spec_.hidden, D = spec_.q.out;
  const size_t T = static_cast<size_t>(batch) * S;
  // positioned = input + position (inference.rs:78, encoder.rs:117)
  check(oxf_slice_binary_broadcast(cs(x, T * H), cs(params_ + off_pos_, static_cast<size_t>(S) * H),
                                   ms(pos_, T * H), OXF_ADD, ST(stream_)));
  qkv_project(batch, training);
  const float* q = qkv_;
  const float* k = qkv_ + T * D;
  const float* v = qkv_ + 2 * T * D;
  if (heads_ > 1) {
    attention_heads_forward(batch, causal, training);
    check(oxf_norm_rows(cs(pre_norm_, T * H), ms(h1_, T * H), H, spec_.norm, 1e-5f, nullptr,
                        nullptr, ST(stream_)));
    return;
  }
  if (!training) {
    // pre_norm = positioned + softmax(Q·Kᵀ / sqrt(query.cols)) · V
    // (attention.rs:243-253, 347-401) through oxf_attention_forward: three
    // launches by default, the fused form under OXF_ATTENTION=fused (then
    // p_ holds per-chunk exponentials, not probabilities; inference keeps
    // nothing for backward).
    const oxf_status st =
        oxf_attention_forward(q, k, v, pos_, pre_norm_, p_, stats_, batch, S, D, H,
                              1.0f / std::sqrt(static_cast<float>(D)), causal ? 1 : 0,
                              ST(stream_));
    check(st);
    check(oxf_norm_rows(cs(pre_norm_, T * H), ms(h1_, T * H), H, spec_.norm, 1e-5f, nullptr,
                        nullptr, ST(stream_)));
    return;
  }
  // scores = Q·Kᵀ / sqrt(query.cols) (attention.rs:359-374), per sequence
  Gemm(S, S, D, false, true, q, k, p_)
      .batch(batch, static_cast<long long>(S) * D, static_cast<long long>(S) * D,
             static_cast<long long>(S) * S)
      .alpha(1.0f / std::sqrt(static_cast<float>(D)))
      .run(stream_);
  // softmax rows, with the decoder's causal mask (attention.rs:347-357)
  check(oxf_matrix_softmax_rows(ms(p_, static_cast<size_t>(batch) * S * S), S, 1.0f,
                                causal ? S : 0, ST(stream_)));
  // pre_norm = positioned + P·V (attention.rs:243-253, 266-267)
  Gemm(S, H, S, false, false, p_, v, pre_norm_)
      .batch(batch, static_cast<long long>(S) * S, static_cast<long long>(S) * H,
             static_cast<long long>(S) * H)
      .residual(pos_, H, static_cast<long long>(S) * H)
      .run(stream_);
  // Post-Norm (Normalization::forward, attention.rs:157-162)
  check(oxf_norm_rows(cs(pre_norm_, T * H), ms(h1_, T * H), H, spec_.norm, 1e-5f, nullptr,
                      nullptr, ST(stream_)));
}

// Multi-head core: for each head j, a batched product over the sequences
// on column slices of Q, K, V (leading dimensions D and H, offsets j*hq and
// j*hv); the probabilities of head j occupy p_[j*batch*S*S, ...), so one
// softmax launch covers every head's rows. P·V adds the positioned input of
// the head's columns as the residual (attention.rs:249).
void TransformerEngine::attention_heads_forward(int batch, bool causal, bool training) {
  const int S = spec_.seq, H = spec_.hidden, D = spec_.q.out, h = heads_;
  const int hq = D / h, hv = H / h;
  const size_t T = static_cast<size_t>(batch) * S;
  const float* q = qkv_;
  const float* k = qkv_ + T * D;
  const float* v = qkv_ + 2 * T * D;
  if (!training) {
    // one fused launch: the scores stay on chip (head widths 32 / 64)
    const oxf_status st = oxf_attention_heads_forward(q, k, v, pos_, pre_norm_, batch, S, D, H,
                                                      h, causal ? 1 : 0, ST(stream_));
    if (st != OXF_ERR_UNSUPPORTED_SHAPE) {
      check(st);
      return;
    }
  }
  ensure_score_buffers();
  const long long sSS = static_cast<long long>(S) * S, sSD = static_cast<long long>(S) * D,
                  sSH = static_cast<long long>(S) * H, head = static_cast<long long>(batch) * sSS;
  for (int j = 0; j < h; ++j)
    Gemm(S, S, hq, false, true, q + j * hq, k + j * hq, p_ + j * head)
        .ld(D, D, S)
        .batch(batch, sSD, sSD, sSS)
        .alpha(1.0f / std::sqrt(static_cast<float>(hq)))
        .run(stream_);
  check(oxf_matrix_softmax_rows(ms(p_, static_cast<size_t>(h) * head), S, 1.0f,
                                causal ? S : 0, ST(stream_)));
  for (int j = 0; j < h; ++j)
    Gemm(S, hv, S, false, false, p_ + j * head, v + j * hv, pre_norm_ + j * hv)
        .ld(S, H, H)
        .batch(batch, sSS, sSH, sSH)
        .residual(pos_ + j * hv, H, sSH)
        .run(stream_);
}

// Backward of the multi-head core into dqkv_ (Attention::backward_self,
// attention.rs:297-308, per head): dP = dR·Vᵀ, dV = Pᵀ·dR, dS =
// softmax'(P, dP)/sqrt(hq) for every head in one launch, dQ = dS·K,
// dK = dSᵀ·Q, each written into the head's columns.
void TransformerEngine::attention_heads_backward(int batch) {
  const int S = spec_.seq, H = spec_.hidden, D = spec_.q.out, h = heads_;
  const int hq = D / h, hv = H / h;
  const size_t T = static_cast<size_t>(batch) * S;
  const float* q = qkv_;
  const float* k = qkv_ + T * D;
  const float* v = qkv_ + 2 * T * D;
  float* dq = dqkv_;
  float* dk = dqkv_ + T * D;
  float* dv = dqkv_ + 2 * T * D;
  const long long sSS = static_cast<long long>(S) * S, sSD = static_cast<long long>(S) * D,
                  sSH = static_cast<long long>(S) * H, head = static_cast<long long>(batch) * sSS;
  for (int j = 0; j < h; ++j) {
    Gemm(S, S, hv, false, true, dr_ + j * hv, v + j * hv, dp_ + j * head)
        .ld(H, H, S)
        .batch(batch, sSH, sSH, sSS)
        .run(stream_);
    Gemm(S, hv, S, true, false, p_ + j * head, dr_ + j * hv, dv + j * hv)
        .ld(S, H, H)
        .batch(batch, sSS, sSH, sSH)
        .run(stream_);
  }
  const size_t rows = static_cast<size_t>(h) * T;
  check(oxf_softmax_rows_backward(cs(p_, rows * S), cs(dp_, rows * S), ms(dp_, rows * S), S,
                                  1.0f / std::sqrt(static_cast<float>(hq)), ST(stream_)));
  for (int j = 0; j < h; ++j) {
    Gemm(S, hq, S, false, false, dp_ + j * head, k + j * hq, dq + j * hq)
        .ld(S, D, D)
        .batch(batch, sSS, sSD, sSD)
        .run(stream_);
    Gemm(S, hq, S, true, false, dp_ + j * head, q + j * hq, dk + j * hq)
        .ld(S, D, D)
        .batch(batch, sSS, sSD, sSD)
        .run(stream_);
  }
}

void TransformerEngine::forward(const float* x, int batch, bool causal) {
  forward_impl(x, batch, causal, false);
}

void TransformerEngine::forward_impl(const float* x, int batch, bool causal, bool training) {
  TimingScope timing_scope(this);
  require(batch >= 1 && batch <= max_batch_, "transformer: batch outside [1, max_batch]");
  batch_ = batch;
  trained_ = training;
  const int H = spec_.hidden;
  const size_t T = static_cast<size_t>(batch) * spec_.seq;
  attention_forward(x, batch, causal, training);
  // ffn + residual (inference.rs:90-101); inference keeps no pre-activations
  ffn_->forward(h1_, pre2_, T, h1_, stream_, training);
  check(oxf_norm_rows(cs(pre2_, T * H), ms(enc_, T * H), H, spec_.norm, 1e-5f, nullptr, nullptr,
                      ST(stream_)));
  // output Linear (inference.rs:102-107)
  const LayerSpec& o = spec_.o;
  Gemm g(static_cast<int>(T), o.out, H, false, false, enc_, params_ + off_o_, y_);
  if (o.bias) g.bias(params_ + off_o_ + static_cast<size_t>(o.in) * o.out);
  if (o.act) {
    if (training) g.pre_out(zo_, o.out);
    g.act(o.act);
  }
  g.run(stream_);
}

void TransformerEngine::train_forward(const float* x, int batch) {
  forward_impl(x, batch, false, true);
}

void TransformerEngine::set_target(const float* target) {
  const size_t T = static_cast<size_t>(batch_) * spec_.seq, O = spec_.o.out;
  check(oxf_mse_loss_grad(cs(y_, T * O), cs(target, T * O), ms(loss_, T), ms(dy_, T * O), O,
                          ST(stream_)));
}

void TransformerEngine::set_output_gradient(const float* dy) {
  const size_t T = static_cast<size_t>(batch_) * spec_.seq, O = spec_.o.out;
  copy_d2d(dy_, dy, T * O, stream_);
}

void TransformerEngine::bucket(int stage, size_t* offset, size_t* count) const {
  if (stage == 0) {
    *offset = off_o_;
    *count = nparams_ - off_o_;
  } else if (stage == 1) {
    *offset = off_ffn_;
    *count = off_o_ - off_ffn_;
  } else {
    *offset = 0;
    *count = off_ffn_;
  }
}

void TransformerEngine::backward_stage(int stage) {
  TimingScope timing_scope(this);
  const int S = spec_.seq, H = spec_.hidden, D = spec_.q.out;
  const int batch = batch_;
  require(batch >= 1, "backward before forward");
  require(trained_, "backward needs the training forward (train_forward), not the inference one");
  const size_t T = static_cast<size_t>(batch) * S;
  const int Ti = static_cast<int>(T);
  const LayerSpec& o = spec_.o;
  const size_t O = o.out;
  if (stage == 0) {
    // Output Linear backward (encoder.rs:140-167; linear.rs:246-275,
    // 373-391, 431-434): G = dY ⊙ act'(Z); dWo += encᵀ·G; dbo += colsum(G);
    // d_enc = G·Woᵀ with the old Wo.
    if (o.act)
      check(oxf_slice_mul_act_derivative(ms(dy_, T * O), cs(zo_, T * O),
                                         static_cast<oxf_activation>(o.act), ST(stream_)));
    Gemm(H, o.out, Ti, true, false, enc_, dy_, grads_ + off_o_).accumulate().run(stream_);
    if (o.bias)
      check(oxf_matrix_sum_cols(cs(dy_, T * O), ms(grads_ + off_o_ + static_cast<size_t>(H) * O, O),
                                O, 1, ST(stream_)));
    Gemm(Ti, H, o.out, false, true, dy_, params_ + off_o_, denc_).run(stream_);
  } else if (stage == 1) {
    // second Post-Norm backward, then the feed-forward (encoder.rs:169-176);
    // d1 = d2 + dFFN/dh1 (encoder.rs:175-176) fused into the last dX GEMM.
    check(oxf_norm_rows_backward(cs(pre2_, T * H), cs(denc_, T * H), ms(d2_, T * H), H,
                                 spec_.norm, 1e-5f, ST(stream_)));
    ffn_->backward(d2_, d1_, T, d2_, stream_);
  } else {
    // Attention::backward_self (attention.rs:283-321)
    const float* q = qkv_;
    const float* k = qkv_ + T * D;
    const float* v = qkv_ + 2 * T * D;
    float* dq = dqkv_;
    float* dk = dqkv_ + T * D;
    float* dv = dqkv_ + 2 * T * D;
    const long long sSS = static_cast<long long>(S) * S, sSH = static_cast<long long>(S) * H,
                    sSD = static_cast<long long>(S) * D;
    check(oxf_norm_rows_backward(cs(pre_norm_, T * H), cs(d1_, T * H), ms(dr_, T * H), H,
                                 spec_.norm, 1e-5f, ST(stream_)));
    if (heads_ > 1) {
      attention_heads_backward(batch);
    } else {
      // dP = dR·Vᵀ, dV = Pᵀ·dR (attention.rs:297-300)
      Gemm(S, S, H, false, true, dr_, v, dp_).batch(batch, sSH, sSH, sSS).run(stream_);
      Gemm(S, H, S, true, false, p_, dr_, dv).batch(batch, sSS, sSH, sSH).run(stream_);
      // dS = softmax'(P, dP) / sqrt(d) (attention.rs:302-304), in place
      check(oxf_softmax_rows_backward(cs(p_, T * S), cs(dp_, T * S), ms(dp_, T * S), S,
                                      1.0f / std::sqrt(static_cast<float>(D)), ST(stream_)));
      // dQ = dS·K, dK = dSᵀ·Q (attention.rs:306-308)
      Gemm(S, D, S, false, false, dp_, k, dq).batch(batch, sSS, sSD, sSD).run(stream_);
      Gemm(S, D, S, true, false, dp_, q, dk).batch(batch, sSS, sSD, sSD).run(stream_);
    }
    // QkvProjection::backward_self (attention.rs:104-144)
    const LayerSpec* ls[3] = {&spec_.q, &spec_.k, &spec_.v};
    const size_t offs[3] = {off_q_, off_k_, off_v_};
    float* ds[3] = {dq, dk, dv};
    for (int j = 0; j < 3; ++j)
      if (ls[j]->act)
        check(oxf_slice_mul_act_derivative(
            ms(ds[j], T * ls[j]->out), cs(qkv_pre_ + (ds[j] - dqkv_), T * ls[j]->out),
            static_cast<oxf_activation>(ls[j]->act), ST(stream_)));
    const bool uniform = spec_.q.out == spec_.v.out && !spec_.q.bias && !spec_.k.bias &&
                         !spec_.v.bias;
    if (uniform) {
      Gemm(H, D, Ti, true, false, pos_, dqkv_, grads_ + off_q_)
          .batch(3, 0, static_cast<long long>(T) * D, static_cast<long long>(spec_.q.param_count()))
          .accumulate()
          .run(stream_);
    } else {
      for (int j = 0; j < 3; ++j) {
        Gemm(H, ls[j]->out, Ti, true, false, pos_, ds[j], grads_ + offs[j]).accumulate().run(stream_);
        if (ls[j]->bias)
          check(oxf_matrix_sum_cols(cs(ds[j], T * ls[j]->out),
                                    ms(grads_ + offs[j] + static_cast<size_t>(H) * ls[j]->out,
                                       ls[j]->out),
                                    ls[j]->out, 1, ST(stream_)));
      }
    }
    // d_positioned = dR + Σ_j dProj_j · W_jᵀ (attention.rs:127-131, 318-319):
    // one batch-reduce GEMM over the three projections when they share a
    // layout, otherwise three GEMMs accumulating through beta = 1.
    if (uniform) {
      Gemm g(Ti, H, D, false, true, dqkv_, params_ + off_q_, dpos_);
      g.batch(3, static_cast<long long>(T) * D, static_cast<long long>(spec_.q.param_count()), 0)
          .reduce_batch()
          .residual(dr_, H)
          .run(stream_);
    } else {
      for (int j = 0; j < 3; ++j) {
        Gemm g(Ti, H, ls[j]->out, false, true, ds[j], params_ + offs[j], dpos_);
        if (j == 0) g.residual(dr_, H);
        else g.beta(1.0f);
        g.run(stream_);
      }
    }
    // position gradient: sum over the batch (encoder.rs:180-184)
    check(oxf_matrix_sum_cols(cs(dpos_, T * H), ms(grads_ + off_pos_, static_cast<size_t>(S) * H),
                              static_cast<size_t>(S) * H, 1, ST(stream_)));
  }
}

void TransformerEngine::zero_grads() {
  check_cuda_call(cudaMemsetAsync(grads_, 0, nparams_ * 4, stream_), "memset");
}

void TransformerEngine::sgd(float lr) {
  check(oxf_sgd_update(ms(params_, nparams_), cs(grads_, nparams_), lr, ST(stream_)));
}

}  // namespace oxf
