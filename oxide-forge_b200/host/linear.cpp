// linear.cpp — Linear over the runtime containers (see linear.hpp).
#include "linear.hpp"

namespace oxf {

namespace {

// The side stream (if any) waits for the primary stream; returns the stream
// the work goes on (linear.rs:124-126 `stream.join(runtime.stream())`).
cudaStream_t on(const CudaRuntime& rt, cudaStream_t s) {
  if (s && s != rt.stream()) rt.fork_streams({s});
  return rt.pick(s);
}

void same_shape(const Matrix& a, const Matrix& b, const char* what) {
  require(a.rows() == b.rows() && a.cols() == b.cols(), what);
}

}  // namespace

Linear::Linear(Matrix weights, std::optional<Vector> bias, Activation activation)
    : weights_(std::move(weights)), bias_(std::move(bias)), activation_(activation) {
  require(weights_.rows() > 0 && weights_.cols() > 0, "Linear: empty weight matrix");
  if (bias_) require(bias_->len() == weights_.cols(), "Linear: bias length != output neurons");
}

// Linear::affine_on (linear.rs:185-206) and activate_on (:225-230) as one
// GEMM: C = input·W, + bias by rows, + residual, [pre-activation stored],
// activation; the epilogue applies them in that order.
void Linear::affine_on(const Matrix& input, const Matrix* residual, Matrix& output, Matrix* pre,
                       bool activate, cudaStream_t s) const {
  require(input.cols() == weights_.rows(), "Linear: input.cols != input neurons");  // :123
  require(output.rows() == input.rows() && output.cols() == weights_.cols(),
          "Linear: output shape");  // :193-194
  if (residual) same_shape(output, *residual, "Linear: residual shape != output shape");
  if (pre) same_shape(output, *pre, "Linear: pre-activation shape != output shape");
  if (input.rows() == 0) return;
  oxf_gemm_desc d;
  oxf_gemm_desc_init(&d, static_cast<int>(input.rows()), static_cast<int>(weights_.cols()),
                     static_cast<int>(weights_.rows()), 0, 0, input.data(), weights_.data(),
                     output.data());
  if (bias_) d.bias = bias_->data();
  if (residual) {
    d.residual = residual->data();
    d.ldr = static_cast<long long>(residual->cols());
  }
  if (activate && activation_ != Activation::Identity) {
    d.act = static_cast<int>(activation_);
    if (pre) {
      d.pre_out = pre->data();
      d.ldp = static_cast<long long>(pre->cols());
    }
  }
  check(oxf_gemm(&d, ST(s)));
  if (pre && !(activate && activation_ != Activation::Identity) && pre->data() != output.data() &&
      output.len())
    check_cuda_call(cudaMemcpyAsync(pre->data(), output.data(), output.len() * sizeof(float),
                                    cudaMemcpyDeviceToDevice, s),
                    "cudaMemcpyAsync D2D");
}

Matrix Linear::forward(const Matrix& input, const Matrix* residual, CudaRuntime& rt,
                       cudaStream_t stream) const {
  require(input.cols() == weights_.rows(), "Linear::forward: input.cols != input neurons");
  Matrix out = rt.new_uninit_matrix(input.rows(), weights_.cols());
  affine_on(input, residual, out, nullptr, true, on(rt, stream));
  return out;
}

Matrix Linear::affine(const Matrix& input, const Matrix* residual, CudaRuntime& rt,
                      cudaStream_t stream) const {
  require(input.cols() == weights_.rows(), "Linear::affine: input.cols != input neurons");
  Matrix out = rt.new_uninit_matrix(input.rows(), weights_.cols());
  affine_on(input, residual, out, nullptr, false, on(rt, stream));
  return out;
}

void Linear::activate(Matrix& output, const CudaRuntime& rt, cudaStream_t stream) const {
  if (activation_ == Activation::Identity || output.len() == 0) return;
  output.activate(activation_, rt, stream);
}

void Linear::forward_into(const Matrix& input, const Matrix* residual, Matrix& output,
                          Matrix* pre_activation, const CudaRuntime& rt,
                          cudaStream_t stream) const {
  affine_on(input, residual, output, pre_activation, true, on(rt, stream));
}

void Linear::backward_into(const Matrix* pre_activation, const Matrix& output_gradient,
                           const Matrix* residual_gradient, Matrix& gradient,
                           Vector* bias_gradient, const CudaRuntime& rt,
                           cudaStream_t stream) const {
  const cudaStream_t s = on(rt, stream);
  require(output_gradient.cols() == weights_.cols(), "Linear::backward: gradient.cols != outputs");
  same_shape(gradient, output_gradient, "Linear::backward: output gradient shape");
  if (residual_gradient)
    same_shape(*residual_gradient, output_gradient,
               "Linear::backward_with_res: residual gradient shape");  // :458-461
  const bool act = activation_ != Activation::Identity;
  if (act) {
    require(pre_activation != nullptr, "activation backward requires pre-activation");  // :251
    same_shape(*pre_activation, output_gradient, "Linear::backward: pre-activation shape");
  }
  if (bias_) {
    require(bias_gradient != nullptr, "Linear::backward: a biased Linear needs a bias gradient");
    require(bias_gradient->len() == weights_.cols(), "Linear::backward: bias gradient length");
  }
  const size_t n = output_gradient.len();
  if (n == 0) return;
  // G = dY (+ dR), then ⊙ act'(Z) in place
  if (residual_gradient)
    check(oxf_slice_binary(output_gradient.cslice(), residual_gradient->cslice(), gradient.slice(),
                           OXF_ADD, ST(s)));
  else if (gradient.data() != output_gradient.data())
    check_cuda_call(cudaMemcpyAsync(gradient.data(), output_gradient.data(), n * sizeof(float),
                                    cudaMemcpyDeviceToDevice, s),
                    "cudaMemcpyAsync D2D");
  if (act)
    check(oxf_slice_mul_act_derivative(gradient.slice(), pre_activation->cslice(),
                                       static_cast<oxf_activation>(activation_), ST(s)));
  // bias gradient: column sums of G (the reference sums the rows of Gᵀ)
  if (bias_)
    check(oxf_matrix_sum_cols(gradient.cslice(), bias_gradient->slice(), gradient.cols(), 0,
                              ST(s)));
}

std::pair<Matrix, std::optional<Vector>> Linear::backward(const Matrix* pre_activation,
                                                          const Matrix& output_gradient,
                                                          CudaRuntime& rt,
                                                          cudaStream_t stream) const {
  Matrix g = rt.new_uninit_matrix(output_gradient.rows(), output_gradient.cols());
  std::optional<Vector> bg;
  if (bias_) bg.emplace(rt.get_uninit_buffer(weights_.cols()));
  backward_into(pre_activation, output_gradient, nullptr, g, bg ? &*bg : nullptr, rt, stream);
  return {std::move(g), std::move(bg)};
}

std::pair<Matrix, std::optional<Vector>> Linear::backward_with_res(
    const Matrix& pre_activation, const Matrix& output_gradient, const Matrix& residual_gradient,
    CudaRuntime& rt, cudaStream_t stream) const {
  same_shape(pre_activation, output_gradient, "Linear::backward_with_res: pre-activation shape");
  Matrix g = rt.new_uninit_matrix(output_gradient.rows(), output_gradient.cols());
  std::optional<Vector> bg;
  if (bias_) bg.emplace(rt.get_uninit_buffer(weights_.cols()));
  backward_into(&pre_activation, output_gradient, &residual_gradient, g, bg ? &*bg : nullptr, rt,
                stream);
  return {std::move(g), std::move(bg)};
}

Vector Linear::loss_rows(const Matrix& output, const Matrix& target, CudaRuntime& rt,
                         cudaStream_t stream) {
  same_shape(output, target, "Linear::loss_rows: output and target shapes differ");
  Vector out(rt.get_uninit_buffer(output.rows()));
  if (output.rows() == 0) return out;
  require(output.cols() > 0, "Linear::loss_rows: cols must be > 0");
  check(oxf_loss_rows(output.cslice(), target.cslice(), out.slice(), output.cols(),
                      ST(on(rt, stream))));
  return out;
}

void Linear::learn(const Matrix& input, const Matrix& gradient, const Vector* bias_gradient,
                   float learning_rate, const CudaRuntime& rt, cudaStream_t stream) {
  const cudaStream_t s = on(rt, stream);
  require(input.cols() == weights_.rows(), "Linear::learn: input.cols != input neurons");
  require(gradient.cols() == weights_.cols(), "Linear::learn: gradient.cols != output neurons");
  require(input.rows() == gradient.rows(), "Linear::learn: input and gradient rows differ");
  if (bias_) {
    require(bias_gradient != nullptr, "missing bias gradient for biased Linear");  // :394
    require(bias_gradient->len() == bias_->len(), "Linear::learn: bias gradient length");
  }
  if (input.rows() > 0) {
    // W = (-lr)·(inputᵀ·G) + W: the epilogue scales the product and adds it
    // to W, the reference's scale-then-subtract in one pass.
    oxf_gemm_desc d;
    oxf_gemm_desc_init(&d, static_cast<int>(weights_.rows()), static_cast<int>(weights_.cols()),
                       static_cast<int>(input.rows()), 1, 0, input.data(), gradient.data(),
                       weights_.data());
    d.alpha = -learning_rate;
    d.beta = 1.0f;
    check(oxf_gemm(&d, ST(s)));
  }
  if (bias_) check(oxf_sgd_update(bias_->slice(), bias_gradient->cslice(), learning_rate, ST(s)));
}

void Linear::input_gradient_into(const Matrix& gradient, Matrix& out, const CudaRuntime& rt,
                                 cudaStream_t stream) const {
  require(gradient.cols() == weights_.cols(), "Linear::input_gradient: gradient.cols");  // :423
  require(out.rows() == gradient.rows() && out.cols() == weights_.rows(),
          "Linear::input_gradient: output shape");
  if (gradient.rows() == 0) return;
  oxf_gemm_desc d;
  oxf_gemm_desc_init(&d, static_cast<int>(gradient.rows()), static_cast<int>(weights_.rows()),
                     static_cast<int>(weights_.cols()), 0, 1, gradient.data(), weights_.data(),
                     out.data());
  check(oxf_gemm(&d, ST(on(rt, stream))));
}

Matrix Linear::input_gradient(const Matrix& gradient, CudaRuntime& rt, cudaStream_t stream) const {
  Matrix out = rt.new_uninit_matrix(gradient.rows(), weights_.rows());
  input_gradient_into(gradient, out, rt, stream);
  return out;
}

}  // namespace oxf
