// linear.hpp — Linear (src/net/linear.rs:72-533) over the CudaRuntime
// containers of runtime.hpp: one fully connected layer, weights [in, out]
// row-major, optional bias [out], an Activation.
//
// Same methods, argument meaning and order of arithmetic as the reference;
// each call is a fused launch instead of the reference's chain:
//   forward / affine  one GEMM, bias + residual (+ activation) in its epilogue
//                     (the reference: GEMM, row-broadcast add, add, for_each)
//   backward          dY ⊙ act'(Z) in one pass over a copy of dY, bias
//                     gradient as a column sum (the reference clones Z,
//                     differentiates, multiplies, transposes G, sums rows)
//   learn             W += (-lr)·XᵀG as one GEMM reading X in place (alpha
//                     -lr, beta 1 into W; the reference transposes X,
//                     multiplies, scales, subtracts); b -= lr·db, one pass
//   input_gradient    G·Wᵀ as one GEMM reading W in place (no transpose)
// Methods returning a Matrix take it from the runtime's exact-size pool, as
// the reference's do. A non-null stream is first made to wait for the
// runtime's primary stream and the work runs there (the reference's
// `stream.join(runtime.stream())`); null runs on the primary stream.
#pragma once
#include <optional>
#include <utility>

#include "runtime.hpp"

namespace oxf {

class Linear {
 public:
  // Linear::new (linear.rs:89-95).
  Linear(Matrix weights, std::optional<Vector> bias, Activation activation);

  size_t input_neurons() const { return weights_.rows(); }
  size_t output_neurons() const { return weights_.cols(); }
  Activation activation() const { return activation_; }
  const Matrix& weights() const { return weights_; }
  Matrix& weights() { return weights_; }
  const Vector* bias() const { return bias_ ? &*bias_ : nullptr; }
  Vector* bias() { return bias_ ? &*bias_ : nullptr; }
  bool needs_pre_activation() const { return activation_ != Activation::Identity; }  // :308

  // Linear::forward (linear.rs:116-132): act(input·W + bias + residual).
  Matrix forward(const Matrix& input, const Matrix* residual, CudaRuntime& rt,
                 cudaStream_t stream = nullptr) const;
  // Linear::affine (linear.rs:157-173): input·W + bias + residual.
  Matrix affine(const Matrix& input, const Matrix* residual, CudaRuntime& rt,
                cudaStream_t stream = nullptr) const;
  // Linear::activate (linear.rs:208-230), in place.
  void activate(Matrix& output, const CudaRuntime& rt, cudaStream_t stream = nullptr) const;
  // forward into caller-provided outputs; pre_activation (optional, same
  // shape as output) receives input·W + bias + residual.
  void forward_into(const Matrix& input, const Matrix* residual, Matrix& output,
                    Matrix* pre_activation, const CudaRuntime& rt,
                    cudaStream_t stream = nullptr) const;

  // Linear::backward (linear.rs:232-306): G = dY ⊙ act'(Z) and, with a
  // bias, its column sums. pre_activation may be null for Identity.
  std::pair<Matrix, std::optional<Vector>> backward(const Matrix* pre_activation,
                                                    const Matrix& output_gradient,
                                                    CudaRuntime& rt,
                                                    cudaStream_t stream = nullptr) const;
  // Linear::backward_with_res (linear.rs:446-533): G = (dY + dR) ⊙ act'(Z).
  std::pair<Matrix, std::optional<Vector>> backward_with_res(const Matrix& pre_activation,
                                                             const Matrix& output_gradient,
                                                             const Matrix& residual_gradient,
                                                             CudaRuntime& rt,
                                                             cudaStream_t stream = nullptr) const;
  // backward into caller-provided outputs (residual_gradient and
  // bias_gradient optional).
  void backward_into(const Matrix* pre_activation, const Matrix& output_gradient,
                     const Matrix* residual_gradient, Matrix& gradient, Vector* bias_gradient,
                     const CudaRuntime& rt, cudaStream_t stream = nullptr) const;

  // Linear::loss_rows (linear.rs:312-348): per row mean of 0.5 (y - t)^2.
  static Vector loss_rows(const Matrix& output, const Matrix& target, CudaRuntime& rt,
                          cudaStream_t stream = nullptr);

  // Linear::learn (linear.rs:350-415): W -= lr·inputᵀ·G; b -= lr·bias_gradient.
  void learn(const Matrix& input, const Matrix& gradient, const Vector* bias_gradient,
             float learning_rate, const CudaRuntime& rt, cudaStream_t stream = nullptr);

  // Linear::input_gradient (linear.rs:417-446): G·Wᵀ.
  Matrix input_gradient(const Matrix& gradient, CudaRuntime& rt,
                        cudaStream_t stream = nullptr) const;
  void input_gradient_into(const Matrix& gradient, Matrix& out, const CudaRuntime& rt,
                           cudaStream_t stream = nullptr) const;

 private:
  void affine_on(const Matrix& input, const Matrix* residual, Matrix& output, Matrix* pre,
                 bool activate, cudaStream_t s) const;
  Matrix weights_;
  std::optional<Vector> bias_;
  Activation activation_;
};

}  // namespace oxf
