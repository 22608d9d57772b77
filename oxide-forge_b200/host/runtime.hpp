// runtime.hpp — C++ host layer mirroring OxideForge's CudaRuntime and its
// containers (src/cuda/runtime.rs, src/cuda/container/*.rs, docs/api.md).
//
// Ownership follows the reference: CudaRuntime hands out device buffers from
// an exact-size pool (runtime.rs:47-110); Matrix / Vector own a buffer and
// return it to the pool when destroyed (the reference recycles explicitly
// with recycle_matrix, matrix.rs:255-258, and frees on Drop); views borrow.
// Work is submitted asynchronously on the runtime's primary stream or on
// extra streams forked from it (runtime.rs:188-211). Every device operation
// goes through the C ABI in include/oxf.h.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "oxf.h"

namespace oxf {

class Error : public std::runtime_error {
 public:
  Error(oxf_status st, const std::string& msg) : std::runtime_error(msg), status(st) {}
  oxf_status status;
};

// Throws Error for a non-OK status (message from oxf_last_error_string()).
void check(oxf_status st);
void check_cuda_call(cudaError_t e, const char* what);
// The reference asserts shapes with assert!/assert_eq! (panic); here the
// same checks throw Error(OXF_ERR_INVALID_ARG).
void require(bool cond, const char* what);

enum class BinaryOp : int { Add = OXF_ADD, Sub = OXF_SUB, Mul = OXF_MUL, Div = OXF_DIV };
enum class Activation : int {
  Identity = OXF_ACT_IDENTITY,
  Gelu = OXF_ACT_GELU,
  Relu = OXF_ACT_RELU,
  Silu = OXF_ACT_SILU
};
// InitType, runtime.rs:6-22. Random fills from a seeded host RNG instead of
// the reference's unseeded device hash (common.rs:3-9).
enum class InitType { Sequence, Reserve, Random, Zero };

class CudaRuntime;

// A pool-backed f32 device buffer (cuda_core::DeviceBuffer<f32>).
class DeviceBuffer {
 public:
  DeviceBuffer() = default;
  DeviceBuffer(CudaRuntime* owner, float* ptr, size_t len) : owner_(owner), ptr_(ptr), len_(len) {}
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  DeviceBuffer(DeviceBuffer&& o) noexcept { swap(o); }
  DeviceBuffer& operator=(DeviceBuffer&& o) noexcept {
    reset();
    swap(o);
    return *this;
  }
  ~DeviceBuffer() { reset(); }

  float* data() const { return ptr_; }
  size_t len() const { return len_; }
  bool empty() const { return len_ == 0; }
  // Returns the pointer to the owner's pool (or forgets a borrowed one).
  void reset();
  // Gives up ownership without recycling; returns the raw pointer.
  float* release() {
    float* p = ptr_;
    owner_ = nullptr;
    ptr_ = nullptr;
    len_ = 0;
    return p;
  }

 private:
  void swap(DeviceBuffer& o) noexcept {
    std::swap(owner_, o.owner_);
    std::swap(ptr_, o.ptr_);
    std::swap(len_, o.len_);
  }
  CudaRuntime* owner_ = nullptr;  // nullptr: borrowed, never freed here
  float* ptr_ = nullptr;
  size_t len_ = 0;
};

class Vector;

// Row-major f32 matrix (container.rs:22-25).
class Matrix {
 public:
  Matrix() = default;
  Matrix(DeviceBuffer buf, size_t rows, size_t cols);
  // A borrowed view of caller-owned device memory.
  static Matrix view(float* ptr, size_t rows, size_t cols);

  size_t rows() const { return rows_; }
  size_t cols() const { return cols_; }
  size_t len() const { return buf_.len(); }
  float* data() const { return buf_.data(); }
  oxf_slice slice() const { return {buf_.data(), buf_.len()}; }
  oxf_cslice cslice() const { return {buf_.data(), buf_.len()}; }
  DeviceBuffer& buffer() { return buf_; }

  std::vector<float> to_host(const CudaRuntime& rt) const;  // matrix.rs:11-13

  // Mutating operations (docs/api.md: they belong to Matrix).
  void scale(float value, const CudaRuntime& rt, cudaStream_t s = nullptr);       // matrix.rs:30
  void add_scalar(float value, const CudaRuntime& rt, cudaStream_t s = nullptr);  // matrix.rs:34
  void activate(Activation act, const CudaRuntime& rt, cudaStream_t s = nullptr);
  void activate_derivative(Activation act, const CudaRuntime& rt, cudaStream_t s = nullptr);
  void binary_assign(const Matrix& rhs, BinaryOp op, const CudaRuntime& rt,
                     cudaStream_t s = nullptr);  // matrix.rs:38-64
  void binary_assign_by_rows(const Vector& v, BinaryOp op, const CudaRuntime& rt,
                             cudaStream_t s = nullptr);  // rows.rs:8-42
  void causal_mask(const CudaRuntime& rt, cudaStream_t s = nullptr);  // matrix.rs:79-92
  void softmax_rows(const CudaRuntime& rt, cudaStream_t s = nullptr);  // norm.rs:8-24
  void layer_norm(const CudaRuntime& rt, cudaStream_t s = nullptr);    // norm.rs:26-48
  void rms_norm(const CudaRuntime& rt, cudaStream_t s = nullptr);      // norm.rs:50-70

 private:
  DeviceBuffer buf_;
  size_t rows_ = 0, cols_ = 0;
};

// f32 vector (container.rs:13-15).
class Vector {
 public:
  Vector() = default;
  explicit Vector(DeviceBuffer buf) : buf_(std::move(buf)) {}
  static Vector view(float* ptr, size_t len);
  size_t len() const { return buf_.len(); }
  float* data() const { return buf_.data(); }
  oxf_slice slice() const { return {buf_.data(), buf_.len()}; }
  oxf_cslice cslice() const { return {buf_.data(), buf_.len()}; }
  std::vector<float> to_host(const CudaRuntime& rt) const;
  void scale(float value, const CudaRuntime& rt, cudaStream_t s = nullptr);  // vector.rs
  void binary_assign(const Vector& rhs, BinaryOp op, const CudaRuntime& rt,
                     cudaStream_t s = nullptr);
  float sum(CudaRuntime& rt) const;  // span.rs:285-287 (synchronises)
  float max(CudaRuntime& rt) const;  // span.rs:289-291 (synchronises)

 private:
  DeviceBuffer buf_;
};

// CudaRuntime, runtime.rs:24-212.
class CudaRuntime {
 public:
  // device: CUDA ordinal (the reference hard-codes 0, runtime.rs:35);
  // stream: borrow this stream as the primary stream, or nullptr to create
  // a non-blocking one.
  explicit CudaRuntime(int device = 0, cudaStream_t stream = nullptr);
  ~CudaRuntime();
  CudaRuntime(const CudaRuntime&) = delete;
  CudaRuntime& operator=(const CudaRuntime&) = delete;

  int device() const { return device_; }
  cudaStream_t stream() const { return stream_; }
  void sync() const;  // runtime.rs:112-114

  // Exact-size pool (runtime.rs:47-110).
  DeviceBuffer get_uninit_buffer(size_t len);
  DeviceBuffer get_zerod_buffer(size_t len);
  void reserve_buffers(size_t len, size_t count);
  void recycle_buffer(DeviceBuffer&& buf);
  void recycle_matrix(Matrix&& m) { recycle_buffer(std::move(m.buffer())); }
  size_t pooled_buffers() const;
  void release_pool();  // frees every pooled buffer (no reference counterpart)

  // Streams (runtime.rs:188-211). Extra streams are owned by the runtime.
  std::vector<cudaStream_t> create_extra_streams(size_t count);
  void fork_streams(const std::vector<cudaStream_t>& streams) const;
  void join_streams(const std::vector<cudaStream_t>& streams) const;
  void sync_streams(const std::vector<cudaStream_t>& streams) const;

  // Allocating operations (docs/api.md: they belong to CudaRuntime).
  Matrix new_matrix(InitType init, size_t rows, size_t cols, unsigned long long seed = 0);
  Matrix new_uninit_matrix(size_t rows, size_t cols);
  Matrix matrix_from_host(const float* values, size_t rows, size_t cols);  // matrix.rs:96-111
  Vector vector_from_host(const float* values, size_t len);
  Matrix clone_matrix(const Matrix& m, cudaStream_t s = nullptr);  // matrix.rs:313-325
  Vector clone_vector(const Vector& v, cudaStream_t s = nullptr);
  Matrix matrix_multiply(const Matrix& a, const Matrix& b, cudaStream_t s = nullptr);  // :113-131
  Matrix matrix_binary(const Matrix& a, const Matrix& b, BinaryOp op, cudaStream_t s = nullptr);
  Matrix matrix_add(const Matrix& a, const Matrix& b) { return matrix_binary(a, b, BinaryOp::Add); }
  Matrix matrix_sub(const Matrix& a, const Matrix& b) { return matrix_binary(a, b, BinaryOp::Sub); }
  Matrix matrix_mul(const Matrix& a, const Matrix& b) { return matrix_binary(a, b, BinaryOp::Mul); }
  Matrix matrix_div(const Matrix& a, const Matrix& b) { return matrix_binary(a, b, BinaryOp::Div); }
  Matrix matrix_transpose(const Matrix& m, cudaStream_t s = nullptr);  // convert.rs:17-63
  Vector matrix_sum_rows(const Matrix& m, cudaStream_t s = nullptr);   // rows.rs:46-88
  Vector matrix_sum_cols(const Matrix& m, cudaStream_t s = nullptr);
  Matrix softmax_rows_backward(const Matrix& p, const Matrix& dy);     // norm.rs:73-101
  Matrix layer_norm_backward(const Matrix& x, const Matrix& dy);       // norm.rs:103-127
  Matrix rms_norm_backward(const Matrix& x, const Matrix& dy);         // norm.rs:129-158

  cudaStream_t pick(cudaStream_t s) const { return s ? s : stream_; }
  // Puts a raw pool pointer of `len` floats back (DeviceBuffer::reset).
  void pool_push(float* p, size_t len) {
    if (p && len) pool_[len].push_back(p);
  }

 private:
  int device_ = 0;
  cudaStream_t stream_ = nullptr;
  bool own_stream_ = false;
  std::unordered_map<size_t, std::vector<float*>> pool_;
  std::vector<cudaStream_t> extra_;
};

inline oxf_stream ST(cudaStream_t s) { return reinterpret_cast<oxf_stream>(s); }

}  // namespace oxf
