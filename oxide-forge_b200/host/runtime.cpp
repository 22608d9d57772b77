// runtime.cpp — CudaRuntime, DeviceBuffer, Matrix and Vector (see runtime.hpp).
#include "runtime.hpp"

#include <cstring>
#include <random>

namespace oxf {

void check(oxf_status st) {
  if (st != OXF_OK) throw Error(st, oxf_last_error_string());
}

void check_cuda_call(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Error(OXF_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

void require(bool cond, const char* what) {
  if (!cond) throw Error(OXF_ERR_INVALID_ARG, what);
}

// ---------------------------------------------------------------- DeviceBuffer
void DeviceBuffer::reset() {
  CudaRuntime* owner = owner_;
  const size_t n = len_;
  float* p = release();
  if (owner) owner->pool_push(p, n);
}

// ---------------------------------------------------------------- CudaRuntime
CudaRuntime::CudaRuntime(int device, cudaStream_t stream) : device_(device) {
  check_cuda_call(cudaSetDevice(device), "cudaSetDevice");
  if (stream) {
    stream_ = stream;
  } else {
    check_cuda_call(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking),
                    "cudaStreamCreate");
    own_stream_ = true;
  }
}

CudaRuntime::~CudaRuntime() {
  cudaSetDevice(device_);
  cudaStreamSynchronize(stream_);
  for (cudaStream_t s : extra_) {
    cudaStreamSynchronize(s);
    cudaStreamDestroy(s);
  }
  release_pool();
  if (own_stream_) cudaStreamDestroy(stream_);
}

void CudaRuntime::sync() const { check_cuda_call(cudaStreamSynchronize(stream_), "sync"); }

DeviceBuffer CudaRuntime::get_uninit_buffer(size_t len) {
  if (len > 0) {
    auto it = pool_.find(len);
    if (it != pool_.end() && !it->second.empty()) {
      float* p = it->second.back();
      it->second.pop_back();
      return DeviceBuffer(this, p, len);
    }
  }
  if (len == 0) return DeviceBuffer(this, nullptr, 0);
  void* p = nullptr;
  check_cuda_call(cudaMallocAsync(&p, len * sizeof(float), stream_), "cudaMallocAsync");
  return DeviceBuffer(this, static_cast<float*>(p), len);
}

DeviceBuffer CudaRuntime::get_zerod_buffer(size_t len) {
  DeviceBuffer b = get_uninit_buffer(len);
  if (len) check_cuda_call(cudaMemsetAsync(b.data(), 0, len * sizeof(float), stream_), "memset");
  return b;
}

void CudaRuntime::reserve_buffers(size_t len, size_t count) {
  if (len == 0) return;
  auto& v = pool_[len];
  while (v.size() < count) {
    void* p = nullptr;
    check_cuda_call(cudaMallocAsync(&p, len * sizeof(float), stream_), "cudaMallocAsync");
    v.push_back(static_cast<float*>(p));
  }
}

void CudaRuntime::recycle_buffer(DeviceBuffer&& buf) {
  // Stream-ordered reuse: every pending use of the buffer must be ordered
  // on the primary stream (runtime.rs:93-97).
  const size_t n = buf.len();
  pool_push(buf.release(), n);
}

size_t CudaRuntime::pooled_buffers() const {
  size_t n = 0;
  for (auto& kv : pool_) n += kv.second.size();
  return n;
}

void CudaRuntime::release_pool() {
  for (auto& kv : pool_)
    for (float* p : kv.second) cudaFreeAsync(p, stream_);
  pool_.clear();
  cudaStreamSynchronize(stream_);
}

std::vector<cudaStream_t> CudaRuntime::create_extra_streams(size_t count) {
  std::vector<cudaStream_t> out;
  for (size_t i = 0; i < count; ++i) {
    cudaStream_t s;
    check_cuda_call(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
    extra_.push_back(s);
    out.push_back(s);
  }
  fork_streams(out);  // a forked stream sees work queued before the fork
  return out;
}

namespace {
void stream_wait(cudaStream_t waiter, cudaStream_t on) {
  cudaEvent_t ev;
  check_cuda_call(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "cudaEventCreate");
  check_cuda_call(cudaEventRecord(ev, on), "cudaEventRecord");
  check_cuda_call(cudaStreamWaitEvent(waiter, ev, 0), "cudaStreamWaitEvent");
  cudaEventDestroy(ev);
}
}  // namespace

void CudaRuntime::fork_streams(const std::vector<cudaStream_t>& streams) const {
  for (cudaStream_t s : streams) stream_wait(s, stream_);
}

void CudaRuntime::join_streams(const std::vector<cudaStream_t>& streams) const {
  for (cudaStream_t s : streams) stream_wait(stream_, s);
}

void CudaRuntime::sync_streams(const std::vector<cudaStream_t>& streams) const {
  join_streams(streams);
  sync();
}

Matrix CudaRuntime::new_uninit_matrix(size_t rows, size_t cols) {
  return Matrix(get_uninit_buffer(rows * cols), rows, cols);
}

Matrix CudaRuntime::new_matrix(InitType init, size_t rows, size_t cols, unsigned long long seed) {
  const size_t n = rows * cols;
  if (init == InitType::Zero) return Matrix(get_zerod_buffer(n), rows, cols);
  std::vector<float> host(n);
  if (init == InitType::Sequence || init == InitType::Reserve) {
    // slice_set_seq_device, elementwise.rs:24-33
    for (size_t i = 0; i < n; ++i)
      host[i] = init == InitType::Sequence ? static_cast<float>(i) : static_cast<float>(n - i);
  } else {
    std::mt19937_64 g(seed);
    std::uniform_real_distribution<float> u(0.0f, 1.0f);
    for (auto& v : host) v = u(g);
  }
  return matrix_from_host(host.data(), rows, cols);
}

Matrix CudaRuntime::matrix_from_host(const float* values, size_t rows, size_t cols) {
  Matrix m = new_uninit_matrix(rows, cols);
  if (m.len())
    check_cuda_call(cudaMemcpyAsync(m.data(), values, m.len() * sizeof(float),
                                    cudaMemcpyHostToDevice, stream_),
                    "cudaMemcpyAsync H2D");
  return m;
}

Vector CudaRuntime::vector_from_host(const float* values, size_t len) {
  Vector v(get_uninit_buffer(len));
  if (len)
    check_cuda_call(cudaMemcpyAsync(v.data(), values, len * sizeof(float), cudaMemcpyHostToDevice,
                                    stream_),
                    "cudaMemcpyAsync H2D");
  return v;
}

Matrix CudaRuntime::clone_matrix(const Matrix& m, cudaStream_t s) {
  Matrix out = new_uninit_matrix(m.rows(), m.cols());
  if (s && s != stream_) fork_streams({s});
  if (m.len())
    check_cuda_call(cudaMemcpyAsync(out.data(), m.data(), m.len() * sizeof(float),
                                    cudaMemcpyDeviceToDevice, pick(s)),
                    "cudaMemcpyAsync D2D");
  return out;
}

Vector CudaRuntime::clone_vector(const Vector& v, cudaStream_t s) {
  Vector out(get_uninit_buffer(v.len()));
  if (s && s != stream_) fork_streams({s});
  if (v.len())
    check_cuda_call(cudaMemcpyAsync(out.data(), v.data(), v.len() * sizeof(float),
                                    cudaMemcpyDeviceToDevice, pick(s)),
                    "cudaMemcpyAsync D2D");
  return out;
}

Matrix CudaRuntime::matrix_multiply(const Matrix& a, const Matrix& b, cudaStream_t s) {
  require(a.cols() == b.rows(), "matrix_multiply: lhs.cols != rhs.rows");  // matrix.rs:114
  Matrix out = new_uninit_matrix(a.rows(), b.cols());
  if (s && s != stream_) fork_streams({s});
  check(oxf_matrix_multiply(a.cslice(), b.cslice(), out.slice(), a.cols(), a.rows(), b.cols(),
                            ST(pick(s))));
  return out;
}

Matrix CudaRuntime::matrix_binary(const Matrix& a, const Matrix& b, BinaryOp op, cudaStream_t s) {
  require(a.rows() == b.rows() && a.cols() == b.cols(), "matrix_binary: shape mismatch");
  Matrix out = new_uninit_matrix(a.rows(), a.cols());
  if (s && s != stream_) fork_streams({s});
  check(oxf_slice_binary(a.cslice(), b.cslice(), out.slice(), static_cast<oxf_binary_op>(op),
                         ST(pick(s))));
  return out;
}

Matrix CudaRuntime::matrix_transpose(const Matrix& m, cudaStream_t s) {
  Matrix out = new_uninit_matrix(m.cols(), m.rows());
  if (s && s != stream_) fork_streams({s});
  check(oxf_matrix_transpose(m.cslice(), out.slice(), m.rows(), m.cols(), ST(pick(s))));
  return out;
}

Vector CudaRuntime::matrix_sum_rows(const Matrix& m, cudaStream_t s) {
  Vector out(get_uninit_buffer(m.rows()));
  if (m.rows() == 0) return out;
  if (s && s != stream_) fork_streams({s});
  check(oxf_matrix_sum_rows(m.cslice(), out.slice(), m.cols(), ST(pick(s))));
  return out;
}

Vector CudaRuntime::matrix_sum_cols(const Matrix& m, cudaStream_t s) {
  Vector out(get_uninit_buffer(m.cols()));
  if (s && s != stream_) fork_streams({s});
  check(oxf_matrix_sum_cols(m.cslice(), out.slice(), m.cols(), 0, ST(pick(s))));
  return out;
}

Matrix CudaRuntime::softmax_rows_backward(const Matrix& p, const Matrix& dy) {
  require(p.rows() == dy.rows() && p.cols() == dy.cols(), "softmax_rows_backward: shapes");
  Matrix out = new_uninit_matrix(p.rows(), p.cols());
  check(oxf_softmax_rows_backward(p.cslice(), dy.cslice(), out.slice(), p.cols(), 1.0f,
                                  ST(stream_)));
  return out;
}

Matrix CudaRuntime::layer_norm_backward(const Matrix& x, const Matrix& dy) {
  require(x.rows() == dy.rows() && x.cols() == dy.cols(), "layer_norm_backward: shapes");
  Matrix out = new_uninit_matrix(x.rows(), x.cols());
  check(oxf_layer_norm_backward(x.cslice(), dy.cslice(), out.slice(), x.cols(), 1e-5f,
                                ST(stream_)));
  return out;
}

Matrix CudaRuntime::rms_norm_backward(const Matrix& x, const Matrix& dy) {
  require(x.rows() == dy.rows() && x.cols() == dy.cols(), "rms_norm_backward: shapes");
  Matrix out = new_uninit_matrix(x.rows(), x.cols());
  check(oxf_matrix_rms_norm_backward(x.cslice(), dy.cslice(), out.slice(), x.cols(), 1e-5f,
                                     ST(stream_)));
  return out;
}

// ---------------------------------------------------------------- Matrix
Matrix::Matrix(DeviceBuffer buf, size_t rows, size_t cols)
    : buf_(std::move(buf)), rows_(rows), cols_(cols) {
  require(buf_.len() == rows * cols, "Matrix: buffer length != rows * cols");
}

Matrix Matrix::view(float* ptr, size_t rows, size_t cols) {
  return Matrix(DeviceBuffer(nullptr, ptr, rows * cols), rows, cols);
}

std::vector<float> Matrix::to_host(const CudaRuntime& rt) const {
  std::vector<float> h(len());
  if (len()) {
    check_cuda_call(cudaMemcpyAsync(h.data(), data(), len() * sizeof(float),
                                    cudaMemcpyDeviceToHost, rt.stream()),
                    "cudaMemcpyAsync D2H");
    rt.sync();
  }
  return h;
}

void Matrix::scale(float v, const CudaRuntime& rt, cudaStream_t s) {
  check(oxf_slice_unary(slice(), OXF_UNARY_SCALE, v, ST(rt.pick(s))));
}
void Matrix::add_scalar(float v, const CudaRuntime& rt, cudaStream_t s) {
  check(oxf_slice_unary(slice(), OXF_UNARY_ADD_SCALAR, v, ST(rt.pick(s))));
}
void Matrix::activate(Activation act, const CudaRuntime& rt, cudaStream_t s) {
  if (act == Activation::Identity) return;
  check(oxf_slice_unary(slice(), OXF_UNARY_ACT_FORWARD, static_cast<float>(act), ST(rt.pick(s))));
}
void Matrix::activate_derivative(Activation act, const CudaRuntime& rt, cudaStream_t s) {
  check(oxf_slice_unary(slice(), OXF_UNARY_ACT_DERIV, static_cast<float>(act), ST(rt.pick(s))));
}
void Matrix::binary_assign(const Matrix& rhs, BinaryOp op, const CudaRuntime& rt,
                           cudaStream_t s) {
  require(rows_ == rhs.rows() && cols_ == rhs.cols(), "binary_assign: shape mismatch");
  check(oxf_slice_binary_assign(slice(), rhs.cslice(), static_cast<oxf_binary_op>(op),
                                ST(rt.pick(s))));
}
void Matrix::binary_assign_by_rows(const Vector& v, BinaryOp op, const CudaRuntime& rt,
                                   cudaStream_t s) {
  require(cols_ == v.len(), "binary_assign_by_rows: cols != vec.len");  // rows.rs:18
  if (!len()) return;
  check(oxf_matrix_binary_assign_by_rows(slice(), v.cslice(), cols_,
                                         static_cast<oxf_binary_op>(op), ST(rt.pick(s))));
}
void Matrix::causal_mask(const CudaRuntime& rt, cudaStream_t s) {
  if (rows_ == 0) return;
  check(oxf_matrix_causal_mask(slice(), cols_, ST(rt.pick(s))));
}
void Matrix::softmax_rows(const CudaRuntime& rt, cudaStream_t s) {
  if (rows_ == 0) return;
  require(cols_ > 0, "softmax_rows: cols must be > 0");
  check(oxf_matrix_softmax_rows(slice(), cols_, 1.0f, 0, ST(rt.pick(s))));
}
void Matrix::layer_norm(const CudaRuntime& rt, cudaStream_t s) {
  if (rows_ == 0) return;
  require(cols_ > 0, "layer_norm: cols must be > 0");
  check(oxf_matrix_layer_norm_rows(slice(), cols_, 1e-5f, nullptr, nullptr, ST(rt.pick(s))));
}
void Matrix::rms_norm(const CudaRuntime& rt, cudaStream_t s) {
  if (rows_ == 0) return;
  require(cols_ > 0, "rms_norm: cols must be > 0");
  check(oxf_rms_norm_assign(slice(), cols_, 1e-5f, nullptr, ST(rt.pick(s))));
}

// ---------------------------------------------------------------- Vector
Vector Vector::view(float* ptr, size_t len) { return Vector(DeviceBuffer(nullptr, ptr, len)); }

std::vector<float> Vector::to_host(const CudaRuntime& rt) const {
  std::vector<float> h(len());
  if (len()) {
    check_cuda_call(cudaMemcpyAsync(h.data(), data(), len() * sizeof(float),
                                    cudaMemcpyDeviceToHost, rt.stream()),
                    "cudaMemcpyAsync D2H");
    rt.sync();
  }
  return h;
}

void Vector::scale(float v, const CudaRuntime& rt, cudaStream_t s) {
  check(oxf_slice_unary(slice(), OXF_UNARY_SCALE, v, ST(rt.pick(s))));
}
void Vector::binary_assign(const Vector& rhs, BinaryOp op, const CudaRuntime& rt, cudaStream_t s) {
  require(len() == rhs.len(), "Vector::binary_assign: length mismatch");
  check(oxf_slice_binary_assign(slice(), rhs.cslice(), static_cast<oxf_binary_op>(op),
                                ST(rt.pick(s))));
}

float Vector::sum(CudaRuntime& rt) const {
  DeviceBuffer out = rt.get_uninit_buffer(1);
  check(oxf_slice_sum(cslice(), out.data(), ST(rt.stream())));
  float h = 0;
  check_cuda_call(cudaMemcpyAsync(&h, out.data(), 4, cudaMemcpyDeviceToHost, rt.stream()), "D2H");
  rt.sync();
  return h;
}

float Vector::max(CudaRuntime& rt) const {
  DeviceBuffer out = rt.get_uninit_buffer(1);
  check(oxf_slice_max(cslice(), out.data(), ST(rt.stream())));
  float h = 0;
  check_cuda_call(cudaMemcpyAsync(&h, out.data(), 4, cudaMemcpyDeviceToHost, rt.stream()), "D2H");
  rt.sync();
  return h;
}

}  // namespace oxf
