// runtime_client.cpp — drives the C++ host layer (oxide-forge_b200/host/
// runtime.hpp, linear.hpp) the way a port of the reference's Rust callers
// would: CudaRuntime's exact-size pool, forked and joined streams, Matrix /
// Vector operations, and Linear. Linked to liboxf.so only; it makes no CUDA
// call of its own.
//
// Usage: runtime_client <dir>. Reads <dir>/a.bin [R,C], a2.bin [R,C],
// b.bin [C,N], v.bin [C], sq.bin [S,S], dyc.bin [R,C], w.bin [C,N],
// bias.bin [N], dyn.bin [R,N], t.bin [R,N], with R C N S in <dir>/dims.txt.
// Writes out_<name>.bin (raw f32) for tests/test_runtime_gpu.py to check
// against the oracle, and prints "key value" lines then "ok" on stdout.
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <string>
#include <vector>

#include "linear.hpp"
#include "runtime.hpp"

using namespace oxf;

static std::string dir;

static std::vector<float> read_bin(const char* name, size_t n) {
  std::vector<float> v(n);
  FILE* f = std::fopen((dir + "/" + name).c_str(), "rb");
  if (!f || std::fread(v.data(), 4, n, f) != n) {
    std::fprintf(stderr, "cannot read %s\n", name);
    std::exit(2);
  }
  std::fclose(f);
  return v;
}

static void write_bin(const std::string& name, const std::vector<float>& v) {
  FILE* f = std::fopen((dir + "/out_" + name + ".bin").c_str(), "wb");
  if (!f || std::fwrite(v.data(), 4, v.size(), f) != v.size()) {
    std::fprintf(stderr, "cannot write %s\n", name.c_str());
    std::exit(2);
  }
  std::fclose(f);
}

static void fail(const char* what) {
  std::fprintf(stderr, "check failed: %s\n", what);
  std::exit(1);
}

int main(int argc, char** argv) {
  if (argc != 2) return 2;
  dir = argv[1];
  size_t R = 0, Cc = 0, N = 0, S = 0;
  {
    std::ifstream d(dir + "/dims.txt");
    d >> R >> Cc >> N >> S;
  }
  try {
    CudaRuntime rt(0);

    // ---- exact-size pool (runtime.rs:47-110)
    {
      DeviceBuffer b = rt.get_uninit_buffer(1000);
      float* p = b.data();
      b.reset();  // back to the pool
      if (rt.pooled_buffers() != 1) fail("a reset buffer returns to the pool");
      DeviceBuffer c = rt.get_uninit_buffer(1000);
      if (c.data() != p) fail("the pool hands the same-size buffer out again");
      if (rt.pooled_buffers() != 0) fail("the reused buffer left the pool");
      DeviceBuffer other = rt.get_uninit_buffer(999);
      if (other.data() == p) fail("sizes are exact");
      rt.reserve_buffers(500, 3);
      if (rt.pooled_buffers() != 3) fail("reserve_buffers fills the pool");
      rt.reserve_buffers(500, 2);
      if (rt.pooled_buffers() != 3) fail("reserve_buffers only tops up");
    }
    std::printf("pooled_after_scope %zu\n", rt.pooled_buffers());

    const auto a_h = read_bin("a.bin", R * Cc), a2_h = read_bin("a2.bin", R * Cc);
    const auto b_h = read_bin("b.bin", Cc * N), v_h = read_bin("v.bin", Cc);
    const auto sq_h = read_bin("sq.bin", S * S), dyc_h = read_bin("dyc.bin", R * Cc);
    const auto w_h = read_bin("w.bin", Cc * N), bias_h = read_bin("bias.bin", N);
    const auto dyn_h = read_bin("dyn.bin", R * N), t_h = read_bin("t.bin", R * N);
    Matrix a = rt.matrix_from_host(a_h.data(), R, Cc);
    Matrix a2 = rt.matrix_from_host(a2_h.data(), R, Cc);
    Matrix b = rt.matrix_from_host(b_h.data(), Cc, N);
    Vector v = rt.vector_from_host(v_h.data(), Cc);
    Matrix sq = rt.matrix_from_host(sq_h.data(), S, S);
    Matrix dyc = rt.matrix_from_host(dyc_h.data(), R, Cc);

    // ---- allocating operations (docs/api.md: they belong to CudaRuntime)
    write_bin("mm", rt.matrix_multiply(a, b).to_host(rt));
    write_bin("transpose", rt.matrix_transpose(a).to_host(rt));
    write_bin("sum_rows", rt.matrix_sum_rows(a).to_host(rt));
    write_bin("sum_cols", rt.matrix_sum_cols(a).to_host(rt));
    write_bin("sub", rt.matrix_sub(a, a2).to_host(rt));
    write_bin("mul", rt.matrix_mul(a, a2).to_host(rt));

    // ---- mutating operations (docs/api.md: they belong to Matrix)
    {
      Matrix m = rt.clone_matrix(a);
      m.softmax_rows(rt);
      write_bin("softmax", m.to_host(rt));
      write_bin("softmax_bwd", rt.softmax_rows_backward(m, dyc).to_host(rt));
    }
    {
      Matrix m = rt.clone_matrix(a);
      m.layer_norm(rt);
      write_bin("layer_norm", m.to_host(rt));
      write_bin("layer_norm_bwd", rt.layer_norm_backward(a, dyc).to_host(rt));
    }
    {
      Matrix m = rt.clone_matrix(a);
      m.rms_norm(rt);
      write_bin("rms_norm", m.to_host(rt));
      write_bin("rms_norm_bwd", rt.rms_norm_backward(a, dyc).to_host(rt));
    }
    {
      Matrix m = rt.clone_matrix(a);
      m.activate(Activation::Gelu, rt);
      write_bin("gelu", m.to_host(rt));
      Matrix d = rt.clone_matrix(a);
      d.activate_derivative(Activation::Gelu, rt);
      write_bin("gelu_deriv", d.to_host(rt));
    }
    {
      Matrix m = rt.clone_matrix(a);
      m.binary_assign_by_rows(v, BinaryOp::Mul, rt);
      m.scale(0.5f, rt);
      m.add_scalar(1.0f, rt);
      write_bin("by_rows_scale_add", m.to_host(rt));
    }
    {
      Matrix m = rt.clone_matrix(sq);
      m.causal_mask(rt);
      write_bin("causal_mask", m.to_host(rt));
    }
    std::printf("v_sum %.9g\nv_max %.9g\n", static_cast<double>(v.sum(rt)),
                static_cast<double>(v.max(rt)));

    // ---- forked streams (runtime.rs:188-211): independent work on two
    // extra streams, joined back into the primary stream
    {
      std::vector<cudaStream_t> side = rt.create_extra_streams(2);
      Matrix m1 = rt.clone_matrix(a);
      Matrix m2 = rt.clone_matrix(a2);
      rt.fork_streams(side);  // the clones are queued before the fork
      m1.scale(3.0f, rt, side[0]);
      m1.add_scalar(-1.0f, rt, side[0]);
      m2.activate(Activation::Relu, rt, side[1]);
      rt.join_streams(side);
      m1.binary_assign(m2, BinaryOp::Add, rt);  // primary stream, after both
      write_bin("fork_join", m1.to_host(rt));
    }

    // ---- Linear (linear.rs): forward, affine, backward, input_gradient,
    // loss_rows, learn
    {
      Matrix w = rt.matrix_from_host(w_h.data(), Cc, N);
      Vector bias = rt.vector_from_host(bias_h.data(), N);
      Linear lin(std::move(w), std::move(bias), Activation::Gelu);
      Matrix dyn = rt.matrix_from_host(dyn_h.data(), R, N);
      Matrix t = rt.matrix_from_host(t_h.data(), R, N);
      Matrix y = lin.forward(a, nullptr, rt);
      Matrix z = lin.affine(a, nullptr, rt);
      write_bin("lin_y", y.to_host(rt));
      write_bin("lin_z", z.to_host(rt));
      const cudaStream_t s = rt.create_extra_streams(1)[0];
      Matrix y_side = lin.forward(a, nullptr, rt, s);
      rt.join_streams({s});
      const auto y1 = y.to_host(rt), y2 = y_side.to_host(rt);
      if (y1 != y2) fail("forward on a forked stream gives the same bits");
      write_bin("lin_loss", Linear::loss_rows(y, t, rt).to_host(rt));
      auto gb = lin.backward(&z, dyn, rt);
      write_bin("lin_g", gb.first.to_host(rt));
      write_bin("lin_bg", gb.second->to_host(rt));
      write_bin("lin_dx", lin.input_gradient(gb.first, rt).to_host(rt));
      lin.learn(a, gb.first, &*gb.second, 0.05f, rt);
      write_bin("lin_w_new", lin.weights().to_host(rt));
      write_bin("lin_b_new", lin.bias()->to_host(rt));
    }
    rt.sync();
    std::printf("pooled_at_end %zu\n", rt.pooled_buffers());
  } catch (const Error& e) {
    std::fprintf(stderr, "oxf error %d: %s\n", static_cast<int>(e.status), e.what());
    return 1;
  }
  std::printf("ok\n");
  return 0;
}
