// rows.cu — HBM-bound kernels: row-wise softmax / LayerNorm / RMSNorm
// forward and backward, row and column sums, loss rows, elementwise and
// row-broadcast ops, grid reductions and transpose.
//
// The reference runs every row kernel as one 1024-thread block per row with
// one element per thread, scalar 4-byte loads and 2-4 block barriers
// (src/cuda/device/row.rs), which caps rows at 1024 columns
// (src/cuda/container/norm.rs:12,30,54). Here a row is loaded once into
// registers with 128-bit loads by a group of G threads (one warp for rows
// up to 2048 wide, a whole block beyond), reduced with warp shuffles, and
// written once: each kernel moves exactly its algorithmic bytes. Rows too
// wide for registers, or not 16-byte aligned, take a looped scalar path.
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <cstdint>

#include "common.cuh"
#include "status.cuh"
#include "ptx.cuh"

namespace oxf {

// ------------------------------------------------------------------ reductions
template <int G>
struct GroupReduce {
  // G == 32: one warp per row, no shared memory. G > 32: one row per block.
  __device__ __forceinline__ static float sum(float v, float* red) {
    v = warp_sum(v);
    if constexpr (G == 32) {
      return v;
    } else {
      const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
      __syncthreads();
      if (l == 0) red[w] = v;
      __syncthreads();
      float t = 0.f;
#pragma unroll
      for (int i = 0; i < G / 32; ++i) t += red[i];
      return t;
    }
  }
  __device__ __forceinline__ static float max(float v, float* red) {
    v = warp_max(v);
    if constexpr (G == 32) {
      return v;
    } else {
      const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
      __syncthreads();
      if (l == 0) red[w] = v;
      __syncthreads();
      float t = -FLT_MAX;
#pragma unroll
      for (int i = 0; i < G / 32; ++i) t = fmaxf(t, red[i]);
      return t;
    }
  }
  __device__ __forceinline__ static float2 sum2(float2 v, float* red) {
    v.x = warp_sum(v.x);
    v.y = warp_sum(v.y);
    if constexpr (G == 32) {
      return v;
    } else {
      const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
      __syncthreads();
      if (l == 0) {
        red[2 * w] = v.x;
        red[2 * w + 1] = v.y;
      }
      __syncthreads();
      float2 t = make_float2(0.f, 0.f);
#pragma unroll
      for (int i = 0; i < G / 32; ++i) {
        t.x += red[2 * i];
        t.y += red[2 * i + 1];
      }
      return t;
    }
  }
};

// Register-resident row: thread t of the group owns float4 chunks
// t, t+G, t+2G, ... (NV of them). Chunks past the row end are "inactive".
template <int G, int NV>
struct Row {
  float4 v[NV];
  __device__ __forceinline__ static bool active(int j, int t, int cols4) {
    return t + j * G < cols4;
  }
  __device__ __forceinline__ void load(const float* row, int t, int cols4, float fill) {
#pragma unroll
    for (int j = 0; j < NV; ++j)
      v[j] = active(j, t, cols4) ? __ldcs(reinterpret_cast<const float4*>(row) + t + j * G)
                                 : make_float4(fill, fill, fill, fill);
  }
  __device__ __forceinline__ void store(float* row, int t, int cols4) const {
#pragma unroll
    for (int j = 0; j < NV; ++j)
      if (active(j, t, cols4)) __stcs(reinterpret_cast<float4*>(row) + t + j * G, v[j]);
  }
};

// Programmatic dependent launch: every kernel here is launched with
// programmatic stream serialisation (launch_pdl below). It lets the next
// kernel of the stream be scheduled as soon as all of this grid's blocks
// are running, then waits, before touching memory, until the previous
// kernel of the stream has completed and its writes are visible. Launched
// without the attribute, both instructions have no effect.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void pdl_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Inputs of at most this many bytes per launch are prefetched into L2 before
// griddepcontrol.wait, so that this kernel's first DRAM reads overlap the
// previous kernel's last writes. L2 is the GPU's point of coherence, so a
// line prefetched before the previous kernel writes it is updated there and
// the loads after the wait read the final data; the cost of such a line is
// one wasted DRAM read. Larger inputs would only evict each other (and the
// previous kernel's working set), so they are not prefetched.
constexpr long long kPrefetchMaxBytes = 64ll << 20;

// Bulk L2 prefetch of one row (16-byte aligned start, bytes % 16 == 0).
__device__ __forceinline__ void prefetch_l2(const void* p, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// PDL entry of a row kernel with inputs a (and b), [rows, cols] each: the
// first thread of each row's group prefetches the row of every input when
// they are small enough, then the kernel waits for its predecessor.
template <int G>
__device__ __forceinline__ void row_enter(long long rows, int cols, const float* a,
                                          const float* b = nullptr) {
  pdl_launch();
  const long long bytes = rows * cols * 4ll * (b ? 2 : 1);
  if (bytes <= kPrefetchMaxBytes) {
    long long r;
    int t;
    if constexpr (G == 32) {
      r = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
      t = threadIdx.x & 31;
    } else {
      r = blockIdx.x;
      t = threadIdx.x;
    }
    if (t == 0 && r < rows) {
      prefetch_l2(a + r * cols, static_cast<unsigned>(cols) * 4u);
      if (b) prefetch_l2(b + r * cols, static_cast<unsigned>(cols) * 4u);
    }
  }
  pdl_wait();
}

// Norm parameters (gamma, beta) of a warp-per-row block, which holds eight
// rows: staged once per block in shared memory by bulk copies that one
// thread issues after the PDL wait and that complete on an mbarrier. Each
// warp waits on that mbarrier only when it applies the parameters, after its
// row's reductions, so no block barrier sits between a row's loads and its
// stores; the one barrier, after the mbarrier's initialisation, comes before
// the PDL wait. The wait is bounded: on expiry it records DEVERR_ROW_PARAMS.
__device__ __forceinline__ void params_init(uint64_t* bar) {
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
}

// Bulk copy global -> shared (both 16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void bulk_load_smem(void* dst, const void* src, unsigned bytes,
                                               uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Thread 0 copies cols floats of g (and of b) into sg (sb); null skips one.
__device__ __forceinline__ void params_issue(uint64_t* bar, float4* sg, const float* g, float4* sb,
                                             const float* b, int cols) {
  if (threadIdx.x != 0) return;
  const unsigned bytes = static_cast<unsigned>(cols) * 4u;
  mbar_arrive_expect_tx(bar, bytes * ((g ? 1u : 0u) + (b ? 1u : 0u)));
  if (g) bulk_load_smem(sg, g, bytes, bar);
  if (b) bulk_load_smem(sb, b, bytes, bar);
}

__device__ __forceinline__ float hsum(float4 a) { return (a.x + a.y) + (a.z + a.w); }
__device__ __forceinline__ float hmax(float4 a) { return fmaxf(fmaxf(a.x, a.y), fmaxf(a.z, a.w)); }

template <int G>
__device__ __forceinline__ bool row_index(long long rows, long long& r, int& t) {
  if constexpr (G == 32) {
    r = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    t = threadIdx.x & 31;
  } else {
    r = blockIdx.x;
    t = threadIdx.x;
  }
  return r < rows;
}

// ------------------------------------------------------------------ softmax
// row.rs:55-113 plus the folded scale (attention.rs:372) and causal mask
// (row.rs:5-14, applied with the row index taken modulo the period).
template <int G, int NV>
__global__ void softmax_fwd_kernel(float* __restrict__ m, long long rows, int cols, float scale,
                                   long long period) {
  row_enter<G>(rows, cols, m);
  __shared__ float red[2 * (G / 32)];
  long long r;
  int t;
  if (!row_index<G>(rows, r, t)) return;  // uniform per group
  const int cols4 = cols >> 2;
  float* row = m + r * cols;
  Row<G, NV> x;
  x.load(row, t, cols4, -INFINITY);
  const long long limit = period ? (r % period) : (1ll << 61);
  float mx = -FLT_MAX;  // f32::MIN, the reference's padding (row.rs:64)
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    // Inactive chunks (past the row end) and masked entries become -inf.
    const long long c0 = Row<G, NV>::active(j, t, cols4) ? (t + j * G) * 4ll : (1ll << 62);
    float4& a = x.v[j];
    a.x = (c0 + 0 <= limit) ? a.x * scale : -INFINITY;
    a.y = (c0 + 1 <= limit) ? a.y * scale : -INFINITY;
    a.z = (c0 + 2 <= limit) ? a.z * scale : -INFINITY;
    a.w = (c0 + 3 <= limit) ? a.w * scale : -INFINITY;
    mx = fmaxf(mx, hmax(a));
  }
  mx = GroupReduce<G>::max(mx, red);
  // The hardware exponential (arguments <= 0 after the max; a few ulp) and
  // one reciprocal per row: per-element IEEE expf and division cost more
  // issue slots than the memory-bound pass can hide.
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    float4& a = x.v[j];
    a.x = __expf(a.x - mx); a.y = __expf(a.y - mx); a.z = __expf(a.z - mx);
    a.w = __expf(a.w - mx);
    s += hsum(a);
  }
  s = GroupReduce<G>::sum(s, red + G / 32);
  const float inv = 1.0f / s;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    float4& a = x.v[j];
    a.x *= inv; a.y *= inv; a.z *= inv; a.w *= inv;
  }
  x.store(row, t, cols4);
}

// row.rs:193-237: dx = p*(dy - sum(p*dy)), times the attention scale
// (attention.rs:302-304).
template <int G, int NV>
__global__ void softmax_bwd_kernel(const float* __restrict__ p, const float* __restrict__ dy,
                                   float* __restrict__ dx, long long rows, int cols, float scale) {
  row_enter<G>(rows, cols, p, dy);
  __shared__ float red[G / 32];
  long long r;
  int t;
  if (!row_index<G>(rows, r, t)) return;
  const int cols4 = cols >> 2;
  Row<G, NV> pv, gv;
  pv.load(p + r * cols, t, cols4, 0.f);
  gv.load(dy + r * cols, t, cols4, 0.f);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j)
    s += pv.v[j].x * gv.v[j].x + pv.v[j].y * gv.v[j].y + pv.v[j].z * gv.v[j].z +
         pv.v[j].w * gv.v[j].w;
  s = GroupReduce<G>::sum(s, red);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    float4& a = gv.v[j];
    const float4 q = pv.v[j];
    a.x = q.x * (a.x - s) * scale; a.y = q.y * (a.y - s) * scale;
    a.z = q.z * (a.z - s) * scale; a.w = q.w * (a.w - s) * scale;
  }
  gv.store(dx + r * cols, t, cols4);
}

// ------------------------------------------------------------------ LayerNorm
// row.rs:115-177: mean, biased variance of (x - mean), 1/sqrt(var + eps).
// STAGED (launched when gamma or beta is given): a warp-per-row block stages
// them in shared memory (params_issue); the plain kernel carries no staging.
template <int G, int NV, bool STAGED>
__device__ __forceinline__ void layernorm_fwd_body(const float* in, float* out, long long rows,
                                                   int cols, float eps,
                                                   const float* __restrict__ gamma,
                                                   const float* __restrict__ beta) {
  __shared__ float red[2 * (G / 32)];
  constexpr bool staged = STAGED && G == 32;
  constexpr int STAGE = staged ? 32 * NV : 1;
  __shared__ alignas(16) float4 sg[STAGE], sb[STAGE];
  __shared__ alignas(8) uint64_t bar;
  if constexpr (staged) params_init(&bar);
  row_enter<G>(rows, cols, in);
  if constexpr (staged) params_issue(&bar, sg, gamma, sb, beta, cols);
  long long r;
  int t;
  if (!row_index<G>(rows, r, t)) return;
  const int cols4 = cols >> 2;
  Row<G, NV> x;
  x.load(in + r * cols, t, cols4, 0.f);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) s += hsum(x.v[j]);
  const float mean = GroupReduce<G>::sum(s, red) / static_cast<float>(cols);
  float v = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    if (!Row<G, NV>::active(j, t, cols4)) continue;
    float4& a = x.v[j];
    a.x -= mean; a.y -= mean; a.z -= mean; a.w -= mean;
    v += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
  }
  v = GroupReduce<G>::sum(v, red + G / 32);
  const float inv_std = 1.0f / sqrtf(v / static_cast<float>(cols) + eps);
  if constexpr (staged) mbar_wait(&bar, 0, DEVERR_ROW_PARAMS);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    if (!Row<G, NV>::active(j, t, cols4)) continue;
    float4& a = x.v[j];
    a.x *= inv_std; a.y *= inv_std; a.z *= inv_std; a.w *= inv_std;
    if (gamma) {
      const float4 g = staged ? sg[t + j * G] : reinterpret_cast<const float4*>(gamma)[t + j * G];
      a.x *= g.x; a.y *= g.y; a.z *= g.z; a.w *= g.w;
    }
    if (beta) {
      const float4 b = staged ? sb[t + j * G] : reinterpret_cast<const float4*>(beta)[t + j * G];
      a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
    }
  }
  x.store(out + r * cols, t, cols4);
}

template <int G, int NV>
__global__ void layernorm_fwd_kernel(const float* in, float* out, long long rows, int cols,
                                     float eps, const float* __restrict__ gamma,
                                     const float* __restrict__ beta) {
  layernorm_fwd_body<G, NV, false>(in, out, rows, cols, eps, gamma, beta);
}

template <int G, int NV>
__global__ void layernorm_fwd_staged_kernel(const float* in, float* out, long long rows, int cols,
                                            float eps, const float* __restrict__ gamma,
                                            const float* __restrict__ beta) {
  layernorm_fwd_body<G, NV, true>(in, out, rows, cols, eps, gamma, beta);
}

// row.rs:239-347: dx = inv_std/N * (N*dy - sum(dy) - xhat*sum(dy*xhat)).
template <int G, int NV>
__global__ void layernorm_bwd_kernel(const float* __restrict__ xin, const float* __restrict__ dy,
                                     float* __restrict__ dx, long long rows, int cols, float eps) {
  row_enter<G>(rows, cols, xin, dy);
  __shared__ float red[4 * (G / 32)];
  long long r;
  int t;
  if (!row_index<G>(rows, r, t)) return;
  const int cols4 = cols >> 2;
  const float n = static_cast<float>(cols);
  Row<G, NV> x, g;
  x.load(xin + r * cols, t, cols4, 0.f);
  g.load(dy + r * cols, t, cols4, 0.f);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) s += hsum(x.v[j]);
  const float mean = GroupReduce<G>::sum(s, red) / n;
  float v = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    if (!Row<G, NV>::active(j, t, cols4)) continue;
    float4& a = x.v[j];
    a.x -= mean; a.y -= mean; a.z -= mean; a.w -= mean;
    v += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
  }
  v = GroupReduce<G>::sum(v, red + G / 32);
  const float inv_std = 1.0f / sqrtf(v / n + eps);
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    float4& a = x.v[j];
    const float4 b = g.v[j];
    a.x *= inv_std; a.y *= inv_std; a.z *= inv_std; a.w *= inv_std;  // xhat
    acc.x += hsum(b);
    acc.y += b.x * a.x + b.y * a.y + b.z * a.z + b.w * a.w;
  }
  acc = GroupReduce<G>::sum2(acc, red + 2 * (G / 32));
  const float k = inv_std / n;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    float4& b = g.v[j];
    const float4 a = x.v[j];
    b.x = k * (n * b.x - acc.x - a.x * acc.y);
    b.y = k * (n * b.y - acc.x - a.y * acc.y);
    b.z = k * (n * b.z - acc.x - a.z * acc.y);
    b.w = k * (n * b.w - acc.x - a.w * acc.y);
  }
  g.store(dx + r * cols, t, cols4);
}

// ------------------------------------------------------------------ RMSNorm
// row.rs:349-396: y = x / sqrt(mean(x^2) + eps).
// STAGED as for LayerNorm (launched when gamma is given).
template <int G, int NV, bool STAGED>
__device__ __forceinline__ void rmsnorm_fwd_body(const float* in, float* out, long long rows,
                                                 int cols, float eps,
                                                 const float* __restrict__ gamma) {
  __shared__ float red[G / 32];
  constexpr bool staged = STAGED && G == 32;
  constexpr int STAGE = staged ? 32 * NV : 1;
  __shared__ alignas(16) float4 sg[STAGE];
  __shared__ alignas(8) uint64_t bar;
  if constexpr (staged) params_init(&bar);
  row_enter<G>(rows, cols, in);
  if constexpr (staged) params_issue(&bar, sg, gamma, nullptr, nullptr, cols);
  long long r;
  int t;
  if (!row_index<G>(rows, r, t)) return;
  const int cols4 = cols >> 2;
  Row<G, NV> x;
  x.load(in + r * cols, t, cols4, 0.f);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const float4 a = x.v[j];
    s += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
  }
  s = GroupReduce<G>::sum(s, red);
  const float rms = sqrtf(s / static_cast<float>(cols) + eps);
  if constexpr (staged) mbar_wait(&bar, 0, DEVERR_ROW_PARAMS);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    if (!Row<G, NV>::active(j, t, cols4)) continue;
    float4& a = x.v[j];
    a.x = a.x / rms; a.y = a.y / rms; a.z = a.z / rms; a.w = a.w / rms;
    if (gamma) {
      const float4 g = staged ? sg[t + j * G] : reinterpret_cast<const float4*>(gamma)[t + j * G];
      a.x *= g.x; a.y *= g.y; a.z *= g.z; a.w *= g.w;
    }
  }
  x.store(out + r * cols, t, cols4);
}

template <int G, int NV>
__global__ void rmsnorm_fwd_kernel(const float* in, float* out, long long rows, int cols,
                                   float eps, const float* __restrict__ gamma) {
  rmsnorm_fwd_body<G, NV, false>(in, out, rows, cols, eps, gamma);
}

template <int G, int NV>
__global__ void rmsnorm_fwd_staged_kernel(const float* in, float* out, long long rows, int cols,
                                          float eps, const float* __restrict__ gamma) {
  rmsnorm_fwd_body<G, NV, true>(in, out, rows, cols, eps, gamma);
}

// row.rs:398-468: dx = dy/r - x*(sum(x*dy)/N)/r^3.
template <int G, int NV>
__global__ void rmsnorm_bwd_kernel(const float* __restrict__ xin, const float* __restrict__ dy,
                                   float* __restrict__ dx, long long rows, int cols, float eps) {
  row_enter<G>(rows, cols, xin, dy);
  __shared__ float red[2 * (G / 32)];
  long long r;
  int t;
  if (!row_index<G>(rows, r, t)) return;
  const int cols4 = cols >> 2;
  const float n = static_cast<float>(cols);
  Row<G, NV> x, g;
  x.load(xin + r * cols, t, cols4, 0.f);
  g.load(dy + r * cols, t, cols4, 0.f);
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const float4 a = x.v[j], b = g.v[j];
    acc.x += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
    acc.y += a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
  }
  acc = GroupReduce<G>::sum2(acc, red);
  const float rms = sqrtf(acc.x / n + eps);
  const float inv = 1.0f / rms;
  const float corr = acc.y / n * inv * inv * inv;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    float4& b = g.v[j];
    const float4 a = x.v[j];
    b.x = b.x * inv - a.x * corr; b.y = b.y * inv - a.y * corr;
    b.z = b.z * inv - a.z * corr; b.w = b.w * inv - a.w * corr;
  }
  g.store(dx + r * cols, t, cols4);
}

// ------------------------------------------------------------------ row sums / loss
// row.rs:16-53.
template <int G, int NV>
__global__ void sum_rows_kernel(const float* __restrict__ m, float* __restrict__ out,
                                long long rows, int cols) {
  row_enter<G>(rows, cols, m);
  __shared__ float red[G / 32];
  long long r;
  int t;
  if (!row_index<G>(rows, r, t)) return;
  const int cols4 = cols >> 2;
  Row<G, NV> x;
  x.load(m + r * cols, t, cols4, 0.f);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) s += hsum(x.v[j]);
  s = GroupReduce<G>::sum(s, red);
  if (t == 0) out[r] = s;
}

// linear.rs:325-333: mean over the row of 0.5 * (y - t)^2.
template <int G, int NV>
__global__ void loss_rows_kernel(const float* __restrict__ y, const float* __restrict__ tg,
                                 float* __restrict__ out, long long rows, int cols) {
  pdl_enter();
  __shared__ float red[G / 32];
  long long r;
  int t;
  if (!row_index<G>(rows, r, t)) return;
  const int cols4 = cols >> 2;
  Row<G, NV> a, b;
  a.load(y + r * cols, t, cols4, 0.f);
  b.load(tg + r * cols, t, cols4, 0.f);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const float dx = a.v[j].x - b.v[j].x, dyy = a.v[j].y - b.v[j].y;
    const float dz = a.v[j].z - b.v[j].z, dw = a.v[j].w - b.v[j].w;
    s += 0.5f * dx * dx + 0.5f * dyy * dyy + 0.5f * dz * dz + 0.5f * dw * dw;
  }
  s = GroupReduce<G>::sum(s, red);
  if (t == 0) out[r] = s * (1.0f / static_cast<float>(cols));
}

// loss_rows and its gradient in one pass over y and t.
template <int G, int NV>
__global__ void loss_grad_rows_kernel(const float* __restrict__ y, const float* __restrict__ tg,
                                      float* __restrict__ out, float* __restrict__ dy,
                                      long long rows, int cols) {
  row_enter<G>(rows, cols, y, tg);
  __shared__ float red[G / 32];
  long long r;
  int t;
  if (!row_index<G>(rows, r, t)) return;
  const int cols4 = cols >> 2;
  const float inv = 1.0f / static_cast<float>(cols);
  Row<G, NV> a, b;
  a.load(y + r * cols, t, cols4, 0.f);
  b.load(tg + r * cols, t, cols4, 0.f);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    float4& d = a.v[j];
    d.x -= b.v[j].x; d.y -= b.v[j].y; d.z -= b.v[j].z; d.w -= b.v[j].w;
    s += 0.5f * d.x * d.x + 0.5f * d.y * d.y + 0.5f * d.z * d.z + 0.5f * d.w * d.w;
    d.x *= inv; d.y *= inv; d.z *= inv; d.w *= inv;
  }
  a.store(dy + r * cols, t, cols4);
  s = GroupReduce<G>::sum(s, red);
  if (t == 0) out[r] = s * inv;
}

// ------------------------------------------------------------------ looped (general) path
// One block per row, any width and alignment, scalar accesses, several
// passes over the row in global memory.
enum LoopOp { LOOP_SOFTMAX, LOOP_LN, LOOP_RMS, LOOP_SOFTMAX_BWD, LOOP_LN_BWD, LOOP_RMS_BWD,
              LOOP_SUM, LOOP_LOSS };

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = -FLT_MAX;
  for (int i = 0; i < nw; ++i) t = fmaxf(t, red[i]);
  return t;
}

__global__ void row_looped_kernel(int op, float* __restrict__ out, const float* __restrict__ a,
                                  const float* __restrict__ b, long long cols, float p0, float p1,
                                  long long period, const float* __restrict__ gamma,
                                  const float* __restrict__ beta) {
  pdl_enter();
  __shared__ float red[32];
  const long long r = blockIdx.x;
  const float n = static_cast<float>(cols);
  const float* ar = a + r * cols;
  const float* br = b ? b + r * cols : nullptr;
  float* orow = out + r * cols;
  switch (op) {
    case LOOP_SOFTMAX: {  // out == a (in place); p0 = scale
      const long long limit = period ? (r % period) : (1ll << 62);
      float mx = -FLT_MAX;
      for (long long c = threadIdx.x; c < cols; c += blockDim.x)
        mx = fmaxf(mx, c <= limit ? ar[c] * p0 : -INFINITY);
      mx = block_max(mx, red);
      float s = 0.f;
      for (long long c = threadIdx.x; c < cols; c += blockDim.x)
        s += expf((c <= limit ? ar[c] * p0 : -INFINITY) - mx);
      s = block_sum(s, red);
      for (long long c = threadIdx.x; c < cols; c += blockDim.x)
        orow[c] = expf((c <= limit ? ar[c] * p0 : -INFINITY) - mx) / s;
      break;
    }
    case LOOP_LN: {  // p0 = eps
      float s = 0.f;
      for (long long c = threadIdx.x; c < cols; c += blockDim.x) s += ar[c];
      const float mean = block_sum(s, red) / n;
      float v = 0.f;
      for (long long c = threadIdx.x; c < cols; c += blockDim.x) {
        const float d = ar[c] - mean;
        v += d * d;
      }
      const float inv_std = 1.0f / sqrtf(block_sum(v, red) / n + p0);
      for (long long c = threadIdx.x; c < cols; c += blockDim.x) {
        float y = (ar[c] - mean) * inv_std;
        if (gamma) y *= gamma[c];
        if (beta) y += beta[c];
        orow[c] = y;
      }
      break;
    }
    case LOOP_RMS: {
      float s = 0.f;
      for (long long c = threadIdx.x; c < cols; c += blockDim.x) s += ar[c] * ar[c];
      const float rms = sqrtf(block_sum(s, red) / n + p0);
      for (long long c = threadIdx.x; c < cols; c += blockDim.x) {
        float y = ar[c] / rms;
        if (gamma) y *= gamma[c];
        orow[c] = y;
      }
      break;
    }
    case LOOP_SOFTMAX_BWD: {  // a = p, b = dy, p0 = scale
      float s = 0.f;
      for (long long c = threadIdx.x; c < cols; c += blockDim.x) s += ar[c] * br[c];
      s = block_sum(s, red);
      for (long long c = threadIdx.x; c < cols; c += blockDim.x)
        orow[c] = ar[c] * (br[c] - s) * p0;
      break;
    }
    case LOOP_LN_BWD: {
      float s = 0.f;
      for (long long c = threadIdx.x; c < cols; c += blockDim.x) s += ar[c];
      const float mean = block_sum(s, red) / n;
      float v = 0.f;
      for (long long c = threadIdx.x; c < cols; c += blockDim.x) {
        const float d = ar[c] - mean;
        v += d * d;
      }
      const float inv_std = 1.0f / sqrtf(block_sum(v, red) / n + p0);
      float gs = 0.f, gns = 0.f;
      for (long long c = threadIdx.x; c < cols; c += blockDim.x) {
        gs += br[c];
        gns += br[c] * ((ar[c] - mean) * inv_std);
      }
      gs = block_sum(gs, red);
      gns = block_sum(gns, red);
      for (long long c = threadIdx.x; c < cols; c += blockDim.x) {
        const float xh = (ar[c] - mean) * inv_std;
        orow[c] = inv_std / n * (n * br[c] - gs - xh * gns);
      }
      break;
    }
    case LOOP_RMS_BWD: {
      float ss = 0.f, dot = 0.f;
      for (long long c = threadIdx.x; c < cols; c += blockDim.x) {
        ss += ar[c] * ar[c];
        dot += ar[c] * br[c];
      }
      ss = block_sum(ss, red);
      dot = block_sum(dot, red);
      const float inv = 1.0f / sqrtf(ss / n + p0);
      const float corr = dot / n * inv * inv * inv;
      for (long long c = threadIdx.x; c < cols; c += blockDim.x)
        orow[c] = br[c] * inv - ar[c] * corr;
      break;
    }
    case LOOP_SUM: {
      float s = 0.f;
      for (long long c = threadIdx.x; c < cols; c += blockDim.x) s += ar[c];
      s = block_sum(s, red);
      if (threadIdx.x == 0) out[r] = s;
      break;
    }
    case LOOP_LOSS: {
      float s = 0.f;
      for (long long c = threadIdx.x; c < cols; c += blockDim.x) {
        const float d = ar[c] - br[c];
        s += 0.5f * d * d;
      }
      s = block_sum(s, red);
      if (threadIdx.x == 0) out[r] = s * (1.0f / n);
      break;
    }
  }
}

// ------------------------------------------------------------------ elementwise
// Activations use the hardware-exponential forms of the GEMM epilogue
// (relative error ~3e-7): with IEEE expf and division, GELU's arithmetic
// alone took half of a memory-bound pass.
__device__ __forceinline__ float unary_apply(int op, float x, float p) {
  switch (op) {
    case OXF_UNARY_SCALE: return x * p;
    case OXF_UNARY_ADD_SCALAR: return x + p;
    case OXF_UNARY_ACT_FORWARD: return act_forward_fast(static_cast<int>(p), x);
    case OXF_UNARY_ACT_DERIV: return act_derivative_fast(static_cast<int>(p), x);
    default: return 0.5f * x * x;
  }
}

enum EwOp { EW_BINARY, EW_BINARY_ASSIGN, EW_UNARY, EW_SGD, EW_MSE_GRAD, EW_BY_ROWS,
             EW_BINARY_BCAST, EW_MUL_ACT_DERIV };

// In-place activation over float4s, software-pipelined: each thread loads
// its next float4 before it computes and stores the current one, so the
// exponential and reciprocal of one piece overlap the load of the next.
template <int ACT>
__device__ __forceinline__ void act_forward_pipelined(float4* __restrict__ o, long long i,
                                                      long long stride, long long n4) {
  if (i >= n4) return;
  float4 x = o[i];
  while (true) {
    const long long nx = i + stride;
    float4 xn = make_float4(0.f, 0.f, 0.f, 0.f);
    if (nx < n4) xn = o[nx];
    o[i] = make_float4(act_forward_fast(ACT, x.x), act_forward_fast(ACT, x.y),
                       act_forward_fast(ACT, x.z), act_forward_fast(ACT, x.w));
    if (nx >= n4) break;
    x = xn;
    i = nx;
  }
}

// Grid-stride elementwise kernel; VEC processes float4s.
template <bool VEC>
__global__ void elementwise_kernel(int kind, int op, float* __restrict__ out,
                                   const float* __restrict__ a, const float* __restrict__ b,
                                   long long n, float p, long long cols) {
  pdl_launch();
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if constexpr (VEC) {
    // L2 prefetch of this block's 4 KB pieces of the full-length inputs (see
    // kPrefetchMaxBytes); a row-vector operand (by-rows kinds) stays in L2
    // anyway.
    const float* x_src = (kind == EW_BINARY || kind == EW_BINARY_BCAST || kind == EW_MSE_GRAD)
                             ? a : out;
    const float* y_src = (kind == EW_BINARY || kind == EW_BINARY_ASSIGN || kind == EW_SGD ||
                          kind == EW_MSE_GRAD || kind == EW_MUL_ACT_DERIV) ? b : nullptr;
    if (threadIdx.x == 0 && n * 4ll * (y_src ? 2 : 1) <= kPrefetchMaxBytes) {
      const long long n4 = n >> 2;
      for (long long c = static_cast<long long>(blockIdx.x) * blockDim.x; c < n4; c += stride) {
        const unsigned bytes =
            static_cast<unsigned>(min(n4 - c, static_cast<long long>(blockDim.x))) * 16u;
        prefetch_l2(reinterpret_cast<const float4*>(x_src) + c, bytes);
        if (y_src) prefetch_l2(reinterpret_cast<const float4*>(y_src) + c, bytes);
      }
    }
  }
  pdl_wait();
  if constexpr (VEC) {
    const long long n4 = n >> 2;
    if (kind == EW_UNARY && op == OXF_UNARY_ACT_FORWARD) {
      float4* o = reinterpret_cast<float4*>(out);
      switch (static_cast<int>(p)) {
        case OXF_ACT_GELU: act_forward_pipelined<OXF_ACT_GELU>(o, i, stride, n4); return;
        case OXF_ACT_SILU: act_forward_pipelined<OXF_ACT_SILU>(o, i, stride, n4); return;
        case OXF_ACT_RELU: act_forward_pipelined<OXF_ACT_RELU>(o, i, stride, n4); return;
        default: break;  // identity: the generic loop below
      }
    }
    for (; i < n4; i += stride) {
      float4 x = (kind == EW_BINARY || kind == EW_BINARY_BCAST)
                     ? reinterpret_cast<const float4*>(a)[i]
                     : reinterpret_cast<const float4*>(out)[i];
      float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
      if (kind == EW_BINARY || kind == EW_BINARY_ASSIGN || kind == EW_SGD ||
          kind == EW_MSE_GRAD)
        y = reinterpret_cast<const float4*>(b)[i];
      if (kind == EW_MSE_GRAD) x = reinterpret_cast<const float4*>(a)[i];
      if (kind == EW_BY_ROWS || kind == EW_BINARY_BCAST)
        y = reinterpret_cast<const float4*>(b)[(i * 4 % cols) >> 2];
      if (kind == EW_MUL_ACT_DERIV) y = reinterpret_cast<const float4*>(b)[i];
      float4 r;
      switch (kind) {
        case EW_MUL_ACT_DERIV:
          r = make_float4(x.x * act_derivative_fast(op, y.x), x.y * act_derivative_fast(op, y.y),
                          x.z * act_derivative_fast(op, y.z), x.w * act_derivative_fast(op, y.w));
          break;
        case EW_UNARY:
          r = make_float4(unary_apply(op, x.x, p), unary_apply(op, x.y, p),
                          unary_apply(op, x.z, p), unary_apply(op, x.w, p));
          break;
        case EW_SGD:
          r = make_float4(x.x - y.x * p, x.y - y.y * p, x.z - y.z * p, x.w - y.w * p);
          break;
        case EW_MSE_GRAD:
          r = make_float4((x.x - y.x) * p, (x.y - y.y) * p, (x.z - y.z) * p, (x.w - y.w) * p);
          break;
        default:
          r = make_float4(apply_binary(x.x, y.x, op), apply_binary(x.y, y.y, op),
                          apply_binary(x.z, y.z, op), apply_binary(x.w, y.w, op));
      }
      reinterpret_cast<float4*>(out)[i] = r;
    }
  } else {
    for (; i < n; i += stride) {
      float x = (kind == EW_BINARY || kind == EW_MSE_GRAD || kind == EW_BINARY_BCAST) ? a[i]
                                                                                   : out[i];
      float y = 0.f;
      if (kind == EW_BINARY || kind == EW_BINARY_ASSIGN || kind == EW_SGD ||
          kind == EW_MSE_GRAD || kind == EW_MUL_ACT_DERIV)
        y = b[i];
      if (kind == EW_BY_ROWS || kind == EW_BINARY_BCAST) y = b[i % cols];
      float r;
      switch (kind) {
        case EW_MUL_ACT_DERIV: r = x * act_derivative_fast(op, y); break;
        case EW_UNARY: r = unary_apply(op, x, p); break;
        case EW_SGD: r = x - y * p; break;
        case EW_MSE_GRAD: r = (x - y) * p; break;
        default: r = apply_binary(x, y, op);
      }
      out[i] = r;
    }
  }
}

// row.rs:5-14 (standalone): M[i,j] = -inf for j > i; one block per row.
__global__ void causal_mask_kernel(float* __restrict__ m, long long rows, long long cols) {
  pdl_enter();
  const long long r = blockIdx.x;
  for (long long c = r + 1 + threadIdx.x; c < cols; c += blockDim.x) m[r * cols + c] = -INFINITY;
}

// Column sums over a strip of 32 columns and a slice of rows; partial sums
// are combined with atomics into a zeroed (or accumulating) result.
__global__ void sum_cols_kernel(const float* __restrict__ m, float* __restrict__ out,
                                long long rows, long long cols, long long rows_per_block) {
  pdl_enter();
  __shared__ float part[8][33];
  const long long c = static_cast<long long>(blockIdx.x) * 32 + threadIdx.x;
  const long long r0 = static_cast<long long>(blockIdx.y) * rows_per_block;
  const long long r1 = min(rows, r0 + rows_per_block);
  float s = 0.f;
  if (c < cols)
    for (long long r = r0 + threadIdx.y; r < r1; r += 8) s += m[r * cols + c];
  part[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && c < cols) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += part[i][threadIdx.x];
    atomicAdd(out + c, t);
  }
}

// Column sums of a wide, short matrix (the position gradient: a few
// sequences' rows, S*H columns), where one strip of rows already covers the
// matrix: each thread owns four columns and sums all rows in order with
// 16-byte loads, four rows in flight at a time, and writes (or adds into)
// its outputs without atomics.
__global__ void sum_cols_vec_kernel(const float4* __restrict__ m, float4* __restrict__ out,
                                    long long rows, long long cols4, int accumulate) {
  pdl_enter();
  const long long c = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (c >= cols4) return;
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  auto add = [&s](const float4 v) {
    s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
  };
  long long r = 0;
  for (; r + 4 <= rows; r += 4) {
    const float4 a = __ldcs(m + r * cols4 + c);
    const float4 b = __ldcs(m + (r + 1) * cols4 + c);
    const float4 e = __ldcs(m + (r + 2) * cols4 + c);
    const float4 f = __ldcs(m + (r + 3) * cols4 + c);
    add(a); add(b); add(e); add(f);
  }
  for (; r < rows; ++r) add(__ldcs(m + r * cols4 + c));
  if (accumulate) {
    const float4 o = out[c];
    s = make_float4(o.x + s.x, o.y + s.y, o.z + s.z, o.w + s.w);
  }
  out[c] = s;
}

// layout.rs:9-55: 32x32 tiles through padded shared memory.
__global__ void transpose_kernel(const float* __restrict__ in, float* __restrict__ out,
                                 long long rows, long long cols) {
  pdl_enter();
  __shared__ float tile[32][33];
  const long long c = static_cast<long long>(blockIdx.x) * 32 + threadIdx.x;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const long long r = static_cast<long long>(blockIdx.y) * 32 + i;
    tile[i][threadIdx.x] = (r < rows && c < cols) ? in[r * cols + c] : 0.f;
  }
  __syncthreads();
  const long long oc = static_cast<long long>(blockIdx.y) * 32 + threadIdx.x;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const long long orow = static_cast<long long>(blockIdx.x) * 32 + i;
    if (orow < cols && oc < rows) out[orow * rows + oc] = tile[threadIdx.x][i];
  }
}

__device__ __forceinline__ void atomic_max_float(float* addr, float v) {
  if (v >= 0.f) atomicMax(reinterpret_cast<int*>(addr), __float_as_int(v));
  else atomicMin(reinterpret_cast<unsigned int*>(addr), __float_as_uint(v));
}

__global__ void fill_kernel(float* p, float v) {
  pdl_enter();
  *p = v;
}

// One-launch reductions (the reference re-launches slice_sum from the host
// until one element is left, span.rs:361-385). map_op >= 0 sums
// unary_apply(map_op, x, map_p) instead of x (slice_map_sum).
// Sum or max of x (each element first mapped by map_op when >= 0), or the
// dot product with y when y is given.
__global__ void slice_reduce_kernel(const float* __restrict__ x, long long n, float* result,
                                    int is_max, int map_op, float map_p,
                                    const float* __restrict__ y) {
  pdl_enter();
  __shared__ float red[32];
  float acc = is_max ? -FLT_MAX : 0.f;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float v = y ? x[i] * y[i] : map_op >= 0 ? unary_apply(map_op, x[i], map_p) : x[i];
    acc = is_max ? fmaxf(acc, v) : acc + v;
  }
  acc = is_max ? block_max(acc, red) : block_sum(acc, red);
  if (threadIdx.x == 0) {
    if (is_max) atomic_max_float(result, acc);
    else atomicAdd(result, acc);
  }
}

// slice_set / slice_set_seq / slice_set_random (elementwise.rs:15-43).
enum FillKind { FILL_VALUE, FILL_SEQ, FILL_RANDOM };

// The reference's integer hash (common.rs:3-9), wrapping 32-bit arithmetic.
__device__ __forceinline__ uint32_t ref_hash(uint32_t x) {
  x += x << 13;
  x -= x >> 17;
  x *= x << 5;
  return x;
}

__global__ void fill_slice_kernel(float* __restrict__ out, long long n, int kind, float value,
                                  int dir, uint32_t seed) {
  pdl_enter();
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float v = value;
    if (kind == FILL_SEQ) {
      v = dir ? static_cast<float>(i) : static_cast<float>(n - i);
    } else if (kind == FILL_RANDOM) {
      // (hash as f32) / (u32::MAX as f32); u32::MAX rounds to 2^32 in f32.
      v = static_cast<float>(ref_hash(seed + static_cast<uint32_t>(i))) / 4294967296.0f;
    }
    out[i] = v;
  }
}

// matrix_slice (layout.rs:58-86): output element l of tile l / (tr*tc).
__global__ void matrix_slice_kernel(const float* __restrict__ in, float* __restrict__ out,
                                    long long n, long long input_cols, long long tile_rows,
                                    long long tile_cols, long long tiles_per_row) {
  pdl_enter();
  const long long tile = tile_rows * tile_cols;
  for (long long l = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; l < n;
       l += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long ti = l / tile, local = l - ti * tile;
    const long long ty = ti / tiles_per_row, tx = ti - ty * tiles_per_row;
    const long long r = ty * tile_rows + local / tile_cols;
    const long long c = tx * tile_cols + local % tile_cols;
    out[l] = in[r * input_cols + c];
  }
}

// ================================================================== host side
namespace {

// Launches `kernel` with programmatic stream serialisation (see pdl_enter)
// and counts it; returns the launch status.
template <typename... KArgs, typename... Args>
oxf_status launch_pdl(const char* name, void (*kernel)(KArgs...), dim3 grid, dim3 block,
                      cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  count_launch();
  return check_cuda(e != cudaSuccess ? e : cudaGetLastError(), name);
}

int sm_count_rows() {
  static int c = 0;
  if (!c) {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    c = v > 0 ? v : 148;
  }
  return c;
}

bool fits_int(long long v) { return v >= 0 && v <= 0x7fffffffll; }

// Launches `K<G,NV>` for the smallest register footprint that holds the
// row, or returns false if the row needs the looped path.
template <template <int, int> class Launcher, typename... Args>
bool dispatch_row(long long rows, long long cols, cudaStream_t s, oxf_status* st,
                  Args... args) {
  if (cols % 4 != 0 || cols > 16384 || !fits_int(cols)) return false;
  const long long c4 = cols / 4;
  if (c4 <= 32) return Launcher<32, 1>::go(rows, s, st, args...);
  if (c4 <= 64) return Launcher<32, 2>::go(rows, s, st, args...);
  if (c4 <= 128) return Launcher<32, 4>::go(rows, s, st, args...);
  if (c4 <= 256) return Launcher<32, 8>::go(rows, s, st, args...);
  if (c4 <= 512) return Launcher<32, 16>::go(rows, s, st, args...);
  if (c4 <= 1024) return Launcher<128, 8>::go(rows, s, st, args...);
  if (c4 <= 2048) return Launcher<256, 8>::go(rows, s, st, args...);
  return Launcher<256, 16>::go(rows, s, st, args...);
}

template <int G>
dim3 row_grid(long long rows, int& threads) {
  if (G == 32) {
    threads = 256;
    return dim3(static_cast<unsigned>((rows + 7) / 8));
  }
  threads = G;
  return dim3(static_cast<unsigned>(rows));
}

// go() launches the kernel (its status goes to *st) and returns true;
// dispatch_row returns false instead when no instantiation fits the row.
#define OXF_ROW_LAUNCHER(NAME, KERNEL, PARAMS, ARGS)                         \
  template <int G, int NV>                                                   \
  struct NAME {                                                              \
    static bool go(long long rows, cudaStream_t s, oxf_status* st, PARAMS) { \
      int threads;                                                           \
      dim3 grid = row_grid<G>(rows, threads);                                \
      *st = launch_pdl(#KERNEL, KERNEL<G, NV>, grid, dim3(threads), s, ARGS); \
      return true;                                                           \
    }                                                                        \
  };

#define P_(...) __VA_ARGS__
OXF_ROW_LAUNCHER(SoftmaxFwdL, softmax_fwd_kernel,
                 P_(float* m, int cols, float scale, long long period),
                 P_(m, rows, cols, scale, period))
OXF_ROW_LAUNCHER(SoftmaxBwdL, softmax_bwd_kernel,
                 P_(const float* p, const float* dy, float* dx, int cols, float scale),
                 P_(p, dy, dx, rows, cols, scale))
OXF_ROW_LAUNCHER(LnFwdL, layernorm_fwd_kernel,
                 P_(const float* in, float* out, int cols, float eps, const float* g,
                    const float* b),
                 P_(in, out, rows, cols, eps, g, b))
OXF_ROW_LAUNCHER(LnFwdStagedL, layernorm_fwd_staged_kernel,
                 P_(const float* in, float* out, int cols, float eps, const float* g,
                    const float* b),
                 P_(in, out, rows, cols, eps, g, b))
OXF_ROW_LAUNCHER(LnBwdL, layernorm_bwd_kernel,
                 P_(const float* x, const float* dy, float* dx, int cols, float eps),
                 P_(x, dy, dx, rows, cols, eps))
OXF_ROW_LAUNCHER(RmsFwdL, rmsnorm_fwd_kernel,
                 P_(const float* in, float* out, int cols, float eps, const float* g),
                 P_(in, out, rows, cols, eps, g))
OXF_ROW_LAUNCHER(RmsFwdStagedL, rmsnorm_fwd_staged_kernel,
                 P_(const float* in, float* out, int cols, float eps, const float* g),
                 P_(in, out, rows, cols, eps, g))
OXF_ROW_LAUNCHER(RmsBwdL, rmsnorm_bwd_kernel,
                 P_(const float* x, const float* dy, float* dx, int cols, float eps),
                 P_(x, dy, dx, rows, cols, eps))
OXF_ROW_LAUNCHER(SumRowsL, sum_rows_kernel, P_(const float* m, float* out, int cols),
                 P_(m, out, rows, cols))
OXF_ROW_LAUNCHER(LossGradL, loss_grad_rows_kernel,
                 P_(const float* y, const float* t, float* out, float* dy, int cols),
                 P_(y, t, out, dy, rows, cols))
OXF_ROW_LAUNCHER(LossRowsL, loss_rows_kernel,
                 P_(const float* y, const float* t, float* out, int cols), P_(y, t, out, rows, cols))
#undef P_

bool al(const void* p) { return p == nullptr || aligned16(p); }

oxf_status looped(int op, float* out, const float* a, const float* b, long long rows,
                  long long cols, float p0, float p1, long long period, const float* g,
                  const float* be, cudaStream_t s) {
  if (rows > 0x7fffffffll) return set_error(OXF_ERR_UNSUPPORTED_SHAPE, "too many rows");
  return launch_pdl("row_looped_kernel", row_looped_kernel, dim3(static_cast<unsigned>(rows)),
                    dim3(256), s, op, out, a, b, cols, p0, p1, period, g, be);
}

unsigned ew_blocks(long long work) {
  const long long per = 256;
  long long b = (work + per - 1) / per;
  const long long cap = static_cast<long long>(sm_count_rows()) * 16;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return static_cast<unsigned>(b);
}

oxf_status elementwise(int kind, int op, float* out, const float* a, const float* b, long long n,
                       float p, long long cols, cudaStream_t s) {
  if (n <= 0) return OXF_OK;
  bool vec = al(out) && al(a) && al(b) && (n % 4 == 0);
  if (kind == EW_BY_ROWS || kind == EW_BINARY_BCAST) vec = vec && (cols % 4 == 0);
  if (vec)
    return launch_pdl("elementwise_kernel", elementwise_kernel<true>, dim3(ew_blocks(n / 4)),
                      dim3(256), s, kind, op, out, a, b, n, p, cols);
  return launch_pdl("elementwise_kernel", elementwise_kernel<false>, dim3(ew_blocks(n)),
                    dim3(256), s, kind, op, out, a, b, n, p, cols);
}

}  // namespace

// ------------------------------------------------------------------ internal API
oxf_status rows_softmax(float* m, long long rows, long long cols, float scale, long long period,
                        cudaStream_t s) {
  if (rows == 0 || cols == 0) return OXF_OK;
  oxf_status st = OXF_OK;
  if (al(m) && dispatch_row<SoftmaxFwdL>(rows, cols, s, &st, m, static_cast<int>(cols), scale, period))
    return st;
  return looped(LOOP_SOFTMAX, m, m, nullptr, rows, cols, scale, 0.f, period, nullptr, nullptr, s);
}

oxf_status rows_softmax_bwd(const float* p, const float* dy, float* dx, long long rows,
                            long long cols, float scale, cudaStream_t s) {
  if (rows == 0 || cols == 0) return OXF_OK;
  oxf_status st = OXF_OK;
  if (al(p) && al(dy) && al(dx) &&
      dispatch_row<SoftmaxBwdL>(rows, cols, s, &st, p, dy, dx, static_cast<int>(cols), scale))
    return st;
  return looped(LOOP_SOFTMAX_BWD, dx, p, dy, rows, cols, scale, 0.f, 0, nullptr, nullptr, s);
}

oxf_status rows_layernorm(const float* in, float* out, long long rows, long long cols, float eps,
                          const float* g, const float* b, cudaStream_t s) {
  if (rows == 0 || cols == 0) return OXF_OK;
  oxf_status st = OXF_OK;
  if (al(in) && al(out) && al(g) && al(b) &&
      ((g || b) ? dispatch_row<LnFwdStagedL>(rows, cols, s, &st, in, out, static_cast<int>(cols),
                                             eps, g, b)
                : dispatch_row<LnFwdL>(rows, cols, s, &st, in, out, static_cast<int>(cols), eps,
                                       g, b)))
    return st;
  return looped(LOOP_LN, out, in, nullptr, rows, cols, eps, 0.f, 0, g, b, s);
}

oxf_status rows_layernorm_bwd(const float* x, const float* dy, float* dx, long long rows,
                              long long cols, float eps, cudaStream_t s) {
  if (rows == 0 || cols == 0) return OXF_OK;
  oxf_status st = OXF_OK;
  if (al(x) && al(dy) && al(dx) &&
      dispatch_row<LnBwdL>(rows, cols, s, &st, x, dy, dx, static_cast<int>(cols), eps))
    return st;
  return looped(LOOP_LN_BWD, dx, x, dy, rows, cols, eps, 0.f, 0, nullptr, nullptr, s);
}

oxf_status rows_rmsnorm(const float* in, float* out, long long rows, long long cols, float eps,
                        const float* g, cudaStream_t s) {
  if (rows == 0 || cols == 0) return OXF_OK;
  oxf_status st = OXF_OK;
  if (al(in) && al(out) && al(g) &&
      (g ? dispatch_row<RmsFwdStagedL>(rows, cols, s, &st, in, out, static_cast<int>(cols), eps, g)
         : dispatch_row<RmsFwdL>(rows, cols, s, &st, in, out, static_cast<int>(cols), eps, g)))
    return st;
  return looped(LOOP_RMS, out, in, nullptr, rows, cols, eps, 0.f, 0, g, nullptr, s);
}

oxf_status rows_rmsnorm_bwd(const float* x, const float* dy, float* dx, long long rows,
                            long long cols, float eps, cudaStream_t s) {
  if (rows == 0 || cols == 0) return OXF_OK;
  oxf_status st = OXF_OK;
  if (al(x) && al(dy) && al(dx) &&
      dispatch_row<RmsBwdL>(rows, cols, s, &st, x, dy, dx, static_cast<int>(cols), eps))
    return st;
  return looped(LOOP_RMS_BWD, dx, x, dy, rows, cols, eps, 0.f, 0, nullptr, nullptr, s);
}

oxf_status rows_sum(const float* m, float* out, long long rows, long long cols, cudaStream_t s) {
  if (rows == 0) return OXF_OK;
  if (cols == 0) return check_cuda(cudaMemsetAsync(out, 0, rows * 4, s), "memset");
  oxf_status st = OXF_OK;
  if (al(m) && dispatch_row<SumRowsL>(rows, cols, s, &st, m, out, static_cast<int>(cols)))
    return st;
  return looped(LOOP_SUM, out, m, nullptr, rows, cols, 0.f, 0.f, 0, nullptr, nullptr, s);
}

oxf_status rows_loss(const float* y, const float* t, float* out, long long rows, long long cols,
                     cudaStream_t s) {
  if (rows == 0) return OXF_OK;
  if (cols == 0) return check_cuda(cudaMemsetAsync(out, 0, rows * 4, s), "memset");
  oxf_status st = OXF_OK;
  if (al(y) && al(t) && dispatch_row<LossRowsL>(rows, cols, s, &st, y, t, out, static_cast<int>(cols)))
    return st;
  return looped(LOOP_LOSS, out, y, t, rows, cols, 0.f, 0.f, 0, nullptr, nullptr, s);
}

oxf_status ew_mse_grad(const float*, const float*, float*, long long, long long, cudaStream_t);

oxf_status rows_loss_grad(const float* y, const float* t, float* out, float* dy, long long rows,
                          long long cols, cudaStream_t s) {
  if (rows == 0) return OXF_OK;
  oxf_status st = OXF_OK;
  if (al(y) && al(t) && al(dy) &&
      dispatch_row<LossGradL>(rows, cols, s, &st, y, t, out, dy, static_cast<int>(cols)))
    return st;
  st = rows_loss(y, t, out, rows, cols, s);
  if (st != OXF_OK) return st;
  return ew_mse_grad(y, t, dy, rows * cols, cols, s);
}

oxf_status ew_binary(const float* a, const float* b, float* out, long long n, int op,
                     cudaStream_t s) {
  return elementwise(EW_BINARY, op, out, a, b, n, 0.f, 1, s);
}
oxf_status ew_binary_assign(float* t, const float* b, long long n, int op, cudaStream_t s) {
  return elementwise(EW_BINARY_ASSIGN, op, t, nullptr, b, n, 0.f, 1, s);
}
oxf_status ew_unary(float* x, long long n, int op, float p, cudaStream_t s) {
  return elementwise(EW_UNARY, op, x, nullptr, nullptr, n, p, 1, s);
}
oxf_status ew_sgd(float* w, const float* g, long long n, float lr, cudaStream_t s) {
  return elementwise(EW_SGD, 0, w, nullptr, g, n, lr, 1, s);
}
oxf_status ew_mse_grad(const float* y, const float* t, float* out, long long n, long long cols,
                       cudaStream_t s) {
  return elementwise(EW_MSE_GRAD, 0, out, y, t, n, 1.0f / static_cast<float>(cols), 1, s);
}
oxf_status ew_by_rows(float* m, const float* row, long long n, long long cols, int op,
                      cudaStream_t s) {
  return elementwise(EW_BY_ROWS, op, m, nullptr, row, n, 0.f, cols, s);
}
oxf_status ew_binary_bcast(const float* a, const float* b, float* out, long long n,
                           long long period, int op, cudaStream_t s) {
  return elementwise(EW_BINARY_BCAST, op, out, a, b, n, 0.f, period, s);
}
oxf_status ew_mul_act_deriv(float* g, const float* pre, long long n, int act, cudaStream_t s) {
  return elementwise(EW_MUL_ACT_DERIV, act, g, nullptr, pre, n, 0.f, 1, s);
}

oxf_status causal_mask(float* m, long long rows, long long cols, cudaStream_t s) {
  if (rows == 0 || cols == 0) return OXF_OK;
  if (rows > 0x7fffffffll) return set_error(OXF_ERR_UNSUPPORTED_SHAPE, "causal mask: rows");
  return launch_pdl("causal_mask_kernel", causal_mask_kernel, dim3(static_cast<unsigned>(rows)),
                    dim3(256), s, m, rows, cols);
}

oxf_status cols_sum(const float* m, float* out, long long rows, long long cols, int accumulate,
                    cudaStream_t s) {
  if (cols == 0) return OXF_OK;
  // Wide and short (fewer rows than one strip of the strip kernel takes):
  // one thread per four columns, no atomics.
  if (rows > 0 && rows <= 128 && cols % 4 == 0 && aligned16(m) && aligned16(out) &&
      (cols + 31) / 32 >= 2ll * sm_count_rows() * 4) {
    const long long cols4 = cols / 4;
    if ((cols4 + 255) / 256 > 0x7fffffffll)
      return set_error(OXF_ERR_UNSUPPORTED_SHAPE, "too many columns");
    return launch_pdl("sum_cols_vec_kernel", sum_cols_vec_kernel,
                      dim3(static_cast<unsigned>((cols4 + 255) / 256)), dim3(256), s,
                      reinterpret_cast<const float4*>(m), reinterpret_cast<float4*>(out), rows,
                      cols4, accumulate);
  }
  if (!accumulate) {
    oxf_status st = check_cuda(cudaMemsetAsync(out, 0, cols * 4, s), "memset");
    if (st != OXF_OK) return st;
  }
  if (rows == 0) return OXF_OK;
  const long long strips = (cols + 31) / 32;
  long long slices = std::max<long long>(1, (2ll * sm_count_rows() * 4) / strips);
  slices = std::min<long long>(slices, (rows + 63) / 64);
  slices = std::max<long long>(1, std::min<long long>(slices, 65535));
  const long long per = (rows + slices - 1) / slices;
  slices = (rows + per - 1) / per;
  if (strips > 0x7fffffffll) return set_error(OXF_ERR_UNSUPPORTED_SHAPE, "too many columns");
  return launch_pdl("sum_cols_kernel", sum_cols_kernel,
                    dim3(static_cast<unsigned>(strips), static_cast<unsigned>(slices)),
                    dim3(32, 8), s, m, out, rows, cols, per);
}

oxf_status transpose(const float* in, float* out, long long rows, long long cols,
                     cudaStream_t s) {
  if (rows == 0 || cols == 0) return OXF_OK;
  if ((rows + 31) / 32 > 65535) return set_error(OXF_ERR_UNSUPPORTED_SHAPE, "transpose: rows");
  dim3 grid(static_cast<unsigned>((cols + 31) / 32), static_cast<unsigned>((rows + 31) / 32));
  return launch_pdl("transpose_kernel", transpose_kernel, grid, dim3(32, 8), s, in, out, rows,
                    cols);
}

oxf_status slice_reduce(const float* x, long long n, float* result, int is_max, cudaStream_t s,
                        int map_op, float map_p, const float* y) {
  const oxf_status st = launch_pdl("fill_kernel", fill_kernel, dim3(1), dim3(1), s, result,
                                   is_max ? -FLT_MAX : 0.f);
  if (st != OXF_OK || n <= 0) return st;
  return launch_pdl("slice_reduce_kernel", slice_reduce_kernel, dim3(ew_blocks((n + 3) / 4)),
                    dim3(256), s, x, n, result, is_max, map_op, map_p, y);
}

oxf_status fill_slice(float* out, long long n, int kind, float value, int dir, uint32_t seed,
                      cudaStream_t s) {
  if (n <= 0) return OXF_OK;
  return launch_pdl("fill_slice_kernel", fill_slice_kernel, dim3(ew_blocks(n)), dim3(256), s, out,
                    n, kind, value, dir, seed);
}

oxf_status matrix_slice(const float* in, float* out, long long n, long long input_cols,
                        long long tile_rows, long long tile_cols, long long tiles_per_row,
                        cudaStream_t s) {
  if (n <= 0) return OXF_OK;
  return launch_pdl("matrix_slice_kernel", matrix_slice_kernel, dim3(ew_blocks(n)), dim3(256), s,
                    in, out, n, input_cols, tile_rows, tile_cols, tiles_per_row);
}

oxf_status rows_read_device_error(uint32_t* code) {
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_oxf_device_error, sizeof(v));
  if (e != cudaSuccess) return check_cuda(e, "read device error word");
  const uint32_t zero = 0;
  e = cudaMemcpyToSymbol(g_oxf_device_error, &zero, sizeof(zero));
  if (e != cudaSuccess) return check_cuda(e, "clear device error word");
  *code = v;
  return OXF_OK;
}

}  // namespace oxf
