// exchange.cu — data-parallel SGD fused with the gradient exchange, one
// kernel per rank over NVLink peer memory (oxf_exchange_sgd in oxf.h).
//
// The reference trains on one GPU (src/cuda/runtime.rs:34-45) and updates
// each Linear with W -= lr * dW (src/net/linear.rs:373-391). Across ranks the
// same update needs the sum of every rank's gradient. A library all-reduce
// followed by an update kernel moves each gradient byte over NVLink twice
// (reduce-scatter + all-gather) and then streams the whole arena through
// HBM once more for the update. Here rank r owns 1/world of the range: it
// pulls that shard's gradients from every rank (peer loads), adds them in
// rank order, applies the update to its copy of the parameters, and pushes
// the updated shard into every rank's parameter arena (peer stores). Each
// byte crosses NVLink once per direction and the update is done once per
// element, by its owner.
//
// HBM / NVLink traffic per rank for n elements: reads n*4 bytes of gradients
// ((world-1)/world of them remote) and n/world*4 bytes of parameters; writes
// n*4 bytes of parameters ((world-1)/world remote).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "../../include/oxf.h"
#include "ptx.cuh"
#include "status.cuh"

namespace oxf {
namespace {

constexpr int XCH_THREADS = 256;
constexpr unsigned long long XCH_DEFAULT_LIMIT_NS = 4000000000ull;  // 4 s
constexpr unsigned long long XCH_MAX_LIMIT_NS = 60000000000ull;     // 60 s

struct XchArgs {
  float* params[OXF_EXCHANGE_MAX_RANKS];
  const float* grads[OXF_EXCHANGE_MAX_RANKS];
  uint32_t* signals[OXF_EXCHANGE_MAX_RANKS];
  int rank;
  uint32_t epoch;
  unsigned long long limit_ns;
  float lr;
  long long base;         // element index of float4 unit 0 (a multiple of 4)
  long long u0, u1;       // this rank's float4 units [u0, u1)
  long long head, tail;   // first element of the scalar head / tail
  int n_head, n_tail;     // their lengths (<= 3 each; nonzero on rank 0 only)
};

// Slot of the pad word that rank `src` sets for CTA `block` at `phase`
// (0 = start, 1 = end).
__device__ __forceinline__ size_t pad_slot(int phase, int block, int src) {
  return (static_cast<size_t>(phase) * OXF_EXCHANGE_MAX_BLOCKS + block) * OXF_EXCHANGE_MAX_RANKS +
         src;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Epochs grow by one per call; a pad word has reached `epoch` when it holds
// it or a later one (a peer may already be one call ahead on the end pad).
__device__ __forceinline__ bool reached(uint32_t v, uint32_t epoch) {
  return static_cast<int32_t>(v - epoch) >= 0;
}

// CTA b of this rank meets CTA b of every rank. Thread q < W stores this
// rank's arrival into rank q's pad (release, system scope, after a system
// fence that orders every store the CTA made before the preceding
// __syncthreads), then waits, bounded, for rank q's arrival in this rank's
// pad. Returns false on expiry (after recording `code`).
// The outcome is combined with __syncthreads_and, so the kernel needs no
// shared memory: a block then fits beside a GEMM CTA that holds all of its
// SM's shared memory but one kilobyte, and overlapped exchanges do not keep
// GEMM CTAs off their SMs.
template <int W>
__device__ bool rank_barrier(const XchArgs& a, int phase, uint32_t code) {
  __syncthreads();
  const int q = threadIdx.x;
  int ok = 1;
  if (q < W) {
    __threadfence_system();
    st_release_sys(a.signals[q] + pad_slot(phase, blockIdx.x, a.rank), a.epoch);
    const uint32_t* in = a.signals[a.rank] + pad_slot(phase, blockIdx.x, q);
    if (!reached(ld_acquire_sys(in), a.epoch)) {
      const unsigned long long t0 = global_timer_ns();
      while (!reached(ld_acquire_sys(in), a.epoch)) {
        __nanosleep(64);
        if (global_timer_ns() - t0 > a.limit_ns) {
          report_device_error(code);
          ok = 0;
          break;
        }
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

__device__ __forceinline__ float4 ld4(const float* p) {
  return __ldcg(reinterpret_cast<const float4*>(p));
}

__device__ __forceinline__ void st4(float* p, float4 v) {
  __stcg(reinterpret_cast<float4*>(p), v);
}

// p - lr * (g[0] + g[1] + ... + g[W-1]), the expression of the update
// kernel (x - y * lr), so world 1 matches oxf_sgd_update bit for bit.
template <int W>
__device__ __forceinline__ float4 update(float4 p, const float4 (&g)[W], float lr) {
  float4 s = g[0];
#pragma unroll
  for (int q = 1; q < W; ++q) {
    s.x += g[q].x;
    s.y += g[q].y;
    s.z += g[q].z;
    s.w += g[q].w;
  }
  return make_float4(p.x - s.x * lr, p.y - s.y * lr, p.z - s.z * lr, p.w - s.w * lr);
}

// U float4 units per thread and iteration, so that every thread has up to
// eight 16-byte loads in flight (fewer at world 4, to stay in 40 registers).
// At most 40 registers per thread (six 256-thread blocks' worth per SM): a
// block then also fits in the registers a GEMM CTA leaves free.
template <int W, int U>
__global__ void __launch_bounds__(XCH_THREADS, 6)
    exchange_sgd_kernel(const __grid_constant__ XchArgs a) {
  if (!rank_barrier<W>(a, 0, OXF_DEVERR_EXCHANGE_START)) return;

  const long long stride = static_cast<long long>(gridDim.x) * XCH_THREADS;
  long long u = a.u0 + static_cast<long long>(blockIdx.x) * XCH_THREADS + threadIdx.x;
  const float* mine = a.params[a.rank];
  for (; u + (U - 1) * stride < a.u1; u += U * stride) {
    float4 g[U][W], p[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const long long e = a.base + 4 * (u + j * stride);
#pragma unroll
      for (int q = 0; q < W; ++q) g[j][q] = ld4(a.grads[q] + e);
      p[j] = ld4(mine + e);
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const long long e = a.base + 4 * (u + j * stride);
      const float4 r = update<W>(p[j], g[j], a.lr);
#pragma unroll
      for (int q = 0; q < W; ++q) st4(a.params[q] + e, r);
    }
  }
  for (; u < a.u1; u += stride) {
    const long long e = a.base + 4 * u;
    float4 g[W];
#pragma unroll
    for (int q = 0; q < W; ++q) g[q] = ld4(a.grads[q] + e);
    const float4 r = update<W>(ld4(mine + e), g, a.lr);
#pragma unroll
    for (int q = 0; q < W; ++q) st4(a.params[q] + e, r);
  }
  // Up to three elements before and after the 16-byte-aligned interior.
  if (blockIdx.x == 0 && threadIdx.x < a.n_head + a.n_tail) {
    const int t = threadIdx.x;
    const long long e = t < a.n_head ? a.head + t : a.tail + (t - a.n_head);
    float s = __ldcg(a.grads[0] + e);
#pragma unroll
    for (int q = 1; q < W; ++q) s += __ldcg(a.grads[q] + e);
    const float r = __ldcg(mine + e) - s * a.lr;
#pragma unroll
    for (int q = 0; q < W; ++q) __stcg(a.params[q] + e, r);
  }

  rank_barrier<W>(a, 1, OXF_DEVERR_EXCHANGE_END);
}

template <int W>
cudaError_t launch_world(const XchArgs& a, int blocks, cudaStream_t s) {
  constexpr int U = W <= 2 ? 4 : W <= 3 ? 2 : 1;  // within 40 registers, no spills
  exchange_sgd_kernel<W, U><<<blocks, XCH_THREADS, 0, s>>>(a);
  return cudaGetLastError();
}

int sm_count() {
  int dev = 0, c = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0)
    return 148;
  return c;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

using GetAddressRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

GetAddressRange address_range_fn() {
  static GetAddressRange fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<GetAddressRange>(p);
    return static_cast<GetAddressRange>(nullptr);
  }();
  return fn;
}

}  // namespace

oxf_status exchange_sgd(const oxf_exchange_desc* d, size_t offset, size_t count, float lr,
                        cudaStream_t s) {
  if (!d) return set_error(OXF_ERR_INVALID_ARG, "oxf_exchange_sgd: null descriptor");
  const int W = d->world;
  if (W < 1 || W > OXF_EXCHANGE_MAX_RANKS)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_exchange_sgd: world must be 1..%d",
                     OXF_EXCHANGE_MAX_RANKS);
  if (d->rank < 0 || d->rank >= W)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_exchange_sgd: rank outside 0..world-1");
  if (d->epoch == 0) return set_error(OXF_ERR_INVALID_ARG, "oxf_exchange_sgd: epoch must be > 0");
  if (d->blocks < 0 || d->blocks > OXF_EXCHANGE_MAX_BLOCKS)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_exchange_sgd: blocks must be 0..%d",
                     OXF_EXCHANGE_MAX_BLOCKS);
  for (int q = 0; q < W; ++q) {
    if (!d->params[q] || !d->grads[q] || !d->signals[q])
      return set_error(OXF_ERR_INVALID_ARG, "oxf_exchange_sgd: null pointer for rank %d", q);
    if (!aligned16(d->params[q]) || !aligned16(d->grads[q]) || !aligned16(d->signals[q]))
      return set_error(OXF_ERR_INVALID_ARG,
                       "oxf_exchange_sgd: arenas and pads must be 16-byte aligned (rank %d)", q);
  }
  if (count == 0) return OXF_OK;

  XchArgs a;
  std::memset(&a, 0, sizeof(a));
  for (int q = 0; q < W; ++q) {
    a.params[q] = d->params[q];
    a.grads[q] = d->grads[q];
    a.signals[q] = d->signals[q];
  }
  a.rank = d->rank;
  a.epoch = d->epoch;
  a.lr = lr;
  unsigned long long limit =
      d->timeout_us ? static_cast<unsigned long long>(d->timeout_us) * 1000ull
                    : XCH_DEFAULT_LIMIT_NS;
  a.limit_ns = limit < XCH_MAX_LIMIT_NS ? limit : XCH_MAX_LIMIT_NS;

  // The 16-byte-aligned interior [a0, a1) is split into world shards of
  // float4 units; the scalar head [offset, a0) and tail [a1, end) go to
  // rank 0. Every quantity but u0/u1 is the same on all ranks.
  const long long off = static_cast<long long>(offset), end = off + static_cast<long long>(count);
  long long a0 = (off + 3) & ~3ll;
  if (a0 > end) a0 = end;
  long long a1 = end & ~3ll;
  if (a1 < a0) a1 = a0;
  const long long units = (a1 - a0) / 4;
  const long long per = (units + W - 1) / W;
  a.base = a0;
  a.u0 = per * d->rank < units ? per * d->rank : units;
  a.u1 = a.u0 + per < units ? a.u0 + per : units;
  a.head = off;
  a.tail = a1;
  if (d->rank == 0) {
    a.n_head = static_cast<int>(a0 - off);
    a.n_tail = static_cast<int>(end - a1);
  }

  long long want = (per + XCH_THREADS - 1) / XCH_THREADS;
  if (want < 1) want = 1;
  long long blocks = d->blocks ? d->blocks : sm_count();
  if (blocks > want) blocks = want;
  if (blocks > OXF_EXCHANGE_MAX_BLOCKS) blocks = OXF_EXCHANGE_MAX_BLOCKS;
  const int nb = static_cast<int>(blocks);

  cudaError_t e;
  switch (W) {
    case 1: e = launch_world<1>(a, nb, s); break;
    case 2: e = launch_world<2>(a, nb, s); break;
    case 3: e = launch_world<3>(a, nb, s); break;
    case 4: e = launch_world<4>(a, nb, s); break;
    case 5: e = launch_world<5>(a, nb, s); break;
    case 6: e = launch_world<6>(a, nb, s); break;
    case 7: e = launch_world<7>(a, nb, s); break;
    default: e = launch_world<8>(a, nb, s); break;
  }
  count_launch();
  return check_cuda(e, "exchange_sgd_kernel launch");
}

oxf_status exchange_read_device_error(uint32_t* code) {
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_oxf_device_error, sizeof(v));
  if (e != cudaSuccess) return check_cuda(e, "read device error word");
  const uint32_t zero = 0;
  e = cudaMemcpyToSymbol(g_oxf_device_error, &zero, sizeof(zero));
  if (e != cudaSuccess) return check_cuda(e, "clear device error word");
  *code = v;
  return OXF_OK;
}

oxf_status ipc_export(const void* ptr, oxf_ipc_handle* out) {
  if (!ptr || !out) return set_error(OXF_ERR_INVALID_ARG, "oxf_ipc_export: null argument");
  GetAddressRange range = address_range_fn();
  if (!range) return set_error(OXF_ERR_CUDA, "oxf_ipc_export: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_ipc_export: not device memory of this context");
  cudaIpcMemHandle_t h;
  oxf_status st = check_cuda(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)),
                             "cudaIpcGetMemHandle");
  if (st != OXF_OK) return st;
  static_assert(sizeof(h) <= sizeof(out->handle), "IPC handle size");
  std::memset(out, 0, sizeof(*out));
  std::memcpy(out->handle, &h, sizeof(h));
  out->offset = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return OXF_OK;
}

oxf_status ipc_open(const oxf_ipc_handle* handle, void** ptr) {
  if (!handle || !ptr) return set_error(OXF_ERR_INVALID_ARG, "oxf_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->handle, sizeof(h));
  void* base = nullptr;
  oxf_status st = check_cuda(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess),
                             "cudaIpcOpenMemHandle");
  if (st != OXF_OK) return st;
  *ptr = static_cast<char*>(base) + handle->offset;
  return OXF_OK;
}

oxf_status ipc_close(const oxf_ipc_handle* handle, void* ptr) {
  if (!handle || !ptr) return set_error(OXF_ERR_INVALID_ARG, "oxf_ipc_close: null argument");
  return check_cuda(cudaIpcCloseMemHandle(static_cast<char*>(ptr) - handle->offset),
                    "cudaIpcCloseMemHandle");
}

}  // namespace oxf
