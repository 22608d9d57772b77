// gemm.cu — TF32 GEMM on the 5th-generation tensor cores (sm_100a).
//
// Replaces matrix_multiply (src/cuda/device/module.rs:179-191 ->
// src/cuda/device/gemm.rs:202-373) and the transposes the reference runs
// before every backward product (src/net/linear.rs:381,432;
// src/net/transformer/attention.rs:297-307,367): operands are read in the
// layout they are stored in, K-major or MN-major, straight from HBM by TMA.
//
// Kernel shape (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: fills a STAGES-deep shared-memory ring
//               (128B-swizzled tiles, mbarrier transaction counts)
//   warp 1      TMEM allocator + MMA issuer: tcgen05.mma.kind::tf32,
//               M=128 x N=BN x K=8 per instruction, accumulators in TMEM,
//               tcgen05.commit frees ring slots and publishes accumulators
//   warps 2..9  epilogue: tcgen05.ld, fused alpha/beta/bias/residual/
//               pre-activation store/activation(-gradient); two warps per
//               TMEM lane quarter take alternate 32-column chunks, so every
//               SM sub-partition runs two epilogue warps. Epilogue operands
//               (C for beta, residual, aux) arrive and results (pre-
//               activation, C) leave as 32 x 32 TMA tiles staged in shared
//               memory, so every global access is a full-line bulk copy.
// Two TMEM accumulators (2*BN columns) let the epilogue of tile i overlap
// the main loop of tile i+1. No cluster multicast is used anywhere.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "ptx.cuh"
#include "tmap.hpp"
#include "umma.cuh"
#include "status.cuh"

namespace oxf {

constexpr int BM = 128;       // tile rows (TMEM lanes)
constexpr int BK = 32;        // K elements per ring slot: 32 x f32 = one 128-byte swizzle row
constexpr int UMMA_K = 8;     // K per tcgen05.mma.kind::tf32
constexpr int EPI_WARPS = 8;  // warps 2..9: two per TMEM lane quarter, splitting columns
constexpr int EPI_GROUPS = EPI_WARPS / 4;  // warps per lane quarter (take alternate chunks)
constexpr int GEMM_THREADS = 64 + 32 * EPI_WARPS;
// CTA-pair kernel with an A-operand transform (XFORM): the epilogue warps of
// group 1 rewrite A tiles instead, one thread per tile row.
constexpr int XFORM_WARPS = 4;

struct GemmArgs {
  int M, N, K, batch;
  int a_mn, b_mn;  // operand stored MN-major (contiguous along M / N)
  int a3d, b3d;    // tensor map carries a batch coordinate
  int a_chunked, b_chunked;  // MN-major tile loaded by one (32, K, chunk) box
  int tiles_m, tiles_n, splits, kblocks;  // kblocks: K blocks of the whole (reduced) K
  int kblocks_item;                       // K blocks of one batch item
  long long units;
  uint32_t idesc;
  float* C; long long ldc, sc;
  float alpha, beta;
  const float* bias;
  const float* R; long long ldr, sr;
  float* P; long long ldp, sp;
  const float* X; long long ldx, sx;
  int act, grad_act, accumulate, vec_ok;
  int reduce_batch;  // sum the batch into one output (K runs over batch x K)
  int bm;            // rows per output tile: 128 (one CTA) or 256 (a CTA pair)
  int group_m;       // raster: tiles walk N within groups of group_m row tiles
  int epi_tma;       // epilogue moves tiles by TMA (else per-thread global accesses)
  int c3d, p3d, r3d, x3d;  // epilogue tensor maps carry a batch coordinate
  // Dynamic schedule: units are claimed from *sched_next (zero at launch);
  // the last CTA to finish resets it and *sched_done. Null: static schedule
  // (CTA c takes units c, c + grid, c + 2 grid, ...).
  unsigned long long* sched_next;
  unsigned int* sched_done;
  // Softmax fused into the two attention products (attention_forward):
  //  stats_out  score product: each stored 32-column chunk of a row holds
  //             E = exp(v - m_c) (0 where masked), where m_c is the chunk's
  //             maximum, and (m_c, sum of E) goes to
  //             stats[(batch * stats_chunks + chunk) * M + row]
  //  stats_in   P·V product (XFORM kernel): those statistics after
  //             softmax_stats_finalize_kernel, whose .x holds each chunk's
  //             factor exp(m_c - max) / sum; every A tile (one chunk per row)
  //             is scaled by it in shared memory before the tensor cores read
  //             it, which makes it the softmax
  //  stats_chunks 32-column chunks per score row
  //  period     > 0: column c of row m is masked (E = 0) when c > m % period
  float2* stats_out;
  const float2* stats_in;
  int stats_chunks;
  long long period;
};

// Tensor maps of the epilogue operands: 32 x 32 f32 boxes, 128B swizzle.
struct EpiMaps {
  CUtensorMap c, p, r, x;
};

constexpr int EPI_TILE_BYTES = 32 * 32 * 4;  // one staging tile per warp and buffer
constexpr int EPI_NB_MAX = 2;                // staging tiles per epilogue warp, at most

template <int BN, int STAGES, bool SPLIT3>
struct GemmCfg {
  static constexpr int A_BYTES = BM * BK * 4;
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int OPS = SPLIT3 ? 2 : 1;  // hi (+ lo) copies of each operand
  static constexpr int STAGE_BYTES = (A_BYTES + B_BYTES) * OPS;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int CTRL_BYTES = 1024;
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_TILE_BYTES;  // one staging tile per epilogue warp
  static constexpr int SMEM_BYTES = 1024 + CTRL_BYTES + STAGES * STAGE_BYTES + EPI_BYTES;
  static_assert(TMEM_COLS >= 32 && TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0,
                "TMEM allocation must be a power of two in [32, 512]");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN must be a multiple of 32 in [32,256]");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

// Depth of the tile queue through which the producer publishes the units it
// claims under the dynamic schedule.
constexpr int TQ = 4;

template <int STAGES>
struct GemmCtrl {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t epi[EPI_WARPS * EPI_NB_MAX];  // per epilogue warp and staging tile: its TMA loads
  uint64_t qfull[TQ];       // tile queue: entry published (one arrive, the leader's producer)
  uint64_t qempty[TQ];      // tile queue (leader CTA): entry read by every consumer
  long long qunit[TQ];      // the published unit, -1 = no more work
  uint64_t afull[STAGES];   // A-operand transform: this CTA's A tile landed
  uint64_t xready[STAGES];  // A-operand transform (leader): both CTAs' tiles transformed
  uint32_t tmem_base;
  volatile uint32_t abort_flag;
};

__device__ __forceinline__ void decode_unit(const GemmArgs& a, long long u, int& b, int& tm,
                                            int& tn, int& kb0, int& kb1) {
  const long long tiles = static_cast<long long>(a.tiles_m) * a.tiles_n;
  const long long per_split = a.reduce_batch ? tiles : tiles * a.batch;
  const int s = static_cast<int>(u / per_split);
  const long long r = u - static_cast<long long>(s) * per_split;
  b = a.reduce_batch ? 0 : static_cast<int>(r / tiles);
  const long long t = r - static_cast<long long>(b) * tiles;
  const long long group_size = static_cast<long long>(a.group_m) * a.tiles_n;
  const int g = static_cast<int>(t / group_size);
  const int first_m = g * a.group_m;
  const int gm = min(a.tiles_m - first_m, a.group_m);
  const int inner = static_cast<int>(t - static_cast<long long>(g) * group_size);
  tm = first_m + inner % gm;
  tn = inner / gm;
  kb0 = static_cast<int>((static_cast<long long>(s) * a.kblocks) / a.splits);
  kb1 = static_cast<int>((static_cast<long long>(s + 1) * a.kblocks) / a.splits);
}

// ---------------------------------------------------------------- unit schedule
// A persistent CTA (or CTA pair) processes the units of its sequence i = 0,
// 1, 2, ... Static: unit first + i * stride. Dynamic: the leader CTA's
// producer claims each unit from a global counter and publishes it through
// the tile queue (qunit/qfull, and the partner CTA's copy for a pair); every
// other role takes it from there. A CTA that starts late, because other
// kernels occupy SMs, then simply claims fewer units instead of delaying the
// whole grid with a fixed share. Units are claimed in increasing order, so
// the tiles in flight stay a contiguous window of the raster, as with the
// static order.

__device__ __forceinline__ long long static_unit(const GemmArgs& a, long long first,
                                                 long long stride, int i) {
  const long long u = first + static_cast<long long>(i) * stride;
  return u < a.units ? u : -1;
}

// Producer of the leader CTA: claims the i-th unit and publishes it to this
// CTA's queue and, for a pair, to the partner's. False on a wait expiry.
template <int STAGES, bool PAIR>
__device__ __forceinline__ bool queue_publish(GemmCtrl<STAGES>* ctrl, const GemmArgs& a, int i,
                                              long long* u_out) {
  const int slot = i % TQ;
  const uint32_t par = static_cast<uint32_t>(i / TQ) & 1u;
  if (!mbar_wait(&ctrl->qempty[slot], par ^ 1u, DEVERR_GEMM_QUEUE)) return false;
  long long u = static_cast<long long>(atomicAdd(a.sched_next, 1ull));
  if (u >= a.units) u = -1;
  ctrl->qunit[slot] = u;
  if (PAIR) {
    st_cluster_s64(map_to_rank(&ctrl->qunit[slot], 1), u);
    mbar_arrive_remote(map_to_rank(&ctrl->qfull[slot], 1));
  }
  mbar_arrive(&ctrl->qfull[slot]);
  *u_out = u;
  return true;
}

// Any other role: reads the i-th published unit. `release` (one thread per
// consumer) frees the entry on the leader CTA's qempty (cluster address of
// qempty[0]; entries are 8 bytes apart). False on a wait expiry.
template <int STAGES>
__device__ __forceinline__ bool queue_take(GemmCtrl<STAGES>* ctrl, int i, uint32_t qempty0,
                                           bool release, long long* u_out) {
  const int slot = i % TQ;
  const uint32_t par = static_cast<uint32_t>(i / TQ) & 1u;
  if (!mbar_wait_cluster(&ctrl->qfull[slot], par, DEVERR_GEMM_QUEUE)) return false;
  *u_out = ctrl->qunit[slot];
  if (release) mbar_arrive_remote(qempty0 + 8u * static_cast<uint32_t>(slot));
  return true;
}

// The i-th unit if it is already published (-2 if not yet), without taking
// it: the epilogue's look-ahead for its next tile's first input.
template <int STAGES>
__device__ __forceinline__ long long queue_peek(GemmCtrl<STAGES>* ctrl, int i) {
  const int slot = i % TQ;
  const uint32_t par = static_cast<uint32_t>(i / TQ) & 1u;
  if (!mbar_test_wait_cluster(&ctrl->qfull[slot], par)) return -2;
  return ctrl->qunit[slot];
}

// Programmatic dependent launch (the persistent kernels are launched with
// programmatic stream serialisation): the prologue (barriers, TMEM,
// tensor-map prefetch, cluster sync) runs while the previous kernel of the
// stream finishes; every thread then waits here for that kernel's completion
// and memory before any global access, the schedule counter included.
// Letting dependents launch at this point only pre-stages them: they wait
// for this grid the same way.
__device__ __forceinline__ void pdl_after_prologue() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Dynamic schedule only: the last CTA of the grid to finish resets the
// counter for the next launch on this slot (every CTA reaches this point,
// aborted ones included, after its producer stopped claiming).
__device__ __forceinline__ void schedule_release(const GemmArgs& a) {
  if (a.sched_next == nullptr || threadIdx.x != 0) return;
  __threadfence();
  if (atomicAdd(a.sched_done, 1u) == gridDim.x - 1) {
    *a.sched_next = 0ull;
    *a.sched_done = 0u;
    __threadfence();
  }
}

__device__ __forceinline__ void epilogue_chunk(const GemmArgs& a, int b, int m, int n0,
                                               float (&v)[32]) {
  float* crow = a.C + b * a.sc + static_cast<long long>(m) * a.ldc;
  const float* rrow = a.R ? a.R + b * a.sr + static_cast<long long>(m) * a.ldr : nullptr;
  float* prow = a.P ? a.P + b * a.sp + static_cast<long long>(m) * a.ldp : nullptr;
  const float* xrow = a.X ? a.X + b * a.sx + static_cast<long long>(m) * a.ldx : nullptr;
  const bool full = a.vec_ok && (n0 + 32 <= a.N);
  if (full) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      float4 acc = make_float4(v[j] * a.alpha, v[j + 1] * a.alpha, v[j + 2] * a.alpha,
                               v[j + 3] * a.alpha);
      if (a.beta != 0.0f) {
        const float4 c = *reinterpret_cast<const float4*>(crow + n0 + j);
        acc.x += a.beta * c.x; acc.y += a.beta * c.y; acc.z += a.beta * c.z; acc.w += a.beta * c.w;
      }
      if (a.bias) {
        const float4 bb = *reinterpret_cast<const float4*>(a.bias + n0 + j);
        acc.x += bb.x; acc.y += bb.y; acc.z += bb.z; acc.w += bb.w;
      }
      if (rrow) {
        const float4 r = *reinterpret_cast<const float4*>(rrow + n0 + j);
        acc.x += r.x; acc.y += r.y; acc.z += r.z; acc.w += r.w;
      }
      if (prow) *reinterpret_cast<float4*>(prow + n0 + j) = acc;
      if (xrow) {
        const float4 x = *reinterpret_cast<const float4*>(xrow + n0 + j);
        acc.x *= act_derivative_fast(a.grad_act, x.x);
        acc.y *= act_derivative_fast(a.grad_act, x.y);
        acc.z *= act_derivative_fast(a.grad_act, x.z);
        acc.w *= act_derivative_fast(a.grad_act, x.w);
      }
      if (a.act != OXF_ACT_IDENTITY) {
        acc.x = act_forward_fast(a.act, acc.x); acc.y = act_forward_fast(a.act, acc.y);
        acc.z = act_forward_fast(a.act, acc.z); acc.w = act_forward_fast(a.act, acc.w);
      }
      if (a.accumulate) atomicAdd(reinterpret_cast<float4*>(crow + n0 + j), acc);
      else *reinterpret_cast<float4*>(crow + n0 + j) = acc;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = n0 + j;
      if (n >= a.N) continue;
      float acc = v[j] * a.alpha;
      if (a.beta != 0.0f) acc += a.beta * crow[n];
      if (a.bias) acc += a.bias[n];
      if (rrow) acc += rrow[n];
      if (prow) prow[n] = acc;
      if (xrow) acc *= act_derivative_fast(a.grad_act, xrow[n]);
      acc = act_forward_fast(a.act, acc);
      if (a.accumulate) atomicAdd(crow + n, acc);
      else crow[n] = acc;
    }
  }
}

// ---------------------------------------------------------------- fused softmax
// The score product's epilogue, per 32-column chunk of row m (values v, the
// final scaled logits): columns past the matrix or the causal limit become
// 0, the others exp(v - m_c) with m_c the chunk's maximum; (m_c, sum) is
// stored in the chunk-major statistics array, so the 32 lanes (rows) of a
// warp write 256 contiguous bytes.
__device__ __forceinline__ void softmax_chunk_exp(const GemmArgs& a, int b, int m, int n0,
                                                  float (&v)[32]) {
  long long lim = a.N;
  if (a.period && m % a.period + 1 < lim) lim = m % a.period + 1;
  float cm = -INFINITY;
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (n0 + j < lim) cm = fmaxf(cm, v[j]);
  float l = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    v[j] = n0 + j < lim ? __expf(v[j] - cm) : 0.0f;  // cm finite whenever a column counts
    l += v[j];
  }
  if (m < a.M)
    a.stats_out[(static_cast<long long>(b) * a.stats_chunks + (n0 >> 5)) * a.M + m] =
        make_float2(cm, l);
}

// Scales row r (0..127) of a K-major 128 x 32 A tile (128B-swizzle layout,
// 128 bytes per row) by f in place. Each lane starts at 16-byte unit r & 7,
// so the 32 lanes of a warp spread over all banks.
__device__ __forceinline__ void scale_tile_row(uint8_t* tile, int r, float f) {
  uint8_t* row = tile + r * 128;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4* q = reinterpret_cast<float4*>(row + (((i + r) & 7) << 4));
    float4 x = *q;
    x.x *= f; x.y *= f; x.z *= f; x.w *= f;
    *q = x;
  }
}

// ---------------------------------------------------------------- TMA epilogue
// Each epilogue warp owns one staging tile of 32 rows x 128 B in the TMA
// 128B-swizzle layout: 16-byte unit j of row r sits at unit j ^ (r & 7), so
// the 32 lanes (lane = row) touching unit j of their rows hit every bank
// once per 8 lanes. A lane only ever reads and writes its own row; the TMA
// engine moves whole tiles between the buffers and global memory.
__device__ __forceinline__ float4* stage_unit(uint8_t* buf, int row, int j) {
  return reinterpret_cast<float4*>(buf + row * 128 + ((j ^ (row & 7)) << 4));
}

__device__ __forceinline__ void stage_write_row(uint8_t* buf, int lane, const float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *stage_unit(buf, lane, j) = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

__device__ __forceinline__ void stage_read_row(uint8_t* buf, int lane, float (&t)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 q = *stage_unit(buf, lane, j);
    t[4 * j] = q.x; t[4 * j + 1] = q.y; t[4 * j + 2] = q.z; t[4 * j + 3] = q.w;
  }
}

// Starts loading the 32 x 32 tile at (column n0, row m0[, batch b]) into
// buf. Prior generic accesses of buf by the warp are ordered before the
// asynchronous write.
__device__ __forceinline__ void epi_issue(uint8_t* buf, const CUtensorMap* map, int is3d,
                                          uint64_t* bar, int n0, int m0, int b, int lane) {
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    mbar_arrive_expect_tx(bar, EPI_TILE_BYTES);
    const uint64_t pol = make_l2_policy(L2_EVICT_FIRST);  // read once
    if (is3d) tma_load_3d(buf, map, bar, n0, m0, b, pol);
    else tma_load_2d(buf, map, bar, n0, m0, pol);
  }
}

// Waits (bounded) for the load issued last on bar.
__device__ __forceinline__ bool epi_wait(uint64_t* bar, uint32_t& phase) {
  const bool ok = mbar_wait(bar, phase, DEVERR_GEMM_EPI_LOAD);
  phase ^= 1u;
  return ok;
}

// Stores (or atomically adds) the staged tile; the lanes' row writes are
// made visible to the TMA engine first.
__device__ __forceinline__ void epi_store(uint8_t* buf, const CUtensorMap* map, int is3d, int n0,
                                          int m0, int b, int lane, bool reduce) {
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (reduce) {
      if (is3d) tma_reduce_add_3d(map, buf, n0, m0, b);
      else tma_reduce_add_2d(map, buf, n0, m0);
    } else {
      if (is3d) tma_store_3d(map, buf, n0, m0, b);
      else tma_store_2d(map, buf, n0, m0);
    }
    bulk_commit_group();
  }
}

// Every store this warp issued has finished reading its staging buffer.
__device__ __forceinline__ void epi_buffers_free(int lane) {
  if (lane == 0) bulk_wait_group_read0();
  __syncwarp();
}

// The epilogue input read first into buffer 0, before any store of the
// chunk: C (when beta != 0), else the residual, else aux when there is no
// pre-activation output. That one can be loaded ahead, while the warp is
// still busy with its previous chunk.
__device__ __forceinline__ const CUtensorMap* epi_first_input(const GemmArgs& a,
                                                              const EpiMaps& em, int& is3d) {
  if (a.beta != 0.0f) { is3d = a.c3d; return &em.c; }
  if (a.R) { is3d = a.r3d; return &em.r; }
  if (a.X && !a.P) { is3d = a.x3d; return &em.x; }
  return nullptr;
}

// The staging tiles of one epilogue warp, used round-robin: NB tiles of
// 32 x 32 f32 in the TMA 128B-swizzle layout, each with an mbarrier for the
// TMA loads into it. Every load into a tile and every store out of one takes
// the next tile of the ring, and a tile is written again only after the
// stores issued from it have finished reading it. With one tile, each chunk
// waits for the previous chunk's store to read the tile; with two, staging a
// chunk overlaps that read.
template <int NB>
struct EpiRing {
  uint8_t* tiles;
  uint64_t* bars;
  uint32_t phases;  // bit k: parity of the next wait on bars[k]
  int next;         // the tile the next acquire returns
  int stores;       // bulk store groups committed so far
  // group number of the last store out of tile 0 / 1, -1 if none pending
  // (two named fields, not an array, so they stay in registers)
  int last0, last1;
  __device__ __forceinline__ uint8_t* tile(int k) const { return tiles + k * EPI_TILE_BYTES; }
  __device__ __forceinline__ int last(int k) const { return k == 0 ? last0 : last1; }
  __device__ __forceinline__ void set_last(int k, int g) {
    if (k == 0) last0 = g;
    else last1 = g;
  }
};

template <int NB>
__device__ __forceinline__ void ring_init(EpiRing<NB>& r, uint8_t* tiles, uint64_t* bars) {
  r.tiles = tiles;
  r.bars = bars;
  r.phases = 0;
  r.next = 0;
  r.stores = 0;
  r.last0 = -1;
  r.last1 = -1;
}

// The next tile of the ring, once the store last issued from it (if any)
// has read it. Stores commit one group each, in order, and a tile is reused
// after at most NB - 1 other uses, so at most NB - 1 later groups may stay
// in flight.
template <int NB>
__device__ __forceinline__ int ring_acquire(EpiRing<NB>& r, int lane) {
  static_assert(NB >= 1 && NB <= EPI_NB_MAX, "staging ring size");
  const int k = r.next;
  r.next = k + 1 == NB ? 0 : k + 1;
  if (r.last(k) >= 0) {
    const int later = r.stores - 1 - r.last(k);
    if (lane == 0) {
      if (NB > 1 && later >= 1) bulk_wait_group_read1();
      else bulk_wait_group_read0();
    }
    __syncwarp();
    r.set_last(k, -1);
  }
  return k;
}

template <int NB>
__device__ __forceinline__ void ring_store(EpiRing<NB>& r, int k, const CUtensorMap* map, int is3d,
                                           int n0, int m0, int b, int lane, bool reduce) {
  epi_store(r.tile(k), map, is3d, n0, m0, b, lane, reduce);
  r.set_last(k, r.stores++);
}

// Waits (bounded) for the load issued last into tile k.
template <int NB>
__device__ __forceinline__ bool ring_wait(EpiRing<NB>& r, int k) {
  const bool ok = mbar_wait(&r.bars[k], (r.phases >> k) & 1u, DEVERR_GEMM_EPI_LOAD);
  r.phases ^= 1u << k;
  return ok;
}

// Issues the first input (epi_first_input) of a later chunk into the next
// tile of the ring. Returns that tile, or -1 if nothing was loaded.
template <int NB>
__device__ __forceinline__ int epi_prefetch(const GemmArgs& a, const EpiMaps& em, EpiRing<NB>& rg,
                                            int b, int m0, int n0, int lane) {
  int is3d = 0;
  const CUtensorMap* map = epi_first_input(a, em, is3d);
  if (!map || m0 >= a.M || n0 >= a.N) return -1;
  const int k = ring_acquire(rg, lane);
  epi_issue(rg.tile(k), map, is3d, &rg.bars[k], n0, m0, b, lane);
  return k;
}

// The fused epilogue of one warp's 32 x 32 chunk (rows m0.., columns n0..),
// in the same arithmetic order as epilogue_chunk, through the warp's staging
// ring. `pf`: the tile into which the first input (epi_first_input) is
// already being loaded, or -1. Returns false if a staged load timed out.
template <int NB>
__device__ __forceinline__ bool epilogue_chunk_tma(const GemmArgs& a, const EpiMaps& em, int b,
                                                   int m0, int n0, float (&v)[32],
                                                   EpiRing<NB>& rg, int lane, int pf) {
  if (m0 >= a.M) return true;  // rows past the matrix (last tile): nothing to move
  if (a.alpha != 1.0f) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] *= a.alpha;
  }
  float t[32];
  // Reads one input tile into t: the prefetched one, else a fresh load.
  auto input = [&](const CUtensorMap* map, int is3d) -> bool {
    int k = pf;
    if (k < 0) {
      k = ring_acquire(rg, lane);
      epi_issue(rg.tile(k), map, is3d, &rg.bars[k], n0, m0, b, lane);
    }
    pf = -1;
    if (!ring_wait(rg, k)) return false;
    stage_read_row(rg.tile(k), lane, t);
    return true;
  };
  if (a.beta != 0.0f) {
    if (!input(&em.c, a.c3d)) return false;
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] += a.beta * t[j];
  }
  if (a.bias) {
    if (a.vec_ok && n0 + 32 <= a.N) {
      const float4* bp = reinterpret_cast<const float4*>(a.bias + n0);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 q = __ldg(bp + j);
        t[4 * j] = q.x; t[4 * j + 1] = q.y; t[4 * j + 2] = q.z; t[4 * j + 3] = q.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) t[j] = n0 + j < a.N ? __ldg(a.bias + n0 + j) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] += t[j];
  }
  if (a.R) {
    if (!input(&em.r, a.r3d)) return false;
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] += t[j];
  }
  if (a.P) {
    const int k = ring_acquire(rg, lane);
    stage_write_row(rg.tile(k), lane, v);
    ring_store(rg, k, &em.p, a.p3d, n0, m0, b, lane, false);
  }
  if (a.X) {  // aux is prefetched only when there is no pre-activation store
    if (!input(&em.x, a.x3d)) return false;
    act_grad_chunk(a.grad_act, v, t);
  }
  act_forward_chunk(a.act, v);
  if (a.stats_out) softmax_chunk_exp(a, b, m0 + lane, n0, v);
  const int k = ring_acquire(rg, lane);
  stage_write_row(rg.tile(k), lane, v);
  ring_store(rg, k, &em.c, a.c3d, n0, m0, b, lane, a.accumulate != 0);
  return true;
}

// The chunk an epilogue warp takes after chunk c of unit u: the next
// alternate column chunk of the same tile, else its first chunk of the next
// unit its CTA (pair) owns. Rows of a unit start at tm * a.bm + row_off.
template <int BN>
__device__ __forceinline__ bool epi_next_chunk(const GemmArgs& a, long long u2, int c, int group,
                                               int row_off, int b, int tn, int m0, int& nb,
                                               int& nm0, int& nn0, int cstep = EPI_GROUPS) {
  const int c2 = c + cstep;
  if (c2 < BN / 32 && tn * BN + c2 * 32 < a.N) {
    nb = b;
    nm0 = m0;
    nn0 = tn * BN + c2 * 32;
    return true;
  }
  if (u2 < 0 || u2 >= a.units) return false;  // no next unit, or not yet known
  int tm2, tn2, kb0, kb1;
  decode_unit(a, u2, nb, tm2, tn2, kb0, kb1);
  nm0 = tm2 * a.bm + row_off;
  nn0 = tn2 * BN + group * 32;
  return nn0 < a.N;
}

template <int BN, int STAGES, bool SPLIT3>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tf32_tcgen05(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmA_lo,
                      const __grid_constant__ CUtensorMap tmB_lo,
                      const __grid_constant__ EpiMaps em, const GemmArgs args) {
  using Cfg = GemmCfg<BN, STAGES, SPLIT3>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  auto* ctrl = reinterpret_cast<GemmCtrl<STAGES>*>(base);
  uint8_t* ring = base + Cfg::CTRL_BYTES;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&ctrl->full[s], 1);
      mbar_init(&ctrl->empty[s], 1);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctrl->tfull[i], 1);
      mbar_init(&ctrl->tempty[i], 32 * EPI_WARPS);
    }
#pragma unroll
    for (int w = 0; w < EPI_WARPS * EPI_NB_MAX; ++w) mbar_init(&ctrl->epi[w], 1);
#pragma unroll
    for (int q = 0; q < TQ; ++q) {
      mbar_init(&ctrl->qfull[q], 1);                // the producer's publish
      mbar_init(&ctrl->qempty[q], 1 + EPI_WARPS);  // the MMA issuer and every epilogue warp
    }
    ctrl->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (SPLIT3) {
      tma_prefetch_desc(&tmA_lo);
      tma_prefetch_desc(&tmB_lo);
    }
  }
  if (warp == 1) {
    tmem_alloc(&ctrl->tmem_base, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_after_prologue();
  const uint32_t tmem_base = ctrl->tmem_base;
  const bool dyn = args.sched_next != nullptr;
  const uint32_t qempty0 = map_to_rank(&ctrl->qempty[0], 0);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      long long fills = 0;
      const uint64_t pol_a = make_l2_policy(L2_NORMAL), pol_b = pol_a;
      for (int i = 0; !ctrl->abort_flag; ++i) {
        long long u;
        if (dyn) {
          if (!queue_publish<STAGES, false>(ctrl, args, i, &u)) {
            ctrl->abort_flag = 1;
            break;
          }
        } else {
          u = static_unit(args, blockIdx.x, gridDim.x, i);
        }
        if (u < 0) break;
        int b, tm, tn, kb0, kb1;
        decode_unit(args, u, b, tm, tn, kb0, kb1);
        // Batch-reduce GEMMs walk K over (batch item, k-block) pairs; the
        // pair advances incrementally (no division in the per-block loop).
        int bk = args.reduce_batch ? kb0 / args.kblocks_item : b;
        int kin = args.reduce_batch ? kb0 - bk * args.kblocks_item : kb0;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&ctrl->empty[stage], phase ^ 1u, DEVERR_GEMM_WAIT_EMPTY)) {
            ctrl->abort_flag = 1;
            break;
          }
          uint8_t* slot = ring + stage * Cfg::STAGE_BYTES;
          mbar_arrive_expect_tx(&ctrl->full[stage], Cfg::STAGE_BYTES);
          const int k0 = kin * BK, item = bk;
          if (++kin == args.kblocks_item && args.reduce_batch) {
            kin = 0;
            ++bk;
          }
          load_operand<BM>(slot, &tmA, &ctrl->full[stage], args.a_mn, args.a3d, args.a_chunked,
                           tm * BM, k0, item, pol_a);
          load_operand<BN>(slot + Cfg::A_BYTES, &tmB, &ctrl->full[stage], args.b_mn, args.b3d,
                           args.b_chunked, tn * BN, k0, item, pol_b);
          if (SPLIT3) {
            uint8_t* lo = slot + Cfg::A_BYTES + Cfg::B_BYTES;
            load_operand<BM>(lo, &tmA_lo, &ctrl->full[stage], args.a_mn, args.a3d,
                             args.a_chunked, tm * BM, k0, item, pol_a);
            load_operand<BN>(lo + Cfg::A_BYTES, &tmB_lo, &ctrl->full[stage], args.b_mn,
                             args.b3d, args.b_chunked, tn * BN, k0, item, pol_b);
          }
          ++fills;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Never leave the CTA with bulk copies still landing in its shared
      // memory: wait for the most recent fill of every slot.
      const long long first = fills > STAGES ? fills - STAGES : 0;
      for (long long j = first; j < fills; ++j)
        mbar_wait(&ctrl->full[j % STAGES], static_cast<uint32_t>((j / STAGES) & 1),
                  DEVERR_GEMM_DRAIN);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      // Descriptors of stage 0, K slice 0; every other (stage, slice) is an
      // address offset from these.
      const uint64_t a_desc0 = operand_desc(smem_u32(ring), args.a_mn, 0);
      const uint64_t b_desc0 = operand_desc(smem_u32(ring) + Cfg::A_BYTES, args.b_mn, 0);
      const uint32_t a_step = operand_kstep(args.a_mn), b_step = operand_kstep(args.b_mn);
      for (int local = 0; !ctrl->abort_flag; ++local) {
        long long u;
        if (dyn) {
          if (!queue_take(ctrl, local, qempty0, true, &u)) {
            ctrl->abort_flag = 1;
            break;
          }
        } else {
          u = static_unit(args, blockIdx.x, gridDim.x, local);
        }
        if (u < 0) break;
        int b, tm, tn, kb0, kb1;
        decode_unit(args, u, b, tm, tn, kb0, kb1);
        const int acc_slot = local & 1;
        const uint32_t use = static_cast<uint32_t>(local >> 1);
        if (!mbar_wait(&ctrl->tempty[acc_slot], (use & 1u) ^ 1u, DEVERR_GEMM_WAIT_TMEM_EMPTY)) {
          ctrl->abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc_slot * BN);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&ctrl->full[stage], phase, DEVERR_GEMM_WAIT_FULL)) {
            ctrl->abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t off = stage * Cfg::STAGE_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            const uint64_t da = desc_advance(a_desc0, off + kk * a_step);
            const uint64_t db = desc_advance(b_desc0, off + kk * b_step);
            const uint32_t accumulate = (kb > kb0 || kk > 0) ? 1u : 0u;
            if (SPLIT3) {
              const uint32_t lo = Cfg::A_BYTES + Cfg::B_BYTES;
              const uint64_t da_lo = desc_advance(a_desc0, off + lo + kk * a_step);
              const uint64_t db_lo = desc_advance(b_desc0, off + lo + kk * b_step);
              umma_tf32(d_tmem, da_lo, db, args.idesc, accumulate);
              umma_tf32(d_tmem, da, db_lo, args.idesc, 1u);
              umma_tf32(d_tmem, da, db, args.idesc, 1u);
            } else {
              umma_tf32(d_tmem, da, db, args.idesc, accumulate);
            }
          }
          umma_commit(&ctrl->empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&ctrl->tfull[acc_slot]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int group = (warp - 2) / 4;  // which alternate 32-column chunks it takes
    const int row_local = quarter * 32 + lane;
    uint8_t* bufs = ring + STAGES * Cfg::STAGE_BYTES + (warp - 2) * EPI_TILE_BYTES;
    EpiRing<1> rg;
    ring_init(rg, bufs, &ctrl->epi[(warp - 2) * EPI_NB_MAX]);
    bool ok = true;
    int pf = -1;  // the tile the next chunk's first input is being loaded into
    // only an epilogue that reads an input tile first looks ahead to prefetch it
    int la3d = 0;
    const bool lookahead = args.epi_tma && epi_first_input(args, em, la3d) != nullptr;
    for (int local = 0; ok; ++local) {
      long long u;
      if (dyn) {
        if (!queue_take(ctrl, local, qempty0, false, &u)) {
          ctrl->abort_flag = 1;
          break;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(qempty0 + 8u * static_cast<uint32_t>(local % TQ));
      } else {
        u = static_unit(args, blockIdx.x, gridDim.x, local);
      }
      if (u < 0) break;
      int b, tm, tn, kb0, kb1;
      decode_unit(args, u, b, tm, tn, kb0, kb1);
      const int acc_slot = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      if (!mbar_wait(&ctrl->tfull[acc_slot], use & 1u, DEVERR_GEMM_WAIT_TMEM_FULL)) {
        ctrl->abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int m = tm * BM + row_local;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc_slot * BN);
#pragma unroll 1
      for (int c = group; c < BN / 32; c += EPI_GROUPS) {
        const int n0 = tn * BN + c * 32;
        if (n0 >= args.N) break;  // uniform across the warp
        float v[32];
        tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(c * 32), v);
        if (args.epi_tma) {
          const int m0 = tm * BM + quarter * 32;
          if (!epilogue_chunk_tma(args, em, b, m0, n0, v, rg, lane, pf)) {
            ctrl->abort_flag = 1;
            ok = false;
            pf = -1;
            break;
          }
          pf = -1;
          if (lookahead) {
            int nb, nm0, nn0;
            long long u2 = -2;  // the next unit, needed after the tile's last chunk only
            if (c + EPI_GROUPS >= BN / 32 || tn * BN + (c + EPI_GROUPS) * 32 >= args.N) {
              if (dyn) {
                if (lane == 0) u2 = queue_peek(ctrl, local + 1);
                u2 = __shfl_sync(0xffffffffu, u2, 0);
              } else {
                u2 = static_unit(args, blockIdx.x, gridDim.x, local + 1);
              }
            }
            if (epi_next_chunk<BN>(args, u2, c, group, quarter * 32, b, tn, m0, nb, nm0, nn0))
              pf = epi_prefetch(args, em, rg, nb, nm0, nn0, lane);
          }
        } else if (m < args.M) {
          epilogue_chunk(args, b, m, n0, v);
        }
      }
      tc_fence_before();
      mbar_arrive(&ctrl->tempty[acc_slot]);
    }
    if (pf >= 0) ring_wait(rg, pf);  // an abandoned prefetch must land before exit
    if (lane == 0) bulk_wait_group0();  // no store may outlive the CTA's shared memory
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
  schedule_release(args);
}

// ---------------------------------------------------------------- CTA-pair kernel
// The same pipeline on a cluster of two CTAs computing a 256 x BN tile with
// tcgen05.mma.cta_group::2: each CTA loads its 128 rows of A and its BN/2
// columns of B (so each SM moves 32 KB instead of 48 KB per K block at
// BN = 256, leaving room for 6 stages), both halves complete on the leader
// CTA's full barrier, the leader alone issues the MMAs and multicast-commits
// to both CTAs' barriers, and each CTA's epilogue drains its own 128 TMEM
// lanes and releases the accumulator to the leader with a remote arrive.
template <int BN, int STAGES, bool SPLIT3, int NB, bool XFORM = false>
struct GemmPairCfg {
  static constexpr int A_BYTES = BM * BK * 4;
  static constexpr int B_BYTES = (BN / 2) * BK * 4;
  static constexpr int OPS = SPLIT3 ? 2 : 1;  // hi (+ lo) copies of each operand
  static constexpr int STAGE_BYTES = (A_BYTES + B_BYTES) * OPS;
  // One MMA covers N = 256 (128 columns from each CTA's half of B). A wider
  // tile issues NSUB of them per K step into consecutive 256-column TMEM
  // ranges, all reading the same A: fewer operand bytes per flop.
  static constexpr int MMA_N = 256;
  static constexpr int NSUB = BN / MMA_N;
  static constexpr int B_SUB_BYTES = 128 * BK * 4;  // one MMA's 128 columns in one CTA
  // Accumulators are double-buffered (the epilogue drains one while the MMA
  // fills the other) unless one tile already fills TMEM's 512 columns.
  static constexpr int ACC_BUFS = 2 * BN <= 512 ? 2 : 1;
  static constexpr int TMEM_COLS = ACC_BUFS * BN;
  static constexpr int CTRL_BYTES = 1024;
  // NB staging tiles per epilogue warp (transform warps stage nothing)
  static constexpr int EPI_BYTES = (EPI_WARPS - (XFORM ? XFORM_WARPS : 0)) * EPI_TILE_BYTES * NB;
  static constexpr int SMEM_BYTES = 1024 + CTRL_BYTES + STAGES * STAGE_BYTES + EPI_BYTES;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(BN % MMA_N == 0 && TMEM_COLS <= 512, "tile shape");
  static_assert(NB >= 1 && NB <= EPI_NB_MAX, "staging tiles per warp");
};

// TMEM column of a pair tile's 32-column output chunk c. CTA r of the pair
// loads tile columns [r*BN/2, (r+1)*BN/2) as 128-column sub-tiles, and MMA h
// reads sub-tile h of both CTAs, so accumulator h (columns h*256..) holds CTA
// 0's sub-tile h, then CTA 1's. For BN = 256 this is the identity.
template <int BN>
__device__ __forceinline__ uint32_t pair_chunk_tmem_col(int c) {
  const int x = c * 32;
  return static_cast<uint32_t>(((x % (BN / 2)) / 128) * 256 + (x / (BN / 2)) * 128 + x % 128);
}

template <int ROWS>
__device__ __forceinline__ void load_operand_pair(uint8_t* dst, const CUtensorMap* map,
                                                  uint32_t bar, int mn_major, int is3d,
                                                  int chunked, int row0, int k0, int b,
                                                  uint64_t pol) {
  if (!mn_major) {
    if (is3d) tma_load_3d_pair(dst, map, bar, k0, row0, b, pol);
    else tma_load_2d_pair(dst, map, bar, k0, row0, pol);
  } else if (chunked) {
    if (is3d) tma_load_4d_pair(dst, map, bar, 0, k0, row0 / 32, b, pol);
    else tma_load_3d_pair(dst, map, bar, 0, k0, row0 / 32, pol);
  } else {
#pragma unroll
    for (int c = 0; c < ROWS / 32; ++c) {
      if (is3d) tma_load_3d_pair(dst + c * 4096, map, bar, row0 + 32 * c, k0, b, pol);
      else tma_load_2d_pair(dst + c * 4096, map, bar, row0 + 32 * c, k0, pol);
    }
  }
}

template <int BN, int STAGES, bool SPLIT3, int NB, bool XFORM>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GEMM_THREADS, 1)
    gemm_tf32_tcgen05_pair(const __grid_constant__ CUtensorMap tmA,
                           const __grid_constant__ CUtensorMap tmB,
                           const __grid_constant__ CUtensorMap tmA_lo,
                           const __grid_constant__ CUtensorMap tmB_lo,
                           const __grid_constant__ EpiMaps em, const GemmArgs args) {
  using Cfg = GemmPairCfg<BN, STAGES, SPLIT3, NB, XFORM>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  auto* ctrl = reinterpret_cast<GemmCtrl<STAGES>*>(base);
  uint8_t* ring = base + Cfg::CTRL_BYTES;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&ctrl->full[s], 1);   // used in the leader: its producer's arrive + both halves' bytes
      mbar_init(&ctrl->empty[s], 1);  // the leader's multicast commit
      if (XFORM) {
        mbar_init(&ctrl->afull[s], 1);          // this CTA's producer's arrive + its A bytes
        mbar_init(&ctrl->xready[s], 2 * XFORM_WARPS);  // leader: every transform warp of the pair
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctrl->tfull[i], 1);  // the leader's multicast commit
      // leader: one arrive per epilogue warp of the pair
      mbar_init(&ctrl->tempty[i], 2 * (EPI_WARPS - (XFORM ? XFORM_WARPS : 0)));
    }
#pragma unroll
    for (int w = 0; w < EPI_WARPS * EPI_NB_MAX; ++w) mbar_init(&ctrl->epi[w], 1);
#pragma unroll
    for (int q = 0; q < TQ; ++q) {
      mbar_init(&ctrl->qfull[q], 1);  // the leader producer's publish (local or remote)
      // leader: its MMA issuer, the partner's producer and both CTAs' epilogue warps
      mbar_init(&ctrl->qempty[q], 2 + 2 * EPI_WARPS);
    }
    ctrl->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (SPLIT3) {
      tma_prefetch_desc(&tmA_lo);
      tma_prefetch_desc(&tmB_lo);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(&ctrl->tmem_base, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  pdl_after_prologue();
  const uint32_t tmem_base = ctrl->tmem_base;
  const uint32_t full0 = map_to_rank(&ctrl->full[0], 0);
  const uint32_t tempty0 = map_to_rank(&ctrl->tempty[0], 0);
  const long long cluster_id = blockIdx.x >> 1;
  const long long nclusters = gridDim.x >> 1;
  const bool dyn = args.sched_next != nullptr;
  const uint32_t qempty0 = map_to_rank(&ctrl->qempty[0], 0);

  if (warp == 0) {
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      long long fills = 0;
      const uint64_t pol_a = make_l2_policy(L2_NORMAL), pol_b = pol_a;
      for (int i = 0; !ctrl->abort_flag; ++i) {
        long long u;
        if (dyn) {
          // the leader claims and publishes; the partner's producer follows
          const bool got = leader ? queue_publish<STAGES, true>(ctrl, args, i, &u)
                                  : queue_take(ctrl, i, qempty0, true, &u);
          if (!got) {
            ctrl->abort_flag = 1;
            break;
          }
        } else {
          u = static_unit(args, cluster_id, nclusters, i);
        }
        if (u < 0) break;
        int b, tm, tn, kb0, kb1;
        decode_unit(args, u, b, tm, tn, kb0, kb1);
        int bk = args.reduce_batch ? kb0 / args.kblocks_item : b;  // as in the single-CTA kernel
        int kin = args.reduce_batch ? kb0 - bk * args.kblocks_item : kb0;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&ctrl->empty[stage], phase ^ 1u, DEVERR_GEMM_WAIT_EMPTY)) {
            ctrl->abort_flag = 1;
            break;
          }
          if (leader)
            mbar_arrive_expect_tx(&ctrl->full[stage],
                                  XFORM ? 2 * Cfg::B_BYTES : 2 * Cfg::STAGE_BYTES);
          uint8_t* slot = ring + stage * Cfg::STAGE_BYTES;
          const uint32_t bar = full0 + 8u * stage;
          const int k0 = kin * BK, item = bk;
          if (++kin == args.kblocks_item && args.reduce_batch) {
            kin = 0;
            ++bk;
          }
          const int arow = tm * 2 * BM + static_cast<int>(rank) * BM;
          const int brow = tn * BN + static_cast<int>(rank) * (BN / 2);
          if (XFORM) {
            // A lands in this CTA alone, for its transform warps to rewrite
            // before the leader's MMAs read it
            mbar_arrive_expect_tx(&ctrl->afull[stage], Cfg::A_BYTES);
            load_operand<BM>(slot, &tmA, &ctrl->afull[stage], args.a_mn, args.a3d, args.a_chunked,
                             arow, k0, item, pol_a);
          } else {
            load_operand_pair<BM>(slot, &tmA, bar, args.a_mn, args.a3d, args.a_chunked, arow, k0,
                                  item, pol_a);
          }
          load_operand_pair<BN / 2>(slot + Cfg::A_BYTES, &tmB, bar, args.b_mn, args.b3d,
                                    args.b_chunked, brow, k0, item, pol_b);
          if (SPLIT3) {
            uint8_t* lo = slot + Cfg::A_BYTES + Cfg::B_BYTES;
            load_operand_pair<BM>(lo, &tmA_lo, bar, args.a_mn, args.a3d, args.a_chunked, arow,
                                  k0, item, pol_a);
            load_operand_pair<BN / 2>(lo + Cfg::A_BYTES, &tmB_lo, bar, args.b_mn, args.b3d,
                                      args.b_chunked, brow, k0, item, pol_b);
          }
          ++fills;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // The leader's full barriers count both halves: once they complete,
      // no copy is still landing in either CTA.
      if (leader) {
        const long long first = fills > STAGES ? fills - STAGES : 0;
        for (long long j = first; j < fills; ++j)
          mbar_wait(&ctrl->full[j % STAGES], static_cast<uint32_t>((j / STAGES) & 1),
                    DEVERR_GEMM_DRAIN);
      }
      if (XFORM) {  // this CTA's own A copies
        const long long first = fills > STAGES ? fills - STAGES : 0;
        for (long long j = first; j < fills; ++j)
          mbar_wait(&ctrl->afull[j % STAGES], static_cast<uint32_t>((j / STAGES) & 1),
                    DEVERR_GEMM_DRAIN);
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      uint32_t stage = 0, phase = 0;
      const uint64_t a_desc0 = operand_desc(smem_u32(ring), args.a_mn, 0);
      const uint64_t b_desc0 = operand_desc(smem_u32(ring) + Cfg::A_BYTES, args.b_mn, 0);
      const uint32_t a_step = operand_kstep(args.a_mn), b_step = operand_kstep(args.b_mn);
      for (int local = 0; !ctrl->abort_flag; ++local) {
        long long u;
        if (dyn) {
          if (!queue_take(ctrl, local, qempty0, true, &u)) {
            ctrl->abort_flag = 1;
            break;
          }
        } else {
          u = static_unit(args, cluster_id, nclusters, local);
        }
        if (u < 0) break;
        int b, tm, tn, kb0, kb1;
        decode_unit(args, u, b, tm, tn, kb0, kb1);
        const int acc_slot = local % Cfg::ACC_BUFS;
        const uint32_t use = static_cast<uint32_t>(local / Cfg::ACC_BUFS);
        if (!mbar_wait(&ctrl->tempty[acc_slot], (use & 1u) ^ 1u, DEVERR_GEMM_WAIT_TMEM_EMPTY)) {
          ctrl->abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc_slot * BN);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&ctrl->full[stage], phase, DEVERR_GEMM_WAIT_FULL)) {
            ctrl->abort_flag = 1;
            ok = false;
            break;
          }
          // both CTAs' A tiles rewritten in place (their transform warps
          // arrive with cluster release after a proxy fence)
          if (XFORM && !mbar_wait_cluster(&ctrl->xready[stage], phase, DEVERR_GEMM_WAIT_FULL)) {
            ctrl->abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t off = stage * Cfg::STAGE_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            const uint64_t da = desc_advance(a_desc0, off + kk * a_step);
            const uint32_t accumulate = (kb > kb0 || kk > 0) ? 1u : 0u;
#pragma unroll
            for (int h = 0; h < Cfg::NSUB; ++h) {
              const uint32_t dh = d_tmem + static_cast<uint32_t>(h * Cfg::MMA_N);
              const uint32_t bo = off + static_cast<uint32_t>(h * Cfg::B_SUB_BYTES);
              const uint64_t db = desc_advance(b_desc0, bo + kk * b_step);
              if (SPLIT3) {
                // lo·hi + hi·lo + hi·hi, as in the one-CTA kernel
                const uint32_t lo = Cfg::A_BYTES + Cfg::B_BYTES;
                umma_tf32_pair(dh, desc_advance(a_desc0, off + lo + kk * a_step), db,
                               args.idesc, accumulate);
                umma_tf32_pair(dh, da, desc_advance(b_desc0, bo + lo + kk * b_step),
                               args.idesc, 1u);
                umma_tf32_pair(dh, da, db, args.idesc, 1u);
              } else {
                umma_tf32_pair(dh, da, db, args.idesc, accumulate);
              }
            }
          }
          umma_commit_pair(&ctrl->empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&ctrl->tfull[acc_slot], 0x3);
      }
    }
  } else if (XFORM && warp >= 2 + EPI_WARPS - XFORM_WARPS) {
    // A-operand transform: one thread per row of this CTA's A tile scales
    // each landed stage in place into softmax probabilities (row statistics
    // from the score product's epilogue), then arrives on the leader's xready.
    const int row_local = (warp & 3) * 32 + lane;
    const uint32_t xready0 = map_to_rank(&ctrl->xready[0], 0);
    uint32_t stage = 0, phase = 0;
    for (int local = 0; !ctrl->abort_flag; ++local) {
      long long u;
      if (dyn) {
        if (!queue_take(ctrl, local, qempty0, false, &u)) {
          ctrl->abort_flag = 1;
          break;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(qempty0 + 8u * static_cast<uint32_t>(local % TQ));
      } else {
        u = static_unit(args, cluster_id, nclusters, local);
      }
      if (u < 0) break;
      int b, tm, tn, kb0, kb1;
      decode_unit(args, u, b, tm, tn, kb0, kb1);
      const int m = tm * 2 * BM + static_cast<int>(rank) * BM + row_local;
      // row statistics, chunk-major: chunk c of row m at st[c * chunk_stride]
      const long long chunk_stride = args.M;
      const float2* st = args.stats_in + static_cast<long long>(b) * args.stats_chunks * args.M + m;
      const bool live = m < args.M;
      // Each chunk's factor exp(m_c - max) / sum, prepared per row by
      // softmax_stats_finalize_kernel. Factors are loaded four stages ahead
      // into four fixed registers, each consumed four stages after its load
      // (no register moves, which would wait on the loads): a global load
      // per stage would otherwise sit between a landed tile and its MMAs.
      auto factor = [&](int kb) { return (live && kb < kb1) ? st[kb * chunk_stride].x : 0.0f; };
      // K block kb is score chunk kb of the row: p = E * factor
      auto step = [&](int kb, float f) -> bool {
        (void)kb;
        if (!mbar_wait(&ctrl->afull[stage], phase, DEVERR_GEMM_WAIT_FULL)) return false;
        scale_tile_row(ring + stage * Cfg::STAGE_BYTES, row_local, f);
        fence_proxy_async_smem();  // generic writes, read next by the tensor cores
        __syncwarp();
        if (lane == 0) {
          if (leader) mbar_arrive(&ctrl->xready[stage]);
          else mbar_arrive_remote(xready0 + 8u * stage);
        }
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
        return true;
      };
      float c0 = factor(kb0), c1 = factor(kb0 + 1), c2 = factor(kb0 + 2), c3 = factor(kb0 + 3);
      bool ok = true;
      for (int kb = kb0; kb < kb1 && ok; kb += 4) {
        ok = step(kb, c0);
        c0 = factor(kb + 4);
        if (!ok || kb + 1 >= kb1) break;
        ok = step(kb + 1, c1);
        c1 = factor(kb + 5);
        if (!ok || kb + 2 >= kb1) break;
        ok = step(kb + 2, c2);
        c2 = factor(kb + 6);
        if (!ok || kb + 3 >= kb1) break;
        ok = step(kb + 3, c3);
        c3 = factor(kb + 7);
      }
      if (!ok) ctrl->abort_flag = 1;
      if (!ok) break;
    }
  } else {
    const int quarter = warp & 3;
    const int group = (warp - 2) / 4;
    const int row_local = quarter * 32 + lane;
    // chunk stride: with transform warps, the epilogue warps of group 0 take
    // every chunk of a tile
    constexpr int cstep = XFORM ? 1 : EPI_GROUPS;
    uint8_t* bufs = ring + STAGES * Cfg::STAGE_BYTES + (warp - 2) * EPI_TILE_BYTES * NB;
    EpiRing<NB> rg;
    ring_init(rg, bufs, &ctrl->epi[(warp - 2) * EPI_NB_MAX]);
    bool ok = true;
    int pf = -1;  // the tile the next chunk's first input is being loaded into
    // only an epilogue that reads an input tile first looks ahead to prefetch it
    int la3d = 0;
    const bool lookahead = args.epi_tma && epi_first_input(args, em, la3d) != nullptr;
    for (int local = 0; ok; ++local) {
      long long u;
      if (dyn) {
        if (!queue_take(ctrl, local, qempty0, false, &u)) {
          ctrl->abort_flag = 1;
          break;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(qempty0 + 8u * static_cast<uint32_t>(local % TQ));
      } else {
        u = static_unit(args, cluster_id, nclusters, local);
      }
      if (u < 0) break;
      int b, tm, tn, kb0, kb1;
      decode_unit(args, u, b, tm, tn, kb0, kb1);
      const int acc_slot = local % Cfg::ACC_BUFS;
      const uint32_t use = static_cast<uint32_t>(local / Cfg::ACC_BUFS);
      if (!mbar_wait(&ctrl->tfull[acc_slot], use & 1u, DEVERR_GEMM_WAIT_TMEM_FULL)) {
        ctrl->abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int m_base = tm * 2 * BM + static_cast<int>(rank) * BM;
      const int m = m_base + row_local;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc_slot * BN);
#pragma unroll 1
      for (int c = group; c < BN / 32; c += cstep) {
        const int n0 = tn * BN + c * 32;
        if (n0 >= args.N) break;
        float v[32];
        tmem_ld_32x32b_x32(taddr + pair_chunk_tmem_col<BN>(c), v);
        if (args.epi_tma) {
          const int m0 = m_base + quarter * 32;
          if (!epilogue_chunk_tma(args, em, b, m0, n0, v, rg, lane, pf)) {
            ctrl->abort_flag = 1;
            ok = false;
            pf = -1;
            break;
          }
          pf = -1;
          if (lookahead) {
            int nb, nm0, nn0;
            long long u2 = -2;  // the next unit, needed after the tile's last chunk only
            if (c + cstep >= BN / 32 || tn * BN + (c + cstep) * 32 >= args.N) {
              if (dyn) {
                if (lane == 0) u2 = queue_peek(ctrl, local + 1);
                u2 = __shfl_sync(0xffffffffu, u2, 0);
              } else {
                u2 = static_unit(args, cluster_id, nclusters, local + 1);
              }
            }
            if (epi_next_chunk<BN>(args, u2, c, group, static_cast<int>(rank) * BM + quarter * 32,
                                   b, tn, m0, nb, nm0, nn0, cstep))
              pf = epi_prefetch(args, em, rg, nb, nm0, nn0, lane);
          }
        } else if (m < args.M) {
          epilogue_chunk(args, b, m, n0, v);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(tempty0 + 8u * static_cast<uint32_t>(acc_slot));
    }
    if (pf >= 0) ring_wait(rg, pf);  // an abandoned prefetch must land before exit
    if (lane == 0) bulk_wait_group0();  // no store may outlive the CTA's shared memory
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its partner may still signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
  schedule_release(args);
}

// ---------------------------------------------------------------- 3xTF32 split
// hi = TF32 (round to nearest, ties away) of x, lo = x - hi; both f32.
__global__ void split_tf32_kernel(const float* __restrict__ src, long long ld, long long stride,
                                  int inner, int outer, float* __restrict__ hi,
                                  float* __restrict__ lo) {
  const long long per = static_cast<long long>(inner) * outer;
  const int b = blockIdx.y;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < per;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / inner, c = i - r * inner;
    const float x = src[b * stride + r * ld + c];
    uint32_t h;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
    const float hf = __uint_as_float(h);
    hi[b * per + i] = hf;
    lo[b * per + i] = x - hf;
  }
}

// ---------------------------------------------------------------- SIMT fallback
// Used only for shapes TMA cannot describe (leading dimension not a multiple
// of 4 elements, misaligned base, K == 0). Operands are rounded to TF32 like
// the reference (gemm.rs:286-347) unless `exact`.
__global__ void gemm_simt_kernel(const GemmArgs a, const float* __restrict__ A, long long lda,
                                 long long sa, const float* __restrict__ B, long long ldb,
                                 long long sb, int exact) {
  __shared__ float As[32][33];
  __shared__ float Bs[32][33];
  const int b = blockIdx.z;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  const int m0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = 0; k0 < a.K; k0 += 32) {
    for (int i = ty; i < 32; i += 8) {
      const int m = m0 + i, k = k0 + tx;
      float va = 0.f;
      if (m < a.M && k < a.K)
        va = a.a_mn ? A[b * sa + static_cast<long long>(k) * lda + m]
                    : A[b * sa + static_cast<long long>(m) * lda + k];
      const int kb = k0 + i, n = n0 + tx;
      float vb = 0.f;
      if (kb < a.K && n < a.N)
        vb = a.b_mn ? B[b * sb + static_cast<long long>(kb) * ldb + n]
                    : B[b * sb + static_cast<long long>(n) * ldb + kb];
      if (!exact) {
        uint32_t h;
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(va));
        va = __uint_as_float(h);
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(vb));
        vb = __uint_as_float(h);
      }
      As[i][tx] = va;
      Bs[i][tx] = vb;
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < 32; ++k) {
      const float bv = Bs[k][tx];
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[r] += As[ty + 8 * r][k] * bv;
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int m = m0 + ty + 8 * r, n = n0 + tx;
    if (m >= a.M || n >= a.N) continue;
    float* crow = a.C + b * a.sc + static_cast<long long>(m) * a.ldc;
    float v = acc[r] * a.alpha;
    if (a.beta != 0.0f) v += a.beta * crow[n];
    if (a.bias) v += a.bias[n];
    if (a.R) v += a.R[b * a.sr + static_cast<long long>(m) * a.ldr + n];
    if (a.P) a.P[b * a.sp + static_cast<long long>(m) * a.ldp + n] = v;
    if (a.X) v *= act_derivative(a.grad_act, a.X[b * a.sx + static_cast<long long>(m) * a.ldx + n]);
    v = act_forward(a.act, v);
    if (a.accumulate) atomicAdd(crow + n, v);
    else crow[n] = v;
  }
}

// ---------------------------------------------------------------- tiny products
// For products of a few million multiply-adds (config 1: 256x64x128) the
// persistent tcgen05 kernel is all fixed latency: TMEM allocation, a TMA
// load, the MMAs, a TMEM read and a TMA store in sequence. This kernel needs
// one memory round trip: a 256-thread CTA owns a 16x16 output tile, loads its
// whole A panel (16 x K) and B panel (K x 16, K <= 256) into shared memory at
// once, rounding each operand to TF32 (round to nearest, ties away, as the
// reference's kernel does), then each thread forms one output with f32 FMAs
// in K order and applies the fused epilogue of the SIMT kernel.
constexpr int SMALL_TILE = 16;
constexpr int SMALL_KMAX = 256;
constexpr double SMALL_MAX_MACS = 4194304.0;  // 2^22 multiply-adds over the batch

__device__ __forceinline__ float round_tf32_rna(float x) {
  uint32_t h;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
  return __uint_as_float(h);
}

__global__ void __launch_bounds__(256)
    gemm_small_kernel(const GemmArgs a, const float* __restrict__ A, long long lda, long long sa,
                      const float* __restrict__ B, long long ldb, long long sb) {
  __shared__ float As[SMALL_TILE][SMALL_KMAX + 1];
  __shared__ float Bs[SMALL_KMAX][SMALL_TILE + 1];
  const int b = blockIdx.z, t = threadIdx.x;
  const int m0 = blockIdx.y * SMALL_TILE, n0 = blockIdx.x * SMALL_TILE;
  const int K = a.K;
  constexpr int PER = SMALL_KMAX / 16;  // k steps of 16 per thread and operand
  // Thread t owns index pair (t / 16, t % 16): the 16 threads of a
  // half-warp read 16 consecutive addresses of whichever layout is given
  // (K-major: along k; MN-major: along m or n), stepping k by 16. Every
  // load is issued before any is used (one round trip).
  const int hi = t >> 4, lo = t & 15;
  const int ar = a.a_mn ? lo : hi, ak = a.a_mn ? hi : lo;  // A: row in tile, first k
  const int bc = a.b_mn ? lo : hi, bk = a.b_mn ? hi : lo;  // B: column in tile, first k
  const bool arow_ok = m0 + ar < a.M, bcol_ok = n0 + bc < a.N;
  const float* ap = A + b * sa + (a.a_mn ? static_cast<long long>(ak) * lda + m0 + ar
                                         : static_cast<long long>(m0 + ar) * lda + ak);
  const float* bp = B + b * sb + (a.b_mn ? static_cast<long long>(bk) * ldb + n0 + bc
                                         : static_cast<long long>(n0 + bc) * ldb + bk);
  const long long astep = a.a_mn ? 16 * lda : 16, bstep = a.b_mn ? 16 * ldb : 16;
  float va[PER], vb[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    va[j] = (arow_ok && ak + 16 * j < K) ? __ldg(ap + j * astep) : 0.f;
    vb[j] = (bcol_ok && bk + 16 * j < K) ? __ldg(bp + j * bstep) : 0.f;
  }
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    if (ak + 16 * j < K) As[ar][ak + 16 * j] = round_tf32_rna(va[j]);
    if (bk + 16 * j < K) Bs[bk + 16 * j][bc] = round_tf32_rna(vb[j]);
  }
  __syncthreads();
  const int r = t / SMALL_TILE, c = t % SMALL_TILE;
  const int m = m0 + r, nn = n0 + c;
  float acc = 0.f;
#pragma unroll 8
  for (int k = 0; k < K; ++k) acc = fmaf(As[r][k], Bs[k][c], acc);
  if (m >= a.M || nn >= a.N) return;
  float* crow = a.C + b * a.sc + static_cast<long long>(m) * a.ldc;
  float v = acc * a.alpha;
  if (a.beta != 0.0f) v += a.beta * crow[nn];
  if (a.bias) v += a.bias[nn];
  if (a.R) v += a.R[b * a.sr + static_cast<long long>(m) * a.ldr + nn];
  if (a.P) a.P[b * a.sp + static_cast<long long>(m) * a.ldp + nn] = v;
  if (a.X) v *= act_derivative(a.grad_act, a.X[b * a.sx + static_cast<long long>(m) * a.ldx + nn]);
  v = act_forward(a.act, v);
  if (a.accumulate) atomicAdd(crow + nn, v);
  else crow[nn] = v;
}

// ---------------------------------------------------------------- reference algorithm
// Measurement-only restatement of the reference GEMM (gemm.rs:131-373):
// 32x32 output tile per 128-thread CTA, four warps of 16x16 (two
// mma.sync.m16n8k8 TF32 each), K tiles of 16 staged by 4-byte cp.async in two
// buffers, B transposed into shared memory with a row stride of 20 floats.
__device__ __forceinline__ void cp_async4_zfill(float* smem, const float* gmem, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(smem)),
               "l"(gmem), "r"(valid ? 4 : 0)
               : "memory");
}

__device__ __forceinline__ uint32_t tf32_rna_bits(float x) {
  uint32_t h;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
  return h;
}

__global__ void __launch_bounds__(128) gemm_refalgo_kernel(const float* __restrict__ A,
                                                           const float* __restrict__ B,
                                                           float* __restrict__ C, int len,
                                                           int rows, int cols) {
  constexpr int T = 32, KT = 16, STRIDE = 20, STAGE = T * STRIDE;
  __shared__ __align__(16) float sa[2 * STAGE];
  __shared__ __align__(16) float sb[2 * STAGE];
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int group = lane / 4, tig = lane % 4;
  const int wr = warp / 2, wc = warp % 2;
  const int br = blockIdx.y * T, bc = blockIdx.x * T;
  float acc0[4] = {0, 0, 0, 0}, acc1[4] = {0, 0, 0, 0};
  auto prefetch = [&](int buf, int k0) {
    for (int l = 0; l < 4; ++l) {
      const int li = tid + l * 128;
      const int ar = li / KT, ak = li % KT, gr = br + ar;
      const bool av = gr < rows;
      cp_async4_zfill(&sa[buf * STAGE + ar * STRIDE + ak], av ? A + (size_t)gr * len + k0 + ak : A,
                      av);
      const int bk = li / T, bcol = li % T, gc = bc + bcol;
      const bool bv = gc < cols;
      cp_async4_zfill(&sb[buf * STAGE + bcol * STRIDE + bk],
                      bv ? B + (size_t)(k0 + bk) * cols + gc : B, bv);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  const int tiles = len / KT;
  prefetch(0, 0);
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  for (int t = 0; t < tiles; ++t) {
    const int rb = (t % 2) * STAGE;
    if (t + 1 < tiles) prefetch((t + 1) % 2, (t + 1) * KT);
#pragma unroll
    for (int kh = 0; kh < 2; ++kh) {
      const int lk = kh * 8, ar0 = wr * 16, bc0 = wc * 16;
      uint32_t a0 = tf32_rna_bits(sa[rb + (ar0 + group) * STRIDE + lk + tig]);
      uint32_t a1 = tf32_rna_bits(sa[rb + (ar0 + group + 8) * STRIDE + lk + tig]);
      uint32_t a2 = tf32_rna_bits(sa[rb + (ar0 + group) * STRIDE + lk + tig + 4]);
      uint32_t a3 = tf32_rna_bits(sa[rb + (ar0 + group + 8) * STRIDE + lk + tig + 4]);
      uint32_t b00 = tf32_rna_bits(sb[rb + (bc0 + group) * STRIDE + lk + tig]);
      uint32_t b01 = tf32_rna_bits(sb[rb + (bc0 + group) * STRIDE + lk + tig + 4]);
      uint32_t b10 = tf32_rna_bits(sb[rb + (bc0 + group + 8) * STRIDE + lk + tig]);
      uint32_t b11 = tf32_rna_bits(sb[rb + (bc0 + group + 8) * STRIDE + lk + tig + 4]);
      asm volatile(
          "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
          "{%8,%9}, {%0,%1,%2,%3};"
          : "+f"(acc0[0]), "+f"(acc0[1]), "+f"(acc0[2]), "+f"(acc0[3])
          : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b00), "r"(b01));
      asm volatile(
          "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
          "{%8,%9}, {%0,%1,%2,%3};"
          : "+f"(acc1[0]), "+f"(acc1[1]), "+f"(acc1[2]), "+f"(acc1[3])
          : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b10), "r"(b11));
    }
    if (t + 1 < tiles) {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
      __syncthreads();
    }
  }
  for (int r = 0; r < 4; ++r) {
    const int orow = br + wr * 16 + group + (r >= 2 ? 8 : 0);
    const int ocol = bc + wc * 16 + tig * 2 + r % 2;
    if (orow < rows && ocol < cols) C[(size_t)orow * cols + ocol] = acc0[r];
    if (orow < rows && ocol + 8 < cols) C[(size_t)orow * cols + ocol + 8] = acc1[r];
  }
}

// ================================================================== host side
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}



// K blocks of 32 (K >= 4096) from which a wide (256 x 512) pair tile's
// exposed epilogue is short against its MMAs: below it, products with a
// heavy epilogue keep 256-wide tiles, and wide tiles stage through two
// tiles per epilogue warp.
constexpr long long kWideMinKBlocks = 128;

// ---------------------------------------------------------------- schedule slots
constexpr int kSchedSlots = 64;
__device__ unsigned long long g_sched_next[kSchedSlots];
__device__ unsigned int g_sched_done[kSchedSlots];

// The dynamic schedule's counter slot for `stream` on device `dev`: one slot
// per stream, so GEMMs that may run concurrently never share a counter;
// launches on one stream are ordered, and each launch's last CTA resets the
// slot before the next launch starts. Static schedule (false) under graph
// capture (a replay could overlap other work of the capturing stream), for
// the per-thread default stream, once every slot is taken, or when the
// environment sets OXF_GEMM_SCHEDULE=static.
bool schedule_slot(cudaStream_t stream, int dev, unsigned long long** next, unsigned int** done) {
  const char* env = std::getenv("OXF_GEMM_SCHEDULE");
  if (env && std::strcmp(env, "static") == 0) return false;
  if (dev < 0 || dev >= kMaxDevices || stream == cudaStreamPerThread) return false;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (cs != cudaStreamCaptureStatusNone) return false;
  static std::mutex mu;
  static std::vector<cudaStream_t> streams[kMaxDevices];
  static unsigned long long* next_base[kMaxDevices];
  static unsigned int* done_base[kMaxDevices];
  static unsigned long long ctx_of[kMaxDevices];
  std::lock_guard<std::mutex> lock(mu);
  const unsigned long long ctx = current_context_id();
  if (!next_base[dev] || (ctx != 0 && ctx != ctx_of[dev])) {
    // first use on this device, or a new context (after a device reset):
    // fresh addresses, and the old context's streams are gone
    void *p = nullptr, *q = nullptr;
    if (cudaGetSymbolAddress(&p, g_sched_next) != cudaSuccess ||
        cudaGetSymbolAddress(&q, g_sched_done) != cudaSuccess) {
      cudaGetLastError();
      next_base[dev] = nullptr;
      return false;
    }
    next_base[dev] = static_cast<unsigned long long*>(p);
    done_base[dev] = static_cast<unsigned int*>(q);
    ctx_of[dev] = current_context_id();
    streams[dev].clear();
  }
  auto& v = streams[dev];
  const size_t k = static_cast<size_t>(std::find(v.begin(), v.end(), stream) - v.begin());
  if (k == v.size()) {
    if (v.size() >= static_cast<size_t>(kSchedSlots)) return false;
    v.push_back(stream);
  }
  *next = next_base[dev] + k;
  *done = done_base[dev] + k;
  return true;
}

int sm_count(int dev) {
  static int counts[kMaxDevices] = {0};
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (counts[dev] == 0) {
    int c = 0;
    cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
    counts[dev] = c > 0 ? c : 148;
  }
  return counts[dev];
}


// Launches a persistent GEMM kernel with programmatic stream serialisation
// (see pdl_after_prologue) and counts it.
using GemmKernel = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap,
                            const CUtensorMap, const EpiMaps, const GemmArgs);
oxf_status launch_gemm_pdl(const char* name, GemmKernel kernel, unsigned grid, int smem,
                           cudaStream_t stream, const CUtensorMap& ta, const CUtensorMap& tb,
                           const CUtensorMap& ta_lo, const CUtensorMap& tb_lo, const EpiMaps& em,
                           const GemmArgs& args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, ta, tb, ta_lo, tb_lo, em, args);
  count_launch();
  return check_cuda(e != cudaSuccess ? e : cudaGetLastError(), name);
}

template <int BN, int STAGES, bool SPLIT3>
oxf_status launch_tcgen05(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta_lo,
                          const CUtensorMap& tb_lo, const EpiMaps& em, GemmArgs& args,
                          cudaStream_t stream, int dev) {
  using Cfg = GemmCfg<BN, STAGES, SPLIT3>;
  // once per device and context (a device reset drops the attribute)
  static unsigned long long configured[kMaxDevices] = {0};
  const unsigned long long ctx = current_context_id();
  if (dev >= 0 && dev < kMaxDevices && (ctx == 0 || configured[dev] != ctx)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tf32_tcgen05<BN, STAGES, SPLIT3>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(gemm)");
    configured[dev] = ctx;
  }
  args.idesc = make_idesc_tf32(BM, BN, args.a_mn != 0, args.b_mn != 0);
  const long long grid = std::min<long long>(args.units, sm_count(dev));
  args.sched_next = nullptr;
  args.sched_done = nullptr;
  if (args.units > grid) schedule_slot(stream, dev, &args.sched_next, &args.sched_done);
  return launch_gemm_pdl("gemm_tf32_tcgen05", gemm_tf32_tcgen05<BN, STAGES, SPLIT3>,
                         static_cast<unsigned>(grid), Cfg::SMEM_BYTES, stream, ta, tb, ta_lo,
                         tb_lo, em, args);
}

template <int BN, int STAGES, bool SPLIT3, int NB, bool XFORM = false>
oxf_status launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta_lo,
                       const CUtensorMap& tb_lo, const EpiMaps& em, GemmArgs& args,
                       cudaStream_t stream, int dev) {
  using Cfg = GemmPairCfg<BN, STAGES, SPLIT3, NB, XFORM>;
  // once per device and context (a device reset drops the attribute)
  static unsigned long long configured[kMaxDevices] = {0};
  const unsigned long long ctx = current_context_id();
  if (dev >= 0 && dev < kMaxDevices && (ctx == 0 || configured[dev] != ctx)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tf32_tcgen05_pair<BN, STAGES, SPLIT3, NB, XFORM>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(gemm pair)");
    configured[dev] = ctx;
  }
  args.idesc = make_idesc_tf32(2 * BM, Cfg::MMA_N, args.a_mn != 0, args.b_mn != 0);
  const long long clusters = std::min<long long>(args.units, sm_count(dev) / 2);
  args.sched_next = nullptr;
  args.sched_done = nullptr;
  if (args.units > clusters) schedule_slot(stream, dev, &args.sched_next, &args.sched_done);
  return launch_gemm_pdl("gemm_tf32_tcgen05_pair",
                         gemm_tf32_tcgen05_pair<BN, STAGES, SPLIT3, NB, XFORM>,
                         static_cast<unsigned>(2 * clusters), Cfg::SMEM_BYTES, stream, ta, tb,
                         ta_lo, tb_lo, em, args);
}

// Chooses how many K splits an accumulating GEMM uses: minimises
// waves * k-blocks-per-unit plus a per-split epilogue cost, for `slots`
// concurrent units (SMs, or CTA pairs for pair tiles).
int choose_splits(long long tiles, int kblocks, int slots) {
  int best = 1;
  double best_cost = 1e300;
  for (int s = 1; s <= 32 && s <= kblocks; ++s) {
    const long long units = tiles * s;
    const long long waves = (units + slots - 1) / slots;
    const double cost = static_cast<double>(waves) * ((kblocks + s - 1) / s) + 2.0 * s;
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

bool tma_ok_ptr(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Epilogue operand map: an [M x N] f32 matrix (leading dimension ld, batch
// stride bstride; 0 = shared by the batch) moved in 32 x 32 boxes with the
// 128B swizzle of the staging tiles.
bool encode_epi_map(CUtensorMap* map, const float* ptr, long long n, long long m, long long ld,
                    int batch, long long bstride, int* is3d) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const bool three = batch > 1 && bstride != 0;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(m),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 4, static_cast<cuuint64_t>(bstride) * 4};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, three ? 3 : 2, const_cast<float*>(ptr),
                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  *is3d = three ? 1 : 0;
  return r == CUDA_SUCCESS;
}

}  // namespace

// The unique ID of the calling thread's current CUDA context (cuCtxGetId),
// or 0 when no context is current yet or the driver cannot say. Host-side
// caches of per-device state (symbol addresses, kernel attributes) record
// it, so that after a cudaDeviceReset, which destroys the context and with
// it every device address of this library's module, they look the state up
// again instead of handing out addresses of the destroyed context.
unsigned long long current_context_id() {
  using GetCurrentFn = CUresult (*)(CUcontext*);
  using GetIdFn = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrentFn get_current = nullptr;
  static GetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetIdFn>(p);
  });
  if (!get_current || !get_id) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// 2-D (or 3-D with a batch dimension) f32 tensor map, zero fill outside the
// tensor. K-major tiles use the 128B swizzle; MN-major tiles the 128B swizzle
// with 32-byte atoms, matching the shared-memory descriptors above.
bool encode_map(CUtensorMap* map, const float* ptr, long long inner, long long outer,
                long long ld, int batch, long long bstride, int box_inner, int box_outer,
                bool mn_major, int* is3d) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const bool three = batch > 1 && bstride != 0;
  if (mn_major && box_outer > 32) {
    // Chunked MN-major view: (32 elements, K rows, inner/32 chunks[, batch]).
    // Only used when inner % 32 == 0, so no box reads past a row's end.
    cuuint64_t dims[4] = {32, static_cast<cuuint64_t>(outer), static_cast<cuuint64_t>(inner / 32),
                          static_cast<cuuint64_t>(batch)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(ld) * 4, 128,
                             static_cast<cuuint64_t>(bstride) * 4};
    cuuint32_t box[4] = {32, 32, static_cast<cuuint32_t>(box_outer / 32), 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, three ? 4 : 3, const_cast<float*>(ptr),
                     dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    *is3d = three ? 1 : 0;
    return r == CUDA_SUCCESS;
  }
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 4, static_cast<cuuint64_t>(bstride) * 4};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, three ? 3 : 2, const_cast<float*>(ptr),
                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  *is3d = three ? 1 : 0;
  return r == CUDA_SUCCESS;
}

size_t gemm_workspace_bytes(const oxf_gemm_desc* d) {
  if (!d || d->precision != OXF_PREC_TF32X3) return 0;
  const long long ba = d->stride_a ? d->batch : 1;
  const long long bb = d->stride_b ? d->batch : 1;
  const long long ea = static_cast<long long>(d->M) * d->K * ba;
  const long long eb = static_cast<long long>(d->K) * d->N * bb;
  // hi and lo of each operand, each region rounded up to 256 bytes
  auto r = [](long long e) { return ((e * 4 + 255) / 256) * 256; };
  return static_cast<size_t>(2 * r(ea) + 2 * r(eb));
}

namespace {

// The descriptor checks of oxf_gemm, shared by every GEMM entry point. OK
// also for an empty output (M or N zero), which the caller treats as a no-op.
oxf_status gemm_validate(const oxf_gemm_desc* d) {
  if (!d) return set_error(OXF_ERR_INVALID_ARG, "oxf_gemm: null descriptor");
  if (d->M < 0 || d->N < 0 || d->K < 0 || d->batch < 1)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_gemm: negative shape or batch < 1");
  if (d->M == 0 || d->N == 0) return OXF_OK;
  if (!d->C || (d->K > 0 && (!d->A || !d->B)))
    return set_error(OXF_ERR_INVALID_ARG, "oxf_gemm: null operand");
  const int split = d->split_k > 1 ? d->split_k : 1;
  if (split > 1 && !d->accumulate)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_gemm: split_k > 1 requires accumulate");
  if (d->accumulate && d->beta != 0.0f)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_gemm: beta must be 0 with accumulate");
  if (d->precision != OXF_PREC_TF32 && d->precision != OXF_PREC_TF32X3 &&
      d->precision != OXF_PREC_F32)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_gemm: unknown precision %d", d->precision);
  const long long min_lda = d->a_trans ? d->M : d->K;
  const long long min_ldb = d->b_trans ? d->K : d->N;
  if (d->lda < min_lda || d->ldb < min_ldb || d->ldc < d->N)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_gemm: leading dimension too small");
  if ((d->residual && d->ldr < d->N) || (d->pre_out && d->ldp < d->N) ||
      (d->aux && d->ldx < d->N))
    return set_error(OXF_ERR_INVALID_ARG, "oxf_gemm: epilogue leading dimension too small");
  if (d->aux && d->grad_act == OXF_ACT_IDENTITY)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_gemm: aux given without grad_act");
  if (d->accumulate && (d->pre_out || d->act != OXF_ACT_IDENTITY) && split > 1)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_gemm: split_k cannot fuse activation");
  if (d->accumulate && (d->bias || d->residual) && split > 1)
    return set_error(OXF_ERR_INVALID_ARG,
                     "oxf_gemm: split_k would add bias / residual once per split");
  return OXF_OK;
}

// Whether a valid, non-empty descriptor runs on the tensor cores: TMA needs
// 16-byte aligned bases, leading dimensions and batch strides, and
// OXF_PREC_F32 asks for f32 products on the CUDA cores. Otherwise the SIMT
// kernel runs, which needs no operand splits for any precision.
bool gemm_tensor_core_path(const oxf_gemm_desc* d) {
  return d->K > 0 && tma_ok_ptr(d->A) && tma_ok_ptr(d->B) && d->lda % 4 == 0 &&
         d->ldb % 4 == 0 && d->stride_a % 4 == 0 && d->stride_b % 4 == 0 &&
         d->precision != OXF_PREC_F32;
}

// The kernel a tensor-core product runs on, its tile, K splits and raster:
// a pure function of the descriptor and the SM count, so that the rule can
// be reported (oxf_gemm_plan) and tested without a GPU.
struct GemmPlan {
  int bn = 256;            // tile width along N (per CTA pair for pair tiles)
  bool pair = false;       // a CTA pair per 256-row tile, else one CTA per 128 rows
  bool split3 = false;     // 3xTF32: hi/lo operand splits, three MMAs per K step
  bool zero_c = false;     // a plain product whose K splits add into a zeroed C
  int stages = 0;          // operand ring stages
  int staging = 1;         // epilogue staging tiles per warp
  int bm = BM, tiles_m = 0, tiles_n = 0, group_m = 1;
  int kblocks_item = 0, kblocks = 0, splits = 1;
  long long units = 0;
};

GemmPlan plan_gemm(const oxf_gemm_desc* d, bool fused, bool fused_transform, int sms) {
  GemmPlan p;
  const int split = d->split_k > 1 ? d->split_k : 1;
  const bool reduce = d->reduce_batch && d->batch > 1;
  const bool split3 = d->precision == OXF_PREC_TF32X3;
  p.split3 = split3;
  // Tile width along N.
  // The one-CTA 3xTF32 kernel is instantiated for BN = 128 only.
  int BN = 256;
  if (split3 || d->N <= 128) BN = 128;
  if (!split3 && d->N <= 64) BN = 64;
  if (!split3 && BN == 256) {
    const long long t256 = static_cast<long long>((d->M + BM - 1) / BM) * ((d->N + 255) / 256) *
                           d->batch;
    if (t256 < sms && !d->accumulate) BN = 128;  // more, smaller tiles when the grid is thin
  }
  // A plain product: nothing in the epilogue but alpha, so K may be split.
  const bool plain = !fused && d->variant == 0 && !split3 && !d->accumulate && split <= 1 &&
                     d->beta == 0.0f && !d->bias && !d->residual && !d->pre_out && !d->aux &&
                     d->act == OXF_ACT_IDENTITY && !reduce && d->batch == 1;
  // A small plain product (at most half a wave of 128 x 64 tiles, K <= 1024;
  // 512^3 has 32) runs on one-CTA 128 x 64 tiles, K split as below: a pair
  // tile's longer set-up and per-tile drain outweigh its operand savings
  // there (512^3: 9 against 13 us per call).
  const bool small_tiles =
      plain && (d->K + BK - 1) / BK <= 32 &&
      static_cast<long long>((d->M + BM - 1) / BM) * ((d->N + 63) / 64) * 2 <= sms;
  if (small_tiles) BN = 64;
  // CTA pairs (256 x 256 tiles, half the L2->SM bytes per flop of a one-CTA
  // tile) whenever there are enough of them to occupy every SM pair;
  // variant 1 forces one CTA, 2 forces pairs.
  bool pair = false, autosplit = false;
  {
    const long long tiles2 = static_cast<long long>((d->M + 2 * BM - 1) / (2 * BM)) *
                             ((d->N + 255) / 256) * (d->reduce_batch ? 1 : d->batch);
    // An accumulating product with long K reaches every pair through K
    // splits even when it has fewer tiles than pairs (weight gradients).
    const bool splittable = d->accumulate && split <= 1 && !d->bias && !d->residual &&
                            static_cast<long long>((d->K + BK - 1) / BK) *
                                    (d->reduce_batch ? d->batch : 1) >= 2 * kWideMinKBlocks;
    // A plain product (nothing in the epilogue but alpha) with too few tiles
    // to fill the GPU splits K: C is zeroed and the splits add into it.
    autosplit = plain && d->M >= 2 * BM && tiles2 < (3 * sms / 2) / 4 &&
                (d->K + BK - 1) / BK >= 16;
    // One partly filled wave of pairs (at least 3/4 of them busy) beats
    // 1.5-2 waves of one-CTA tiles with twice the operand bytes per flop.
    const long long pair_min = (3 * (sms / 2)) / 4;
    pair = fused || d->variant == 2 || d->variant == 3 ||
           (d->variant == 0 && !small_tiles && d->M >= 2 * BM &&
            (tiles2 >= pair_min || splittable || autosplit));
    if (pair) BN = 256;
  }
  // Wide pair tiles (256 x 512): a quarter fewer operand bytes per flop
  // through L2, but a tile fills TMEM, so its epilogue no longer overlaps the
  // next tile's MMAs. Taken whenever the fewer, larger tiles fill the last
  // wave of CTA pairs about as well and keep at least 3/4 of the pairs busy
  // (config 3's residual products: 64 wide units in one partial wave ran 3%
  // faster than 128 narrow ones in 1.73 waves), except for short-K products whose
  // epilogue reads an input tile, writes a second output or applies an
  // activation: there the exposed epilogue outweighs the saved bytes, and
  // the 256-wide tile's two accumulators hide it. OXF_GEMM_TILE=256 / 512
  // overrides the choice.
  if (pair && !split3) {
    const long long kbl = static_cast<long long>((d->K + BK - 1) / BK) *
                          (d->reduce_batch ? d->batch : 1);
    const long long mt = (d->M + 2 * BM - 1) / (2 * BM), nb = d->reduce_batch ? 1 : d->batch;
    long long units_w = mt * ((d->N + 511) / 512) * nb;
    long long units_n = mt * ((d->N + 255) / 256) * nb;
    const long long pairs = sms / 2;
    auto waves = [pairs](long long u) { return (u + pairs - 1) / pairs; };
    auto fill = [pairs, waves](long long t) {
      return static_cast<double>(t) / static_cast<double>(waves(t) * pairs);
    };
    const bool auto_split = d->accumulate && split <= 1 && !d->bias && !d->residual;
    // For a K-split product: the estimated time of each tile in 256-tile K
    // blocks. A wave of units costs its K blocks (a wide one 1.77: twice the
    // flops at the wide tile's 13% higher rate) plus about 8 for the unit's
    // pipeline start and drain.
    double est_w = 0.0, est_n = 0.0;
    if (auto_split) {
      // split K as the launch below will, so that the fill compares units
      const int sw = choose_splits(units_w, static_cast<int>(kbl), static_cast<int>(pairs));
      const int sn = choose_splits(units_n, static_cast<int>(kbl), static_cast<int>(pairs));
      units_w *= sw;
      units_n *= sn;
      est_w = static_cast<double>(waves(units_w)) * (1.77 * ((kbl + sw - 1) / sw) + 8.0);
      est_n = static_cast<double>(waves(units_n)) * (static_cast<double>((kbl + sn - 1) / sn) + 8.0);
    }
    // an activation makes a drain of the same bytes about half as long again
    const bool heavy_epilogue = d->pre_out || d->aux || d->residual || d->beta != 0.0f ||
                                d->act != OXF_ACT_IDENTITY;
    // A K-split product also takes wide tiles where the 256 tile fills the
    // last wave better but only through several times more K splits, each a
    // unit with its own pipeline start and drain, so that its estimated time
    // is longer: config 3's weight gradients ran 18-21% faster on 64 wide
    // units of 2 splits than on 512 narrow units of 8, and the Q/K/V weight
    // gradients of a 16-sequence training step 16% faster on 288 wide units
    // of 3 splits than on 960 narrow units of 5.
    const bool split_prefers_wide = auto_split && est_w <= est_n;
    bool wide = d->variant == 3 ||
                (d->variant == 0 && d->N >= 512 && units_w >= (3 * pairs) / 4 &&
                 (kbl >= kWideMinKBlocks || !heavy_epilogue) &&
                 (fill(units_w) >= fill(units_n) - 0.02 || split_prefers_wide));
    const char* env = std::getenv("OXF_GEMM_TILE");
    if (env && d->variant == 0) {
      if (std::strcmp(env, "256") == 0) wide = false;
      if (std::strcmp(env, "512") == 0) wide = d->N >= 512;
    }
    // fused attention products: 256-wide tiles, whose two accumulators let the
    // heavier epilogue (scores) or the 4-warp epilogue (P·V) overlap the MMAs;
    // the transform kernel is instantiated at 256 only
    if (fused) wide = false;
    if (wide) BN = 512;
  }
  p.bm = pair ? 2 * BM : BM;
  p.tiles_m = (d->M + p.bm - 1) / p.bm;
  p.tiles_n = (d->N + BN - 1) / BN;
  // Raster order for L2 reuse. Concurrent tiles share A panels along a
  // tile row and B panels along a tile column. With few column tiles (N up
  // to 16 tiles) walk N fastest, so a handful of row panels and every
  // column panel stay hot; with many, walk M fastest inside groups of 16
  // tile rows. Both measured the lowest DRAM traffic on the transformer's
  // GEMMs (e.g. 2.0 GB vs 3.5 GB for a 32768 x 8192 x 2048 product).
  p.group_m = p.tiles_n <= 16 ? 1 : 16;
  if (const char* g = std::getenv("OXF_GEMM_GROUP_M")) {  // measurement override
    const int v = std::atoi(g);
    if (v >= 1) p.group_m = std::min(v, p.tiles_m);
  }
  p.kblocks_item = (d->K + BK - 1) / BK;
  p.kblocks = p.kblocks_item * (reduce ? d->batch : 1);
  const long long tiles =
      static_cast<long long>(p.tiles_m) * p.tiles_n * (reduce ? 1 : d->batch);
  if (d->accumulate) {
    // Each K split adds its partial product into C, so terms added once per
    // output (bias, residual) rule splitting out.
    const bool additive = d->bias != nullptr || d->residual != nullptr;
    // waves are counted in CTA pairs for pair tiles
    p.splits = split > 1 ? std::min(split, p.kblocks)
                         : (additive ? 1 : choose_splits(tiles, p.kblocks, pair ? sms / 2 : sms));
  } else if (autosplit) {
    p.splits = choose_splits(tiles, p.kblocks, pair ? sms / 2 : sms);
    p.zero_c = p.splits > 1;  // the splits add into C, which starts at zero
  } else {
    p.splits = 1;
  }
  p.units = tiles * p.splits;
  p.units = tiles * p.splits;
  p.bn = BN;
  p.pair = pair;
  // Ring depth and epilogue staging of the kernel the launch picks. A wide
  // tile's epilogue is exposed (one accumulator), so its warps stage through
  // two tiles each, with a ring stage fewer, when the epilogue reads an
  // input tile, writes a pre-activation, adds into C, or has little K to
  // hide behind: a chunk's TMA loads and stores then overlap the previous
  // chunk's. Plain long-K products keep the fourth ring stage (measured 2-4%
  // faster there). On 256-wide tiles the epilogue hides behind the next
  // tile's MMAs, and a second staging tile measured no gain.
  if (fused_transform) {
    p.stages = 6;
    p.staging = 2;
  } else if (split3) {
    p.stages = 3;
  } else if (pair && BN == 512) {
    const bool two_staging = p.kblocks < kWideMinKBlocks || d->accumulate || p.zero_c ||
                             d->residual || d->pre_out || d->aux || d->beta != 0.0f;
    p.stages = two_staging ? 3 : 4;
    p.staging = two_staging ? 2 : 1;
  } else if (pair) {
    p.stages = 6;
  } else {
    p.stages = BN == 256 ? 4 : BN == 128 ? 6 : 8;
  }
  return p;
}

}  // namespace

// Softmax fused into an attention product (the GemmArgs fields of the same
// names): the score product writes row statistics, the P·V product reads
// them and transforms its A operand.
struct GemmFuse {
  float2* stats_out = nullptr;
  const float2* stats_in = nullptr;
  int stats_chunks = 0;
  long long period = 0;
};

oxf_status gemm_run_fused(const oxf_gemm_desc* d, const GemmFuse* fuse, cudaStream_t stream);

oxf_status gemm_run(const oxf_gemm_desc* d, cudaStream_t stream) {
  return gemm_run_fused(d, nullptr, stream);
}

oxf_status gemm_run_fused(const oxf_gemm_desc* d, const GemmFuse* fuse, cudaStream_t stream) {
  const oxf_status valid = gemm_validate(d);
  if (valid != OXF_OK) return valid;
  if (d->M == 0 || d->N == 0) return OXF_OK;
  const int split = d->split_k > 1 ? d->split_k : 1;
  // The fused softmax needs whole tiles on the CTA pair with a TMA epilogue:
  // plain TF32, no accumulation or K split, one output per batch item.
  if (fuse && (d->precision != OXF_PREC_TF32 || d->accumulate || split > 1 ||
               (d->reduce_batch && d->batch > 1) || !gemm_tensor_core_path(d) ||
               (fuse->stats_in && d->a_trans)))
    return set_error(OXF_ERR_UNSUPPORTED_SHAPE, "attention products: no fused form for this shape");

  int dev = 0;
  cudaGetDevice(&dev);

  GemmArgs a{};
  a.M = d->M; a.N = d->N; a.K = d->K; a.batch = d->batch;
  a.a_mn = d->a_trans ? 1 : 0;
  a.b_mn = d->b_trans ? 0 : 1;
  a.C = d->C; a.ldc = d->ldc; a.sc = d->stride_c;
  a.alpha = d->alpha; a.beta = d->beta;
  a.bias = d->bias;
  a.R = d->residual; a.ldr = d->ldr; a.sr = d->stride_r;
  a.P = d->pre_out; a.ldp = d->ldp; a.sp = d->stride_p;
  a.X = d->aux; a.ldx = d->ldx; a.sx = d->stride_x;
  a.act = d->act; a.grad_act = d->aux ? d->grad_act : OXF_ACT_IDENTITY;
  a.accumulate = d->accumulate ? 1 : 0;
  a.reduce_batch = (d->reduce_batch && d->batch > 1) ? 1 : 0;
  if (a.reduce_batch && (d->stride_c || d->stride_r || d->stride_p || d->stride_x))
    return set_error(OXF_ERR_INVALID_ARG,
                     "oxf_gemm: reduce_batch writes one output (output strides must be 0)");
  auto vec = [](const void* p, long long ld, long long st) {
    return p == nullptr || (aligned16(p) && ld % 4 == 0 && st % 4 == 0);
  };
  a.vec_ok = vec(d->C, d->ldc, d->stride_c) && vec(d->residual, d->ldr, d->stride_r) &&
             vec(d->pre_out, d->ldp, d->stride_p) && vec(d->aux, d->ldx, d->stride_x) &&
             (d->bias == nullptr || aligned16(d->bias));

  // TMA needs 16-byte aligned bases, leading dimensions and batch strides.
  // OXF_PREC_F32 asks for f32 products on the CUDA cores: the SIMT kernel.
  const bool tma_ok = gemm_tensor_core_path(d);
  if (!tma_ok) {
    if (a.reduce_batch)
      return set_error(OXF_ERR_UNSUPPORTED_SHAPE,
                       "oxf_gemm: reduce_batch runs on the tensor cores only (16-byte aligned "
                       "operands, TF32 or TF32X3 precision)");
    a.splits = 1;
    if (d->K == 0) {
      // C = epilogue(0): run the SIMT kernel with an empty K loop.
    }
    dim3 grid((d->N + 31) / 32, (d->M + 31) / 32, d->batch);
    gemm_simt_kernel<<<grid, dim3(32, 8), 0, stream>>>(a, d->A, d->lda, d->stride_a, d->B,
                                                        d->ldb, d->stride_b,
                                                        d->precision != OXF_PREC_TF32);
    return check_launch("gemm_simt_kernel");
  }

  // Tiny TF32 products: one memory round trip on the CUDA cores beats the
  // fixed latency of the tensor-core pipeline (variant 0 only).
  if (!fuse && d->variant == 0 && d->precision == OXF_PREC_TF32 && !a.reduce_batch && d->K > 0 &&
      d->K <= SMALL_KMAX &&
      static_cast<double>(d->M) * d->N * d->K * d->batch <= SMALL_MAX_MACS) {
    dim3 grid((d->N + SMALL_TILE - 1) / SMALL_TILE, (d->M + SMALL_TILE - 1) / SMALL_TILE,
              d->batch);
    gemm_small_kernel<<<grid, 256, 0, stream>>>(a, d->A, d->lda, d->stride_a, d->B, d->ldb,
                                                 d->stride_b);
    return check_launch("gemm_small_kernel");
  }

  const bool split3 = d->precision == OXF_PREC_TF32X3;
  const float* A = d->A;
  const float* B = d->B;
  long long lda = d->lda, ldb = d->ldb, sa = d->stride_a, sb = d->stride_b;
  const float *A_lo = nullptr, *B_lo = nullptr;
  if (split3) {
    const size_t need = gemm_workspace_bytes(d);
    if (!d->workspace || d->workspace_bytes < need)
      return set_error(OXF_ERR_INVALID_ARG, "oxf_gemm: TF32X3 needs %zu bytes of workspace",
                       need);
    if (!aligned16(d->workspace))
      return set_error(OXF_ERR_INVALID_ARG, "oxf_gemm: workspace must be 16-byte aligned");
    const long long ba = d->stride_a ? d->batch : 1;
    const long long bb = d->stride_b ? d->batch : 1;
    const long long a_inner = d->a_trans ? d->M : d->K, a_outer = d->a_trans ? d->K : d->M;
    const long long b_inner = d->b_trans ? d->K : d->N, b_outer = d->b_trans ? d->N : d->K;
    auto r = [](long long e) { return ((e * 4 + 255) / 256) * 256; };
    uint8_t* ws = static_cast<uint8_t*>(d->workspace);
    float* a_hi = reinterpret_cast<float*>(ws);
    float* a_lo = reinterpret_cast<float*>(ws + r(a_inner * a_outer * ba));
    float* b_hi = reinterpret_cast<float*>(ws + 2 * r(a_inner * a_outer * ba));
    float* b_lo = reinterpret_cast<float*>(ws + 2 * r(a_inner * a_outer * ba) +
                                           r(b_inner * b_outer * bb));
    const int threads = 256;
    auto blocks = [&](long long e) {
      return static_cast<unsigned>(std::min<long long>((e + threads - 1) / threads, 4096));
    };
    split_tf32_kernel<<<dim3(blocks(a_inner * a_outer), static_cast<unsigned>(ba)), threads, 0,
                        stream>>>(d->A, d->lda, d->stride_a, static_cast<int>(a_inner),
                                  static_cast<int>(a_outer), a_hi, a_lo);
    count_launch();  // the second split launch is counted by check_launch
    split_tf32_kernel<<<dim3(blocks(b_inner * b_outer), static_cast<unsigned>(bb)), threads, 0,
                        stream>>>(d->B, d->ldb, d->stride_b, static_cast<int>(b_inner),
                                  static_cast<int>(b_outer), b_hi, b_lo);
    oxf_status st = check_launch("split_tf32_kernel");
    if (st != OXF_OK) return st;
    A = a_hi; A_lo = a_lo; B = b_hi; B_lo = b_lo;
    lda = a_inner; ldb = b_inner;
    sa = d->stride_a ? a_inner * a_outer : 0;
    sb = d->stride_b ? b_inner * b_outer : 0;
  }

  const int sms = sm_count(dev);
  const GemmPlan plan =
      plan_gemm(d, fuse != nullptr, fuse != nullptr && fuse->stats_in != nullptr, sms);
  const int BN = plan.bn;
  const bool pair = plan.pair;
  a.bm = plan.bm;
  a.tiles_m = plan.tiles_m;
  a.tiles_n = plan.tiles_n;
  a.group_m = plan.group_m;
  a.kblocks_item = plan.kblocks_item;
  a.kblocks = plan.kblocks;
  a.splits = plan.splits;
  a.units = plan.units;
  if (plan.zero_c) {
    oxf_status zs = check_cuda(cudaMemset2DAsync(d->C, static_cast<size_t>(d->ldc) * 4, 0,
                                                 static_cast<size_t>(d->N) * 4,
                                                 static_cast<size_t>(d->M), stream),
                               "oxf_gemm: zeroing C for split K");
    if (zs != OXF_OK) return zs;
    a.accumulate = 1;
  }

  CUtensorMap ta, tb, ta_lo, tb_lo;
  std::memset(&ta_lo, 0, sizeof(ta_lo));
  std::memset(&tb_lo, 0, sizeof(tb_lo));
  int a3d = 0, b3d = 0, dummy = 0;
  const long long a_inner = d->a_trans ? d->M : d->K, a_outer = d->a_trans ? d->K : d->M;
  const long long b_inner = d->b_trans ? d->K : d->N, b_outer = d->b_trans ? d->N : d->K;
  // MN-major tiles whose extent is a multiple of 32 load in one chunked box
  // (box_outer carries the tile rows); otherwise one 32x32 box per chunk.
  a.a_chunked = a.a_mn && (a_inner % 32 == 0) ? 1 : 0;
  a.b_chunked = a.b_mn && (b_inner % 32 == 0) ? 1 : 0;
  const int b_rows = pair ? BN / 2 : BN;  // a CTA of a pair loads half of B
  const int a_box_outer = a.a_mn ? (a.a_chunked ? BM : 32) : BM;
  const int b_box_outer = a.b_mn ? (a.b_chunked ? b_rows : 32) : b_rows;
  const bool amn = a.a_mn != 0, bmn = a.b_mn != 0;
  bool ok =
      encode_map(&ta, A, a_inner, a_outer, lda, d->batch, sa, 32, a_box_outer, amn, &a3d) &&
      encode_map(&tb, B, b_inner, b_outer, ldb, d->batch, sb, 32, b_box_outer, bmn, &b3d);
  if (ok && split3)
    ok = encode_map(&ta_lo, A_lo, a_inner, a_outer, lda, d->batch, sa, 32, a_box_outer, amn,
                    &dummy) &&
         encode_map(&tb_lo, B_lo, b_inner, b_outer, ldb, d->batch, sb, 32, b_box_outer, bmn,
                    &dummy);
  if (!ok) return set_error(OXF_ERR_CUDA, "oxf_gemm: cuTensorMapEncodeTiled failed");
  a.a3d = a3d;
  a.b3d = b3d;

  // Epilogue tiles go through TMA when every epilogue matrix allows a map
  // (16-byte aligned base, leading dimension and batch stride); otherwise
  // each thread accesses its row directly.
  EpiMaps em;
  std::memset(&em, 0, sizeof(em));
  a.epi_tma = vec(d->C, d->ldc, d->stride_c) && vec(d->residual, d->ldr, d->stride_r) &&
              vec(d->pre_out, d->ldp, d->stride_p) && vec(d->aux, d->ldx, d->stride_x);
  if (a.epi_tma) {
    const int eb = a.reduce_batch ? 1 : d->batch;
    bool eok = encode_epi_map(&em.c, d->C, d->N, d->M, d->ldc, eb, d->stride_c, &a.c3d);
    if (eok && d->residual)
      eok = encode_epi_map(&em.r, d->residual, d->N, d->M, d->ldr, eb, d->stride_r, &a.r3d);
    if (eok && d->pre_out)
      eok = encode_epi_map(&em.p, d->pre_out, d->N, d->M, d->ldp, eb, d->stride_p, &a.p3d);
    if (eok && d->aux)
      eok = encode_epi_map(&em.x, d->aux, d->N, d->M, d->ldx, eb, d->stride_x, &a.x3d);
    a.epi_tma = eok ? 1 : 0;
  }
  if (fuse) {
    if (fuse->stats_out && !a.epi_tma)
      return set_error(OXF_ERR_UNSUPPORTED_SHAPE,
                       "attention products: the score epilogue needs TMA-aligned outputs");
    a.stats_out = fuse->stats_out;
    a.stats_in = fuse->stats_in;
    a.stats_chunks = fuse->stats_chunks;
    a.period = fuse->period;
    // four epilogue warps with two staging tiles each: a chunk's residual
    // load and store overlap the previous chunk's store
    if (fuse->stats_in) return launch_pair<256, 6, false, 2, true>(ta, tb, ta, tb, em, a, stream, dev);
  }

  if (split3 && pair)
    return launch_pair<256, 3, true, 1>(ta, tb, ta_lo, tb_lo, em, a, stream, dev);
  if (split3) return launch_tcgen05<128, 3, true>(ta, tb, ta_lo, tb_lo, em, a, stream, dev);
  // wide tiles: ring depth and staging as the plan gives them
  if (pair && BN == 512) {
    if (plan.staging == 2) return launch_pair<512, 3, false, 2>(ta, tb, ta, tb, em, a, stream, dev);
    return launch_pair<512, 4, false, 1>(ta, tb, ta, tb, em, a, stream, dev);
  }
  if (pair) return launch_pair<256, 6, false, 1>(ta, tb, ta, tb, em, a, stream, dev);
  if (BN == 256) return launch_tcgen05<256, 4, false>(ta, tb, ta, tb, em, a, stream, dev);
  if (BN == 128) return launch_tcgen05<128, 6, false>(ta, tb, ta, tb, em, a, stream, dev);
  return launch_tcgen05<64, 8, false>(ta, tb, ta, tb, em, a, stream, dev);
}

// ---------------------------------------------------------------- attention
oxf_status rows_softmax(float*, long long, long long, float, long long, cudaStream_t);

// Between the two attention products: for every score row, the row maximum
// and sum over its chunk statistics (chunk-major, (m_c, l_c)), then each
// chunk's factor exp(m_c - max) / sum written over m_c (0 for a chunk with
// no unmasked column). One thread per row; consecutive threads take
// consecutive rows, so every chunk's loads and stores are coalesced.
__global__ void __launch_bounds__(256) softmax_stats_finalize_kernel(float2* __restrict__ stats,
                                                                   int batch, long long M,
                                                                   int chunks) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(batch) * M) return;
  const long long b = i / M, m = i - b * M;
  float2* st = stats + b * chunks * M + m;
  float mx = -INFINITY, l = 0.0f;
#pragma unroll 8
  for (int c = 0; c < chunks; ++c) {  // online: rescale the sum as the maximum grows
    const float2 e = st[c * M];
    if (e.x == -INFINITY) continue;
    const float nm = fmaxf(mx, e.x);
    l = l * __expf(mx - nm) + e.y * __expf(e.x - nm);
    mx = nm;
  }
  const float inv = 1.0f / l;
#pragma unroll 8
  for (int c = 0; c < chunks; ++c) {
    float2 e = st[c * M];
    e.x = e.x == -INFINITY ? 0.0f : __expf(e.x - mx) * inv;
    st[c * M] = e;
  }
}

// Row-statistics entries per score row: one per 32-column chunk.
long long attention_stats_parts(long long seq) { return (seq + 31) / 32; }

// out = residual + softmax(scale * Q·Kᵀ [causal]) · V for `batch` independent
// sequences (Attention::forward's scaled dot-product part,
// src/net/transformer/attention.rs:243-253, 359-401). Q, K: [batch][seq][dqk],
// V, residual, out: [batch][seq][dv], scores: [batch][seq][seq] workspace,
// stats: attention_stats_parts(seq) float2 per score row.
//
// Fused form (OXF_ATTENTION=fused): the score product's epilogue writes,
// per 32-column chunk of a row, E = exp(s - chunk max) and the chunk's
// (max, sum of E); a small
// kernel turns each row's chunk statistics into the factors exp(chunk max -
// row max) / row sum; the P·V product loads E as its A operand (one chunk
// per K block) and scales each A tile row by its factor in shared memory
// before the tensor cores read it. P is never written, and no softmax pass
// over the S x S matrix runs. Otherwise, and for shapes the fused kernels
// cannot take (rows not 16-byte aligned), the three-launch form runs:
// scores, softmax in place, P·V; scores then holds P.
oxf_status attention_forward(const float* q, const float* k, const float* v, const float* residual,
                             float* out, float* scores, float* stats, int batch, int seq, int dqk,
                             int dv, float scale, int causal, cudaStream_t stream) {
  if (batch < 0 || seq < 0 || dqk < 0 || dv < 0)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_attention_forward: negative shape");
  if (batch == 0 || seq == 0 || dv == 0) return OXF_OK;
  if (!q || !k || !v || !out || !scores || (dqk > 0 && !stats))
    return set_error(OXF_ERR_INVALID_ARG, "oxf_attention_forward: null pointer");
  const long long sSS = static_cast<long long>(seq) * seq;
  const long long sQ = static_cast<long long>(seq) * dqk, sV = static_cast<long long>(seq) * dv;
  oxf_gemm_desc s;
  oxf_gemm_desc_init(&s, seq, seq, dqk, 0, 1, q, k, scores);
  s.batch = batch;
  s.stride_a = sQ;
  s.stride_b = sQ;
  s.stride_c = sSS;
  s.alpha = scale;
  oxf_gemm_desc pv;
  oxf_gemm_desc_init(&pv, seq, dv, seq, 0, 0, scores, v, out);
  pv.batch = batch;
  pv.stride_a = sSS;
  pv.stride_b = sV;
  pv.stride_c = sV;
  if (residual) {
    pv.residual = residual;
    pv.ldr = dv;
    pv.stride_r = sV;
  }
  // The fused form is chosen with OXF_ATTENTION=fused (read at every call).
  // Measured on B200 at config 4's widths (64 x [2048, 1024]) it takes 3.5 ms
  // against 2.2 ms for the three launches: the in-place rewrite of each A
  // tile adds a third stream of shared-memory traffic beside the TMA writes
  // and the TF32 MMA reads, and the partner CTA signals every stage with a
  // cluster-scope release. The three-launch form is therefore the default.
  const char* env = std::getenv("OXF_ATTENTION");
  const bool want_fused = env && std::strcmp(env, "fused") == 0;
  const bool fusable = want_fused && seq % 4 == 0 && dqk % 4 == 0 && dv % 4 == 0 && dqk > 0 &&
                       aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out) &&
                       aligned16(scores) && (!residual || aligned16(residual)) &&
                       (reinterpret_cast<uintptr_t>(stats) & 7) == 0;
  bool have_scores = false;
  if (fusable) {
    GemmFuse f1;
    f1.stats_out = reinterpret_cast<float2*>(stats);
    f1.stats_chunks = static_cast<int>(attention_stats_parts(seq));
    f1.period = causal ? seq : 0;
    oxf_status st = gemm_run_fused(&s, &f1, stream);
    if (st != OXF_OK && st != OXF_ERR_UNSUPPORTED_SHAPE) return st;
    if (st == OXF_OK) {
      const long long rows = static_cast<long long>(batch) * seq;
      softmax_stats_finalize_kernel<<<static_cast<unsigned>((rows + 255) / 256), 256, 0, stream>>>(
          reinterpret_cast<float2*>(stats), batch, seq, f1.stats_chunks);
      st = check_launch("softmax_stats_finalize_kernel");
      if (st != OXF_OK) return st;
      GemmFuse f2;
      f2.stats_in = reinterpret_cast<const float2*>(stats);
      f2.stats_chunks = f1.stats_chunks;
      f2.period = f1.period;
      st = gemm_run_fused(&pv, &f2, stream);
      if (st != OXF_ERR_UNSUPPORTED_SHAPE) return st;
      have_scores = true;  // S is written: normalise it below
    }
  }
  oxf_status st = have_scores ? OXF_OK : gemm_run(&s, stream);
  if (st != OXF_OK) return st;
  st = rows_softmax(scores, static_cast<long long>(batch) * seq, seq, 1.0f, causal ? seq : 0,
                    stream);
  if (st != OXF_OK) return st;
  return gemm_run(&pv, stream);
}

// The path and kernel oxf_gemm takes for a descriptor, as gemm_run_fused
// decides it (without fusion); sms <= 0 asks the current device.
oxf_status gemm_plan_report(const oxf_gemm_desc* d, int sms, oxf_gemm_plan_info* out) {
  if (!out) return set_error(OXF_ERR_INVALID_ARG, "oxf_gemm_plan: null output");
  std::memset(out, 0, sizeof(*out));
  const oxf_status valid = gemm_validate(d);
  if (valid != OXF_OK) return valid;
  if (d->M == 0 || d->N == 0) return OXF_OK;  // OXF_GEMM_PATH_NONE
  const bool reduce = d->reduce_batch && d->batch > 1;
  if (reduce && (d->stride_c || d->stride_r || d->stride_p || d->stride_x))
    return set_error(OXF_ERR_INVALID_ARG,
                     "oxf_gemm: reduce_batch writes one output (output strides must be 0)");
  if (!gemm_tensor_core_path(d)) {
    if (reduce)
      return set_error(OXF_ERR_UNSUPPORTED_SHAPE,
                       "oxf_gemm: reduce_batch runs on the tensor cores only (16-byte aligned "
                       "operands, TF32 or TF32X3 precision)");
    out->path = OXF_GEMM_PATH_SIMT;
    out->tile_m = out->tile_n = 32;
    out->splits = 1;
    out->units = static_cast<long long>((d->M + 31) / 32) * ((d->N + 31) / 32) * d->batch;
    return OXF_OK;
  }
  if (d->variant == 0 && d->precision == OXF_PREC_TF32 && !reduce && d->K <= SMALL_KMAX &&
      static_cast<double>(d->M) * d->N * d->K * d->batch <= SMALL_MAX_MACS) {
    out->path = OXF_GEMM_PATH_TINY;
    out->tile_m = out->tile_n = SMALL_TILE;
    out->splits = 1;
    out->units = static_cast<long long>((d->M + SMALL_TILE - 1) / SMALL_TILE) *
                 ((d->N + SMALL_TILE - 1) / SMALL_TILE) * d->batch;
    return OXF_OK;
  }
  if (sms <= 0) {
    int dev = 0;
    const oxf_status st = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (st != OXF_OK) return st;
    sms = sm_count(dev);
  }
  const GemmPlan p = plan_gemm(d, false, false, sms);
  out->path = p.pair ? OXF_GEMM_PATH_CTA_PAIR : OXF_GEMM_PATH_ONE_CTA;
  out->tile_m = p.bm;
  out->tile_n = p.bn;
  out->stages = p.stages;
  out->staging = p.staging;
  out->splits = p.splits;
  out->group_m = p.group_m;
  out->zero_c = p.zero_c ? 1 : 0;
  out->units = p.units;
  return OXF_OK;
}

// ---------------------------------------------------------------- no-allocation variant
// Some callers cannot call cudaMalloc: plugin hosts that own the whole device
// memory budget through their own allocator and forbid allocations from
// libraries, and latency-critical paths that must not pay for cudaMalloc's
// implicit device synchronisation. For them the 3xTF32 GEMM can take its
// hi/lo operand splits from this fixed array instead of a caller workspace.
// It is a file-scope device array, so every GPU that loads this library
// holds these 16 MiB until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

oxf_status gemm_tf32x3_noalloc(const oxf_gemm_desc* d, cudaStream_t stream) {
  // The same checks and errors as oxf_gemm, before anything is sized.
  const oxf_status valid = gemm_validate(d);
  if (valid != OXF_OK) return valid;
  if (d->M == 0 || d->N == 0) return OXF_OK;
  oxf_gemm_desc desc = *d;
  desc.precision = OXF_PREC_TF32X3;
  desc.workspace = nullptr;
  desc.workspace_bytes = 0;
  // Operands the tensor cores cannot read (misaligned, or K = 0) take the
  // SIMT kernel, which splits nothing: no scratch, no size limit.
  if (!gemm_tensor_core_path(&desc)) return gemm_run(&desc, stream);
  const size_t need = gemm_workspace_bytes(&desc);
  if (need > kNoAllocScratchBytes)
    return set_error(OXF_ERR_UNSUPPORTED_SHAPE,
                     "oxf_gemm_tf32x3_noalloc: this shape needs %zu bytes of operand splits, "
                     "the static scratch holds %zu (16 MiB); use oxf_gemm with a workspace",
                     need, kNoAllocScratchBytes);
  int dev = 0;
  oxf_status st = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (st != OXF_OK) return st;
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(OXF_ERR_UNSUPPORTED_SHAPE, "oxf_gemm_tf32x3_noalloc: device ordinal %d", dev);
  // In host code the array's name only stands in for it; its device address
  // is looked up with the device current, on the first call there and again
  // after a device reset (a new context has a new address). The lookup may
  // load this library's module, which a stream capture would not allow, so
  // a lookup that falls inside a capture is refused.
  static std::mutex mu;
  static void* scratch[kMaxDevices] = {nullptr};
  static unsigned long long ctx_of[kMaxDevices] = {0};
  void* ptr = nullptr;
  {
    std::lock_guard<std::mutex> lock(mu);
    const unsigned long long ctx = current_context_id();
    if (!scratch[dev] || (ctx != 0 && ctx != ctx_of[dev])) {
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      st = check_cuda(cudaStreamIsCapturing(stream, &cs), "cudaStreamIsCapturing");
      if (st != OXF_OK) return st;
      if (cs != cudaStreamCaptureStatusNone)
        return set_error(OXF_ERR_INVALID_ARG,
                         "oxf_gemm_tf32x3_noalloc: the first call on a device (and the first "
                         "after a device reset) must come before any stream capture");
      void* p = nullptr;
      st = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                      "cudaGetSymbolAddress(no-alloc scratch)");
      if (st != OXF_OK) return st;
      scratch[dev] = p;
      ctx_of[dev] = current_context_id();
    }
    ptr = scratch[dev];
  }
  // Nothing in the scratch needs to start at zero: the split kernels write
  // every element the GEMM then reads (TMA zero-fills reads past the edges).
  desc.workspace = ptr;
  desc.workspace_bytes = kNoAllocScratchBytes;
  return gemm_run(&desc, stream);
}

oxf_status gemm_refalgo(const float* A, const float* B, float* C, size_t len, size_t rows,
                        size_t cols, cudaStream_t stream) {
  if (rows % 16 || cols % 16 || len % 16)
    return set_error(OXF_ERR_INVALID_ARG,
                     "matrix_multiply_refalgo: rows, cols and len must be multiples of 16");
  if (rows == 0 || cols == 0) return OXF_OK;
  dim3 grid(static_cast<unsigned>((cols + 31) / 32), static_cast<unsigned>((rows + 31) / 32));
  gemm_refalgo_kernel<<<grid, 128, 0, stream>>>(A, B, C, static_cast<int>(len),
                                                static_cast<int>(rows), static_cast<int>(cols));
  return check_launch("gemm_refalgo_kernel");
}

// Failure-detection self-test: one thread waits on an mbarrier that nothing
// arrives at, with a short bound, so the wait expires exactly as a stalled
// pipeline's would: it records DEVERR_WAIT_SELFTEST in the device error
// word and returns. Nothing hangs and nothing faults; the context stays
// usable.
__global__ void wait_selftest_kernel(unsigned long long limit_ns, int* waited) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_barrier_init();
  const bool ok = mbar_wait(&bar, 0, DEVERR_WAIT_SELFTEST, limit_ns);
  *waited = ok ? 0 : 1;
}

oxf_status wait_selftest(unsigned long long limit_ns, int* waited, cudaStream_t stream) {
  wait_selftest_kernel<<<1, 32, 0, stream>>>(limit_ns, waited);
  return check_launch("wait_selftest_kernel");
}

oxf_status gemm_read_device_error(uint32_t* code) {
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
