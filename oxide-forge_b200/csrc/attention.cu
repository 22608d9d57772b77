// attention.cu — fused multi-head attention forward on tcgen05
// (oxf_attention_heads_forward): per 128-row query tile, the scores stay in
// TMEM, the softmax runs online in registers, and P·V accumulates in TMEM.
// The single-head attention of the reference (three launches, or the GEMM
// kernels with the softmax fused into their epilogue and operand path) is in
// gemm.cu.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "ptx.cuh"
#include "status.cuh"
#include "tmap.hpp"
#include "umma.cuh"

namespace oxf {

// ---------------------------------------------------------------- fused multi-head attention
// Multi-head attention forward in one kernel, FlashAttention-style: for a
// 128-row query tile of one head of one sequence, the scores of each
// 128-row key/value tile go to TMEM, the softmax runs online in registers
// (running row maximum and sum, the accumulated output rescaled when the
// maximum grows), the probabilities are written to shared memory as the A
// operand of the P·V product, and the output accumulates in TMEM. The S x S
// score matrix never reaches HBM. Head j reads columns [j*HD, (j+1)*HD) of
// Q, K and V; out = residual + softmax(Q_j K_jᵀ / sqrt(HD)) V_j in the same
// columns (attention.rs:359-401 per head; docs/api.md:440-442 anticipates the
// head split). Warp 0 issues the TMA loads, warp 1 the MMAs, warps 2-9 run
// the softmax, two threads per query row. Every wait is bounded.
constexpr int FA_ROWS = 128;
constexpr float FA_RESCALE = 8.0f;  // see the softmax: lazy output rescaling
constexpr int FA_SOFTMAX_WARPS = 8;
constexpr int FA_THREADS = 64 + 32 * FA_SOFTMAX_WARPS;

struct FaArgs {
  float* out;             // [batch * seq, ldo]
  const float* residual;  // the same layout, or null
  long long ldo;
  int seq, tiles;         // tiles = seq / 128
  int causal;
  float scale;            // 1 / sqrt(HD)
};

template <int HD>
struct FaCfg {
  static constexpr int KB = HD / 32;                    // 32-column blocks of a Q / K row
  static constexpr int Q_BYTES = KB * 16384;            // [128 x HD], K-major, 128B swizzle
  static constexpr int K_BYTES = KB * 16384;            // [128 keys x HD], K-major
  static constexpr int V_KBLOCK = (HD / 32) * 4096;     // 32 keys x HD, MN-major
  static constexpr int V_BYTES = 4 * V_KBLOCK;          // 128 keys
  static constexpr int STAGES = HD == 32 ? 6 : 3;       // K / V ring depth
  static constexpr int CTRL_BYTES = 2048;               // barriers; row-sum exchange at 1024
  static constexpr int SMEM_BYTES = 1024 + CTRL_BYTES + Q_BYTES + STAGES * (K_BYTES + V_BYTES);
  static constexpr uint32_t TMEM_COLS = 512;            // S / P x 2 (256 columns) + O (HD)
  static constexpr uint32_t O_COL = 256;
  static constexpr uint32_t X_COL = 448;                // row-maximum exchange, 4 columns
  static_assert(HD == 32 || HD == 64, "head widths 32 and 64");
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};

constexpr int FA_MAX_STAGES = 6;

struct FaCtrl {
  uint64_t q_full;
  uint64_t k_full[FA_MAX_STAGES], k_empty[FA_MAX_STAGES];  // K ring: S products release
  uint64_t v_full[FA_MAX_STAGES], v_empty[FA_MAX_STAGES];  // V ring: P·V products release
  uint64_t s_full[2];   // S landed in TMEM buffer b
  uint64_t s_read[2];   // every softmax warp has posted its half-row maxima of buffer b
  uint64_t s_free[2];   // the P·V that read buffer b has finished
  uint64_t p_ready;     // P of the tile in TMEM, O rescaled
  uint64_t pv_done;     // the tile's P·V has finished
  uint32_t tmem_base;
  int abort_flag;
};

template <int HD>
__global__ void __launch_bounds__(FA_THREADS, 1)
    attention_heads_flash_kernel(const __grid_constant__ CUtensorMap tmQ,
                                 const __grid_constant__ CUtensorMap tmK,
                                 const __grid_constant__ CUtensorMap tmV, const FaArgs args) {
  using Cfg = FaCfg<HD>;
  constexpr int NS = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t fa_smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fa_smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  auto* ctrl = reinterpret_cast<FaCtrl*>(base);
  float* lsum = reinterpret_cast<float*>(base + 1024);  // [2][128] row-sum halves
  uint8_t* qs = base + Cfg::CTRL_BYTES;
  uint8_t* ks = qs + Cfg::Q_BYTES;       // NS stages
  uint8_t* vs = ks + NS * Cfg::K_BYTES;  // NS stages

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, head = blockIdx.y, seq_i = blockIdx.z;
  const int n_tiles = args.causal ? qt + 1 : args.tiles;
  const int q_row0 = seq_i * args.seq + qt * FA_ROWS;  // first query row of the tile
  const int kv_row0 = seq_i * args.seq;
  const int col0 = head * HD;

  if (threadIdx.x == 0) {
    mbar_init(&ctrl->q_full, 1);
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      mbar_init(&ctrl->k_full[s], 1);
      mbar_init(&ctrl->k_empty[s], 1);
      mbar_init(&ctrl->v_full[s], 1);
      mbar_init(&ctrl->v_empty[s], 1);
    }
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      mbar_init(&ctrl->s_full[s], 1);
      mbar_init(&ctrl->s_read[s], FA_SOFTMAX_WARPS);
      mbar_init(&ctrl->s_free[s], 1);
    }
    mbar_init(&ctrl->p_ready, FA_SOFTMAX_WARPS);
    mbar_init(&ctrl->pv_done, 1);
    ctrl->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(&ctrl->tmem_base, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctrl->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = make_l2_policy(L2_NORMAL);
      mbar_arrive_expect_tx(&ctrl->q_full, Cfg::Q_BYTES);
#pragma unroll
      for (int kb = 0; kb < Cfg::KB; ++kb)
        tma_load_2d(qs + kb * 16384, &tmQ, &ctrl->q_full, col0 + kb * 32, q_row0, pol);
      int kfills = 0, vfills = 0;  // tiles whose K / V loads were issued
      for (int t = 0; t < n_tiles && !ctrl->abort_flag; ++t) {
        const int st = t % NS;
        const uint32_t prev = static_cast<uint32_t>((t / NS - 1) & 1);
        const int kv0 = kv_row0 + t * FA_ROWS;
        if (t >= NS && !mbar_wait(&ctrl->k_empty[st], prev, DEVERR_ATTN_WAIT)) {
          ctrl->abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&ctrl->k_full[st], Cfg::K_BYTES);
#pragma unroll
        for (int kb = 0; kb < Cfg::KB; ++kb)
          tma_load_2d(ks + st * Cfg::K_BYTES + kb * 16384, &tmK, &ctrl->k_full[st],
                      col0 + kb * 32, kv0, pol);
        kfills = t + 1;
        if (t >= NS && !mbar_wait(&ctrl->v_empty[st], prev, DEVERR_ATTN_WAIT)) {
          ctrl->abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&ctrl->v_full[st], Cfg::V_BYTES);
#pragma unroll
        for (int kb = 0; kb < 4; ++kb)
          load_operand<HD>(vs + st * Cfg::V_BYTES + kb * Cfg::V_KBLOCK, &tmV, &ctrl->v_full[st],
                           1, 0, HD > 32 ? 1 : 0, col0, kv0 + kb * 32, 0, pol);
        vfills = t + 1;
      }
      // no copy may still be landing when the CTA exits
      mbar_wait(&ctrl->q_full, 0, DEVERR_ATTN_WAIT);
      for (int t = kfills > NS ? kfills - NS : 0; t < kfills; ++t)
        mbar_wait(&ctrl->k_full[t % NS], (t / NS) & 1, DEVERR_ATTN_WAIT);
      for (int t = vfills > NS ? vfills - NS : 0; t < vfills; ++t)
        mbar_wait(&ctrl->v_full[t % NS], (t / NS) & 1, DEVERR_ATTN_WAIT);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = make_idesc_tf32(128, 128, false, false);
      constexpr uint32_t id_o = make_idesc_tf32(128, HD, false, true);
      const uint32_t q_addr = smem_u32(qs), k_addr = smem_u32(ks), v_addr = smem_u32(vs);
      // O += P·V for tile t: P is read from TMEM (it overwrote the tile's S)
      auto issue_pv = [&](int t) -> bool {
        const int st = t % NS;
        if (!mbar_wait(&ctrl->p_ready, t & 1, DEVERR_ATTN_WAIT) ||
            !mbar_wait(&ctrl->v_full[st], (t / NS) & 1, DEVERR_ATTN_WAIT))
          return false;
        tc_fence_after();
        const uint32_t p_col = tmem + static_cast<uint32_t>((t & 1) * 128);
#pragma unroll
        for (int kb = 0; kb < 4; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_tf32_tmem_a(tmem + Cfg::O_COL, p_col + kb * 32 + kk * 8,
                             desc_advance(operand_desc(v_addr + st * Cfg::V_BYTES +
                                                           kb * Cfg::V_KBLOCK,
                                                       1, 0),
                                          kk * 1024),
                             id_o, (t > 0 || kb > 0 || kk > 0) ? 1u : 0u);
        // releases first: once pv_done completes, no arrive is pending
        umma_commit(&ctrl->v_empty[st]);
        umma_commit(&ctrl->s_free[t & 1]);
        umma_commit(&ctrl->pv_done);
        return true;
      };
      bool ok = mbar_wait(&ctrl->q_full, 0, DEVERR_ATTN_WAIT);
      for (int t = 0; ok && t < n_tiles; ++t) {
        const int st = t % NS, sb = t & 1;
        ok = mbar_wait(&ctrl->k_full[st], (t / NS) & 1, DEVERR_ATTN_WAIT) &&
             (t < 2 || mbar_wait(&ctrl->s_free[sb], ((t - 2) >> 1) & 1, DEVERR_ATTN_WAIT));
        if (!ok) break;
        tc_fence_after();
        // S[sb] = Q·K_tᵀ (the scale is applied in the softmax)
#pragma unroll
        for (int kb = 0; kb < Cfg::KB; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_tf32(tmem + sb * 128,
                      desc_advance(operand_desc(q_addr + kb * 16384, 0, 0), kk * 32),
                      desc_advance(operand_desc(k_addr + st * Cfg::K_BYTES + kb * 16384, 0, 0),
                                   kk * 32),
                      id_s, (kb > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&ctrl->k_empty[st]);
        umma_commit(&ctrl->s_full[sb]);
        // the previous tile's P·V runs while the softmax works on this one
        if (t > 0) ok = issue_pv(t - 1);
      }
      if (ok) ok = issue_pv(n_tiles - 1);
      if (!ok) ctrl->abort_flag = 1;
    }
  } else {
    // Softmax: two threads per query row r (= TMEM lane r). Warps 2-5 own
    // keys 0-63 of every tile, warps 6-9 keys 64-127; the two threads of a
    // row exchange their half-row maxima, then each exponentiates its own 64
    // keys, writes their probabilities over its scores in TMEM (the A
    // operand of P·V), rescales its 32-column chunk of the output, and
    // finally normalises and stores that chunk.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t row_tmem = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const float scale2 = args.scale * 1.4426950408889634f;  // exp(s * scale) = 2^(s * scale2)
    const bool own_o = half < HD / 32;  // HD = 32: one chunk, owned by half 0
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int t = 0; t < n_tiles; ++t) {
      const int sb = t & 1;
      if (!mbar_wait(&ctrl->s_full[sb], (t >> 1) & 1, DEVERR_ATTN_WAIT)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t s_row = row_tmem + sb * 128;
      // on the diagonal tile of a causal pass, key j > row r is masked
      const bool diag = args.causal && t == qt;
      float v[2][32];
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int kc = half * 2 + c;
        tmem_ld_32x32b_x32(s_row + kc * 32, v[c]);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (diag && kc * 32 + j > r) v[c][j] = -INFINITY;
          mx[j & 3] = fmaxf(mx[j & 3], v[c][j]);
        }
      }
      // the row maximum: this half's, exchanged with the partner thread
      // through a spare TMEM column per (buffer, half)
      const float mine = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      tmem_st_32x32b_x1(row_tmem + Cfg::X_COL + sb * 2 + half, mine);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctrl->s_read[sb]);
      if (!mbar_wait(&ctrl->s_read[sb], (t >> 1) & 1, DEVERR_ATTN_WAIT)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float mt = fmaxf(mine, tmem_ld_32x32b_x1(row_tmem + Cfg::X_COL + sb * 2 + (1 - half)));
      // The exponent reference m moves only when the tile's maximum exceeds it
      // by more than FA_RESCALE (log2 units): probabilities then stay <= 2^8,
      // and the output rescale below is skipped on most tiles. O / l does not
      // depend on the reference.
      const float mts = mt * scale2;  // scale2 > 0
      const float m_new = mts > m + FA_RESCALE ? mts : m;
      const float alpha = ex2_approx(m - m_new);  // 1 if kept; 0 on the first tile
      float sm[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float p = ex2_approx(fmaf(v[c][j], scale2, -m_new));
          v[c][j] = p;
          sm[j & 3] += p;
        }
      l = l * alpha + ((sm[0] + sm[1]) + (sm[2] + sm[3]));
      m = m_new;
      if (t > 0) {
        // the previous P·V has finished: O holds tiles 0..t-1
        if (!mbar_wait(&ctrl->pv_done, (t - 1) & 1, DEVERR_ATTN_WAIT)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (own_o && __any_sync(0xffffffffu, alpha != 1.0f)) {
          float o[32];
          tmem_ld_32x32b_x32(row_tmem + Cfg::O_COL + half * 32, o);
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] *= alpha;
          tmem_st_32x32b_x32(row_tmem + Cfg::O_COL + half * 32, o);
        }
      }
      // this half's probabilities over its own scores
#pragma unroll
      for (int c = 0; c < 2; ++c) tmem_st_32x32b_x32(s_row + (half * 2 + c) * 32, v[c]);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctrl->p_ready);
    }
    if (ok) ok = mbar_wait(&ctrl->pv_done, (n_tiles - 1) & 1, DEVERR_ATTN_WAIT);
    if (!ok) ctrl->abort_flag = 1;
    // the row sum is split over the two halves; the named barrier is reached
    // by all eight softmax warps on every path
    lsum[half * FA_ROWS + r] = l;
    asm volatile("bar.sync 1, %0;" ::"r"(32 * FA_SOFTMAX_WARPS) : "memory");
    l += lsum[(1 - half) * FA_ROWS + r];
    if (ok && own_o) {
      tc_fence_after();
      const float inv = 1.0f / l;
      const long long row = q_row0 + r;
      float* orow = args.out + row * args.ldo + col0 + half * 32;
      const float* rrow =
          args.residual ? args.residual + row * args.ldo + col0 + half * 32 : nullptr;
      float o[32];
      tmem_ld_32x32b_x32(row_tmem + Cfg::O_COL + half * 32, o);
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 y = make_float4(o[j] * inv, o[j + 1] * inv, o[j + 2] * inv, o[j + 3] * inv);
        if (rrow) {
          const float4 x = *reinterpret_cast<const float4*>(rrow + j);
          y.x += x.x; y.y += x.y; y.z += x.z; y.w += x.w;
        }
        *reinterpret_cast<float4*>(orow + j) = y;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// Two query tiles per CTA (rows 256*i .. 256*i+255 of one head of one
// sequence), so that the tensor cores work on one tile's products while the
// other tile's softmax runs. Each query tile has its own score buffer (128
// TMEM columns), output accumulator and group of four softmax warps (one
// thread per row); the probabilities of both tiles pass through one shared
// 128-column P buffer. A tile's next scores S(t+1) are issued as soon as its
// softmax has loaded S(t) into registers, so they overlap that softmax's
// exponentials instead of waiting for its P·V; P·V of one tile reads the P
// buffer while the other tile's softmax computes, and a softmax writes P
// once the previous P·V (in issue order: A(t), B(t), A(t+1), ...) has read
// it. Per key/value tile t the MMA thread issues S_A(t+1), S_B(t+1),
// P·V_A(t), P·V_B(t). K and V are loaded once for both tiles.
constexpr int FA2_THREADS = 64 + 32 * 8;

template <int HD>
struct Fa2Cfg {
  static constexpr int KB = HD / 32;
  static constexpr int Q_BYTES = KB * 16384;            // one query tile, K-major
  static constexpr int K_BYTES = KB * 16384;
  static constexpr int V_KBLOCK = (HD / 32) * 4096;
  static constexpr int V_BYTES = 4 * V_KBLOCK;
  static constexpr int STAGES = HD == 32 ? 6 : 2;
  static constexpr int CTRL_BYTES = 2048;
  static constexpr int SMEM_BYTES =
      1024 + CTRL_BYTES + 2 * Q_BYTES + STAGES * (K_BYTES + V_BYTES);
  static constexpr uint32_t TMEM_COLS = 512;  // S_A 0, S_B 128, P 256, O_A 384, O_B 384 + HD
  static constexpr uint32_t P_COL = 256;
  static constexpr uint32_t O_COL = 384;
  static_assert(HD == 32 || HD == 64, "head widths 32 and 64");
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};

struct Fa2Ctrl {
  uint64_t q_full;
  uint64_t k_full[FA_MAX_STAGES], k_empty[FA_MAX_STAGES];
  uint64_t v_full[FA_MAX_STAGES], v_empty[FA_MAX_STAGES];
  uint64_t s_full[2];   // per query tile: S landed
  uint64_t s_read[2];   // per query tile: its softmax holds S in registers (S may be overwritten)
  uint64_t p_ready[2];  // per query tile: P in the shared P buffer, O rescaled
  uint64_t pv_done[2];  // per query tile: P·V finished (O final for t, P buffer read)
  uint32_t tmem_base;
  int abort_flag;
};

template <int HD>
__global__ void __launch_bounds__(FA2_THREADS, 1)
    attention_heads_flash2_kernel(const __grid_constant__ CUtensorMap tmQ,
                                  const __grid_constant__ CUtensorMap tmK,
                                  const __grid_constant__ CUtensorMap tmV, const FaArgs args) {
  using Cfg = Fa2Cfg<HD>;
  constexpr int NS = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t fa2_smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fa2_smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  auto* ctrl = reinterpret_cast<Fa2Ctrl*>(base);
  uint8_t* qs = base + Cfg::CTRL_BYTES;  // tile A, then tile B
  uint8_t* ks = qs + 2 * Cfg::Q_BYTES;
  uint8_t* vs = ks + NS * Cfg::K_BYTES;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pair = blockIdx.x, head = blockIdx.y, seq_i = blockIdx.z;
  const int qa = 2 * pair;  // query tile index of A (B is qa + 1)
  // key/value tiles each query tile visits; causal: up to its diagonal
  const int n_a = args.causal ? qa + 1 : args.tiles;
  const int n_b = args.causal ? qa + 2 : args.tiles;
  const int q_row0 = seq_i * args.seq + qa * FA_ROWS;
  const int kv_row0 = seq_i * args.seq;
  const int col0 = head * HD;

  if (threadIdx.x == 0) {
    mbar_init(&ctrl->q_full, 1);
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      mbar_init(&ctrl->k_full[s], 1);
      mbar_init(&ctrl->k_empty[s], 1);
      mbar_init(&ctrl->v_full[s], 1);
      mbar_init(&ctrl->v_empty[s], 1);
    }
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      mbar_init(&ctrl->s_full[g], 1);
      mbar_init(&ctrl->s_read[g], 4);
      mbar_init(&ctrl->p_ready[g], 4);
      mbar_init(&ctrl->pv_done[g], 1);
    }
    ctrl->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(&ctrl->tmem_base, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctrl->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = make_l2_policy(L2_NORMAL);
      mbar_arrive_expect_tx(&ctrl->q_full, 2 * Cfg::Q_BYTES);
#pragma unroll
      for (int g = 0; g < 2; ++g)
#pragma unroll
        for (int kb = 0; kb < Cfg::KB; ++kb)
          tma_load_2d(qs + g * Cfg::Q_BYTES + kb * 16384, &tmQ, &ctrl->q_full, col0 + kb * 32,
                      q_row0 + g * FA_ROWS, pol);
      int kfills = 0, vfills = 0;
      for (int t = 0; t < n_b && !ctrl->abort_flag; ++t) {
        const int st = t % NS;
        const uint32_t prev = static_cast<uint32_t>((t / NS - 1) & 1);
        const int kv0 = kv_row0 + t * FA_ROWS;
        if (t >= NS && !mbar_wait(&ctrl->k_empty[st], prev, DEVERR_ATTN_WAIT)) {
          ctrl->abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&ctrl->k_full[st], Cfg::K_BYTES);
#pragma unroll
        for (int kb = 0; kb < Cfg::KB; ++kb)
          tma_load_2d(ks + st * Cfg::K_BYTES + kb * 16384, &tmK, &ctrl->k_full[st],
                      col0 + kb * 32, kv0, pol);
        kfills = t + 1;
        if (t >= NS && !mbar_wait(&ctrl->v_empty[st], prev, DEVERR_ATTN_WAIT)) {
          ctrl->abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&ctrl->v_full[st], Cfg::V_BYTES);
#pragma unroll
        for (int kb = 0; kb < 4; ++kb)
          load_operand<HD>(vs + st * Cfg::V_BYTES + kb * Cfg::V_KBLOCK, &tmV, &ctrl->v_full[st],
                           1, 0, HD > 32 ? 1 : 0, col0, kv0 + kb * 32, 0, pol);
        vfills = t + 1;
      }
      // no copy may still be landing when the CTA exits
      mbar_wait(&ctrl->q_full, 0, DEVERR_ATTN_WAIT);
      for (int t = kfills > NS ? kfills - NS : 0; t < kfills; ++t)
        mbar_wait(&ctrl->k_full[t % NS], (t / NS) & 1, DEVERR_ATTN_WAIT);
      for (int t = vfills > NS ? vfills - NS : 0; t < vfills; ++t)
        mbar_wait(&ctrl->v_full[t % NS], (t / NS) & 1, DEVERR_ATTN_WAIT);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = make_idesc_tf32(128, 128, false, false);
      constexpr uint32_t id_o = make_idesc_tf32(128, HD, false, true);
      const uint32_t q_addr = smem_u32(qs), k_addr = smem_u32(ks), v_addr = smem_u32(vs);
      // S_g = Q_g · K_tᵀ into tile g's buffer, once its softmax holds S_g(t-1)
      auto issue_s = [&](int g, int t) -> bool {
        if (t > 0 && !mbar_wait(&ctrl->s_read[g], (t - 1) & 1, DEVERR_ATTN_WAIT)) return false;
        tc_fence_after();
        const int st = t % NS;
#pragma unroll
        for (int kb = 0; kb < Cfg::KB; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_tf32(tmem + g * 128,
                      desc_advance(operand_desc(q_addr + g * Cfg::Q_BYTES + kb * 16384, 0, 0),
                                   kk * 32),
                      desc_advance(operand_desc(k_addr + st * Cfg::K_BYTES + kb * 16384, 0, 0),
                                   kk * 32),
                      id_s, (kb > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&ctrl->s_full[g]);
        return true;
      };
      // O_g += P_g · V_t, P read from the shared P buffer in TMEM
      auto issue_pv = [&](int g, int t) -> bool {
        const int st = t % NS;
        if (!mbar_wait(&ctrl->p_ready[g], t & 1, DEVERR_ATTN_WAIT) ||
            !mbar_wait(&ctrl->v_full[st], (t / NS) & 1, DEVERR_ATTN_WAIT))
          return false;
        tc_fence_after();
#pragma unroll
        for (int kb = 0; kb < 4; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_tf32_tmem_a(tmem + Cfg::O_COL + g * HD, tmem + Cfg::P_COL + kb * 32 + kk * 8,
                             desc_advance(operand_desc(v_addr + st * Cfg::V_BYTES +
                                                           kb * Cfg::V_KBLOCK,
                                                       1, 0),
                                          kk * 1024),
                             id_o, (t > 0 || kb > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&ctrl->pv_done[g]);
        return true;
      };
      bool ok = mbar_wait(&ctrl->q_full, 0, DEVERR_ATTN_WAIT) &&
                mbar_wait(&ctrl->k_full[0], 0, DEVERR_ATTN_WAIT);
      if (ok) ok = issue_s(0, 0) && issue_s(1, 0);
      if (ok) umma_commit(&ctrl->k_empty[0]);
      for (int t = 0; ok && t < n_b; ++t) {
        const int st = t % NS;
        const int st1 = (t + 1) % NS;
        if (t + 1 < n_b) {
          if (!(ok = mbar_wait(&ctrl->k_full[st1], ((t + 1) / NS) & 1, DEVERR_ATTN_WAIT))) break;
          if (t + 1 < n_a && !(ok = issue_s(0, t + 1))) break;
          if (!(ok = issue_s(1, t + 1))) break;
          umma_commit(&ctrl->k_empty[st1]);  // tile B is the last reader of K_{t+1}
        }
        if (t < n_a && !(ok = issue_pv(0, t))) break;
        if (!(ok = issue_pv(1, t))) break;
        umma_commit(&ctrl->v_empty[st]);  // tile B is the last reader of V_t
      }
      if (!ok) ctrl->abort_flag = 1;
    }
  } else {
    // softmax of query tile g (warps 2-5: A, warps 6-9: B); thread r of the
    // group owns row r of the tile (= TMEM lane r)
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int n = g == 0 ? n_a : n_b;
    const int diag_t = qa + g;  // the tile's diagonal key/value tile (causal)
    const uint32_t row_tmem = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t s_row = row_tmem + g * 128;
    const uint32_t p_row = row_tmem + Cfg::P_COL;
    const uint32_t o_row = row_tmem + Cfg::O_COL + g * HD;
    const float scale2 = args.scale * 1.4426950408889634f;  // exp(s * scale) = 2^(s * scale2)
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int t = 0; t < n; ++t) {
      if (!mbar_wait(&ctrl->s_full[g], t & 1, DEVERR_ATTN_WAIT)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool diag = args.causal && t == diag_t;
      float v[4][32];
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tmem_ld_32x32b_x32(s_row + c * 32, v[c]);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (diag && c * 32 + j > r) v[c][j] = -INFINITY;
          mx[j & 3] = fmaxf(mx[j & 3], v[c][j]);
        }
      }
      // S(t) is in registers: the MMA thread may overwrite it with S(t+1)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctrl->s_read[g]);
      const float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      // The exponent reference m moves only when the tile's maximum exceeds it
      // by more than FA_RESCALE (log2 units): probabilities then stay <= 2^8,
      // and the output rescale below is skipped on most tiles. O / l does not
      // depend on the reference.
      const float mts = mt * scale2;  // scale2 > 0
      const float m_new = mts > m + FA_RESCALE ? mts : m;
      const float alpha = ex2_approx(m - m_new);  // 1 if kept; 0 on the first tile
      float sm[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float p = ex2_approx(fmaf(v[c][j], scale2, -m_new));
          v[c][j] = p;
          sm[j & 3] += p;
        }
      l = l * alpha + ((sm[0] + sm[1]) + (sm[2] + sm[3]));
      m = m_new;
      // The P buffer's previous reader, in P·V issue order A(0), B(0), A(1),
      // ...: B(t-1) for tile A; A(t) for tile B, or B(t-1) where A has no
      // key tile t (causal). Its completion also covers this tile's own
      // previous P·V, issued before it: O then holds key tiles 0..t-1.
      if (g == 1 || t > 0) {
        const int gb = (g == 0 || t < n_a) ? 1 - g : g;
        const int done = (g == 1 && t < n_a) ? t : t - 1;
        if (!mbar_wait(&ctrl->pv_done[gb], static_cast<uint32_t>(done & 1), DEVERR_ATTN_WAIT)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if (t > 0) {
        if (__any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            float o[32];
            tmem_ld_32x32b_x32(o_row + c * 32, o);
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] *= alpha;
            tmem_st_32x32b_x32(o_row + c * 32, o);
          }
        }
      }
      // P into the shared buffer: the A operand of this tile's P·V
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_st_32x32b_x32(p_row + c * 32, v[c]);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctrl->p_ready[g]);
    }
    if (ok) ok = mbar_wait(&ctrl->pv_done[g], (n - 1) & 1, DEVERR_ATTN_WAIT);
    if (ok) {
      tc_fence_after();
      const float inv = 1.0f / l;
      const long long row = q_row0 + g * FA_ROWS + r;
      float* orow = args.out + row * args.ldo + col0;
      const float* rrow = args.residual ? args.residual + row * args.ldo + col0 : nullptr;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        float o[32];
        tmem_ld_32x32b_x32(o_row + c * 32, o);
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          float4 y = make_float4(o[j] * inv, o[j + 1] * inv, o[j + 2] * inv, o[j + 3] * inv);
          if (rrow) {
            const float4 x = *reinterpret_cast<const float4*>(rrow + c * 32 + j);
            y.x += x.x; y.y += x.y; y.z += x.z; y.w += x.w;
          }
          *reinterpret_cast<float4*>(orow + c * 32 + j) = y;
        }
      }
    } else {
      ctrl->abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

template <int HD>
oxf_status launch_attention_heads2(const CUtensorMap& tq, const CUtensorMap& tk,
                                   const CUtensorMap& tv, const FaArgs& args, int batch,
                                   int heads, cudaStream_t stream, int dev) {
  using Cfg = Fa2Cfg<HD>;
  static unsigned long long configured[kMaxDevices] = {0};
  const unsigned long long ctx = current_context_id();
  if (dev >= 0 && dev < kMaxDevices && (ctx == 0 || configured[dev] != ctx)) {
    cudaError_t e = cudaFuncSetAttribute(attention_heads_flash2_kernel<HD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(attention)");
    configured[dev] = ctx;
  }
  dim3 grid(static_cast<unsigned>(args.tiles / 2), static_cast<unsigned>(heads),
            static_cast<unsigned>(batch));
  attention_heads_flash2_kernel<HD><<<grid, FA2_THREADS, Cfg::SMEM_BYTES, stream>>>(tq, tk, tv,
                                                                                    args);
  return check_launch("attention_heads_flash2_kernel");
}

template <int HD>
oxf_status launch_attention_heads(const CUtensorMap& tq, const CUtensorMap& tk,
                                  const CUtensorMap& tv, const FaArgs& args, int batch, int heads,
                                  cudaStream_t stream, int dev) {
  using Cfg = FaCfg<HD>;
  static unsigned long long configured[kMaxDevices] = {0};
  const unsigned long long ctx = current_context_id();
  if (dev >= 0 && dev < kMaxDevices && (ctx == 0 || configured[dev] != ctx)) {
    cudaError_t e = cudaFuncSetAttribute(attention_heads_flash_kernel<HD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(attention)");
    configured[dev] = ctx;
  }
  dim3 grid(static_cast<unsigned>(args.tiles), static_cast<unsigned>(heads),
            static_cast<unsigned>(batch));
  attention_heads_flash_kernel<HD><<<grid, FA_THREADS, Cfg::SMEM_BYTES, stream>>>(tq, tk, tv,
                                                                                  args);
  return check_launch("attention_heads_flash_kernel");
}

// out[:, j*HD..] = residual + softmax(Q_j K_jᵀ / sqrt(HD)) V_j for every
// head j of every sequence, in one launch. q, k: [batch*seq, dqk]; v, out,
// residual: [batch*seq, dv]; HD = dqk/heads = dv/heads. UNSUPPORTED_SHAPE
// (nothing launched) unless HD is 32 or 64, seq is a multiple of 128 and
// every matrix is 16-byte aligned.
oxf_status attention_heads_forward(const float* q, const float* k, const float* v,
                                   const float* residual, float* out, int batch, int seq,
                                   int dqk, int dv, int heads, int causal, cudaStream_t stream) {
  if (batch < 0 || seq < 0 || dqk < 0 || dv < 0 || heads < 1)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_attention_heads_forward: bad shape");
  if (batch == 0 || seq == 0 || dv == 0) return OXF_OK;
  if (!q || !k || !v || !out)
    return set_error(OXF_ERR_INVALID_ARG, "oxf_attention_heads_forward: null pointer");
  if (dqk % heads || dv % heads)
    return set_error(OXF_ERR_INVALID_ARG,
                     "oxf_attention_heads_forward: heads must divide d_qk and d_v");
  const int hd = dqk / heads;
  if (dv / heads != hd || (hd != 32 && hd != 64) || seq % FA_ROWS != 0 || batch > 65535 ||
      heads > 65535 ||
      !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) ||
      (residual && !aligned16(residual)))
    return set_error(OXF_ERR_UNSUPPORTED_SHAPE,
                     "oxf_attention_heads_forward: needs equal query and value head widths of "
                     "32 or 64, seq a multiple of 128 and 16-byte aligned matrices");
  const long long rows = static_cast<long long>(batch) * seq;
  CUtensorMap tq, tk, tv;
  int is3d = 0;
  bool ok = encode_map(&tq, q, dqk, rows, dqk, 1, 0, 32, FA_ROWS, false, &is3d) &&
            encode_map(&tk, k, dqk, rows, dqk, 1, 0, 32, FA_ROWS, false, &is3d) &&
            encode_map(&tv, v, dv, rows, dv, 1, 0, 32, hd, true, &is3d);
  if (!ok) return set_error(OXF_ERR_CUDA, "oxf_attention_heads_forward: tensor map encode failed");
  FaArgs a;
  a.out = out;
  a.residual = residual;
  a.ldo = dv;
  a.seq = seq;
  a.tiles = seq / FA_ROWS;
  a.causal = causal ? 1 : 0;
  a.scale = 1.0f / std::sqrt(static_cast<float>(hd));
  int dev = 0;
  oxf_status st = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (st != OXF_OK) return st;
  // two query tiles per CTA where the sequence has an even number of them
  const char* env = std::getenv("OXF_ATTENTION_TILES");  // measurement: "1" forces one
  const bool two = a.tiles % 2 == 0 && !(env && std::strcmp(env, "1") == 0);
  if (two)
    return hd == 32 ? launch_attention_heads2<32>(tq, tk, tv, a, batch, heads, stream, dev)
                    : launch_attention_heads2<64>(tq, tk, tv, a, batch, heads, stream, dev);
  return hd == 32 ? launch_attention_heads<32>(tq, tk, tv, a, batch, heads, stream, dev)
                  : launch_attention_heads<64>(tq, tk, tv, a, batch, heads, stream, dev);
}

oxf_status attention_read_device_error(uint32_t* code) {
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
