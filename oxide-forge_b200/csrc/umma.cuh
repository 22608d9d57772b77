// umma.cuh — shared-memory operand tiles of the tcgen05 kernels (GEMM and
// fused attention): the matrix descriptors of one K=8 slice and the TMA loads
// that fill a tile.
#pragma once
#include <cstdint>

#include "ptx.cuh"

namespace oxf {

// Shared-memory descriptor of one K=8 slice of an operand tile.
//  K-major tile: rows of 128 B (32 K values), 128B swizzle in 8-row atoms
//    1024 B apart (SBO); K slice kk starts kk*32 B into the row.
//  MN-major tile: 32-element MN chunks (one TMA box of 32 K rows, 4 KB,
//    LBO apart), 128B swizzle with 32-byte atoms: 4-row atoms 512 B apart
//    (SBO); K slice kk starts at K row 8*kk (1024 B).
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int mn_major, int kk) {
  return mn_major ? make_smem_desc(base + kk * 1024, 4096, 512, kLayoutSW128Atom32B)
                  : make_smem_desc(base + kk * 32, 16, 1024, kLayoutSW128);
}

// Byte step between the K=8 slices of an operand tile (see operand_desc).
__device__ __forceinline__ uint32_t operand_kstep(int mn_major) { return mn_major ? 1024u : 32u; }

// A descriptor moved by `bytes` within shared memory: only the start
// address field (bits [0,14), in 16-byte units) changes, and shared memory
// addresses stay below 2^18, so the add never carries out of the field.
__device__ __forceinline__ uint64_t desc_advance(uint64_t desc, uint32_t bytes) {
  return desc + (bytes >> 4);
}

template <int ROWS>
__device__ __forceinline__ void load_operand(uint8_t* dst, const CUtensorMap* map, uint64_t* bar,
                                             int mn_major, int is3d, int chunked, int row0, int k0,
                                             int b, uint64_t pol) {
  if (!mn_major) {
    if (is3d) tma_load_3d(dst, map, bar, k0, row0, b, pol);
    else tma_load_2d(dst, map, bar, k0, row0, pol);
  } else if (chunked) {
    // One box covers all ROWS/32 chunks: smem chunk c lands at c * 4096 B.
    if (is3d) tma_load_4d(dst, map, bar, 0, k0, row0 / 32, b, pol);
    else tma_load_3d(dst, map, bar, 0, k0, row0 / 32, pol);
  } else {
#pragma unroll
    for (int c = 0; c < ROWS / 32; ++c) {
      if (is3d) tma_load_3d(dst + c * 4096, map, bar, row0 + 32 * c, k0, b, pol);
      else tma_load_2d(dst + c * 4096, map, bar, row0 + 32 * c, k0, pol);
    }
  }
}

}  // namespace oxf
