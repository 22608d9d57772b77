// tmap.hpp — host helpers shared by the tcgen05 kernels' launchers (defined
// in gemm.cu): tensor-map encoding of f32 operand tiles and the CUDA
// context identity that keys per-device launch caches.
#pragma once
#include <cuda.h>

namespace oxf {

constexpr int kMaxDevices = 64;

// The current CUDA context's identity (0 if none can be read): caches that
// hold per-context state compare it, so a new context after a device reset
// is configured again.
unsigned long long current_context_id();

// Tensor map of an f32 operand for TMA tile loads: `inner` contiguous
// elements per row (leading dimension ld), `outer` rows, `batch` items
// bstride apart. K-major tiles take boxes of box_inner x box_outer with the
// 128B swizzle; MN-major tiles (mn_major) take 32-element chunks (see
// umma.cuh). *is3d reports whether the map carries a batch coordinate.
bool encode_map(CUtensorMap* map, const float* ptr, long long inner, long long outer,
                long long ld, int batch, long long bstride, int box_inner, int box_outer,
                bool mn_major, int* is3d);

}  // namespace oxf
