// exchange.cpp — the host side of the fused gradient exchange + SGD
// (oxf_exchange_* in include/oxf_host.h): this rank's signal pad, the IPC
// mappings of every other rank's arenas and pad, and the epoch counter that
// makes each launch's barrier values unique.
#include <cuda_runtime.h>

#include <cstring>
#include <exception>
#include <new>

#include "errors.hpp"
#include "oxf_host.h"

struct oxf_exchange_s {
  oxf_exchange_desc desc{};
  size_t count = 0;
  uint32_t* pad = nullptr;  // this rank's signal pad (cudaMalloc)
  bool connected = false;
  oxf_ipc_handle peer[OXF_EXCHANGE_MAX_RANKS][3]{};  // handles of the mapped ranks
  bool mapped[OXF_EXCHANGE_MAX_RANKS][3]{};
};

namespace {

oxf_status cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return OXF_OK;
  return oxf::set_error(OXF_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

void unmap(oxf_exchange ex) {
  for (int q = 0; q < ex->desc.world; ++q) {
    if (q == ex->desc.rank) continue;
    void* ptrs[3] = {ex->desc.params[q], const_cast<float*>(ex->desc.grads[q]),
                     ex->desc.signals[q]};
    for (int k = 0; k < 3; ++k)
      if (ex->mapped[q][k]) {
        oxf_ipc_close(&ex->peer[q][k], ptrs[k]);
        ex->mapped[q][k] = false;
      }
  }
}

}  // namespace

extern "C" {

oxf_status oxf_exchange_create(int rank, int world, float* params, float* grads, size_t count,
                               oxf_exchange* out) {
  if (!out) return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_exchange_create: null out");
  *out = nullptr;
  if (world < 1 || world > OXF_EXCHANGE_MAX_RANKS || rank < 0 || rank >= world)
    return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_exchange_create: rank %d of world %d", rank,
                          world);
  if (!params || !grads)
    return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_exchange_create: null arena");
  oxf_exchange ex = new (std::nothrow) oxf_exchange_s;
  if (!ex) return oxf::set_error(OXF_ERR_CUDA, "out of host memory");
  ex->desc.rank = rank;
  ex->desc.world = world;
  ex->desc.params[rank] = params;
  ex->desc.grads[rank] = grads;
  ex->count = count;
  void* pad = nullptr;
  oxf_status st = cuda(cudaMalloc(&pad, OXF_EXCHANGE_SIGNAL_BYTES), "cudaMalloc (signal pad)");
  if (st == OXF_OK) st = cuda(cudaMemset(pad, 0, OXF_EXCHANGE_SIGNAL_BYTES), "cudaMemset");
  if (st != OXF_OK) {
    if (pad) cudaFree(pad);
    delete ex;
    return st;
  }
  ex->pad = static_cast<uint32_t*>(pad);
  ex->desc.signals[rank] = ex->pad;
  if (world == 1) ex->connected = true;  // nothing to map
  *out = ex;
  return OXF_OK;
}

oxf_status oxf_exchange_handles(oxf_exchange ex, oxf_ipc_handle out[3]) {
  if (!ex || !out) return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_exchange_handles: null");
  const int r = ex->desc.rank;
  oxf_status st = oxf_ipc_export(ex->desc.params[r], &out[0]);
  if (st == OXF_OK) st = oxf_ipc_export(ex->desc.grads[r], &out[1]);
  if (st == OXF_OK) st = oxf_ipc_export(ex->pad, &out[2]);
  return st;
}

oxf_status oxf_exchange_connect(oxf_exchange ex, const oxf_ipc_handle* all) {
  if (!ex || !all) return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_exchange_connect: null");
  if (ex->connected && ex->desc.world > 1)
    return oxf::set_error(OXF_ERR_STATE, "oxf_exchange_connect: already connected");
  for (int q = 0; q < ex->desc.world; ++q) {
    if (q == ex->desc.rank) continue;
    void* p[3] = {nullptr, nullptr, nullptr};
    for (int k = 0; k < 3; ++k) {
      ex->peer[q][k] = all[3 * q + k];
      // Two arenas inside one allocation share a handle; it is mapped once
      // (a process may not open the same handle twice).
      int same = -1;
      for (int j = 0; j < k; ++j)
        if (std::memcmp(all[3 * q + j].handle, all[3 * q + k].handle, sizeof(all->handle)) == 0)
          same = j;
      if (same >= 0) {
        char* base = static_cast<char*>(p[same]) - all[3 * q + same].offset;
        p[k] = base + all[3 * q + k].offset;
      } else {
        oxf_status st = oxf_ipc_open(&all[3 * q + k], &p[k]);
        if (st != OXF_OK) {
          unmap(ex);
          return st;
        }
        ex->mapped[q][k] = true;
      }
      if (k == 0) ex->desc.params[q] = static_cast<float*>(p[0]);
      if (k == 1) ex->desc.grads[q] = static_cast<const float*>(p[1]);
      if (k == 2) ex->desc.signals[q] = static_cast<uint32_t*>(p[2]);
    }
  }
  ex->connected = true;
  return OXF_OK;
}

oxf_status oxf_exchange_step(oxf_exchange ex, size_t offset, size_t count, float lr, int blocks,
                             oxf_stream stream) {
  if (!ex) return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_exchange_step: null exchange");
  if (!ex->connected) return oxf::set_error(OXF_ERR_STATE, "oxf_exchange_step: not connected");
  if (offset > ex->count || count > ex->count - offset)
    return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_exchange_step: range outside the arenas");
  oxf_exchange_desc d = ex->desc;
  d.epoch = ex->desc.epoch + 1;
  d.blocks = blocks;
  const oxf_status st = oxf_exchange_sgd(&d, offset, count, lr, stream);
  if (st == OXF_OK && count > 0) ex->desc.epoch = d.epoch;
  return st;
}

oxf_status oxf_exchange_set_timeout(oxf_exchange ex, uint32_t timeout_us) {
  if (!ex) return oxf::set_error(OXF_ERR_INVALID_ARG, "oxf_exchange_set_timeout: null");
  ex->desc.timeout_us = timeout_us;
  return OXF_OK;
}

oxf_status oxf_exchange_destroy(oxf_exchange ex) {
  if (!ex) return OXF_OK;
  unmap(ex);
  oxf_status st = OXF_OK;
  if (ex->pad) st = cuda(cudaFree(ex->pad), "cudaFree (signal pad)");
  delete ex;
  return st;
}

}  // extern "C"
