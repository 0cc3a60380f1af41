// The C ABI of the tensor-parallel exchange (include/webgllm_comm.h): IPC
// buffers, the communicator, and the consumer-side reduction.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>

#include "../../include/webgllm_comm.h"
#include "capi_internal.cuh"
#include "comm.cuh"

namespace {

int cfail(wg_ctx *ctx, int status, const char *fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    ctx->last_error = buf;
  }
  return status;
}

int cuda_fail(wg_ctx *ctx, cudaError_t e, const char *what) {
  return cfail(ctx, wg::status_of(e), "%s: %s", what, cudaGetErrorString(e));
}

int begin(wg_ctx *ctx) {
  if (!ctx) return WG_INVALID_ARGUMENT;
  cudaError_t e = cudaSetDevice(ctx->device);
  return e == cudaSuccess ? WG_OK : cuda_fail(ctx, e, "cudaSetDevice");
}

}  // namespace

extern "C" {

int wg_ipc_alloc(wg_ctx *ctx, size_t bytes, void **dptr, void *handle) {
  if (int st = begin(ctx)) return st;
  if (!dptr || !handle || bytes < (size_t)wg::kCommHeaderBytes + 256)
    return cfail(ctx, WG_INVALID_ARGUMENT, "wg_ipc_alloc: bytes %zu (at least %d)", bytes,
                 wg::kCommHeaderBytes + 256);
  *dptr = nullptr;
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMalloc");
  if ((e = cudaMemset(p, 0, bytes)) != cudaSuccess || (e = cudaDeviceSynchronize()) != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(ctx, e, "cudaMemset");
  }
  cudaIpcMemHandle_t h;
  if ((e = cudaIpcGetMemHandle(&h, p)) != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(ctx, e, "cudaIpcGetMemHandle");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == WG_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof h);
  *dptr = p;
  return WG_OK;
}

int wg_ipc_free(wg_ctx *ctx, void *dptr) {
  if (int st = begin(ctx)) return st;
  if (!dptr) return WG_OK;
  cudaError_t e = cudaFree(dptr);
  return e == cudaSuccess ? WG_OK : cuda_fail(ctx, e, "cudaFree");
}

int wg_ipc_open(wg_ctx *ctx, const void *handle, void **dptr) {
  if (int st = begin(ctx)) return st;
  if (!handle || !dptr) return cfail(ctx, WG_INVALID_ARGUMENT, "wg_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  void *p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaIpcOpenMemHandle");
  *dptr = p;
  return WG_OK;
}

int wg_ipc_close(wg_ctx *ctx, void *dptr) {
  if (int st = begin(ctx)) return st;
  if (!dptr) return WG_OK;
  cudaError_t e = cudaIpcCloseMemHandle(dptr);
  return e == cudaSuccess ? WG_OK : cuda_fail(ctx, e, "cudaIpcCloseMemHandle");
}

int wg_comm_init(wg_ctx *ctx, int world, int rank, void *const *buffers, size_t bytes, wg_comm **out) {
  if (int st = begin(ctx)) return st;
  if (!out || !buffers) return cfail(ctx, WG_INVALID_ARGUMENT, "wg_comm_init: null argument");
  *out = nullptr;
  if (world < 1 || world > wg::kCommMaxRanks || rank < 0 || rank >= world)
    return cfail(ctx, WG_INVALID_ARGUMENT, "wg_comm_init: rank %d of %d (at most %d ranks)", rank, world,
                 wg::kCommMaxRanks);
  if (bytes < (size_t)wg::kCommHeaderBytes + 2 * world * 64)
    return cfail(ctx, WG_INVALID_ARGUMENT, "wg_comm_init: buffers of %zu bytes are too small", bytes);
  for (int r = 0; r < world; r++)
    if (!buffers[r] || ((uintptr_t)buffers[r] & 255u))
      return cfail(ctx, WG_INVALID_ARGUMENT, "wg_comm_init: buffer %d is null or not 256-byte aligned", r);
  wg_comm *c = new (std::nothrow) wg_comm{};
  if (!c) return WG_OUT_OF_MEMORY;
  c->device = ctx->device;
  c->world = world;
  c->rank = rank;
  c->bytes = bytes;
  c->dev.world = world;
  c->dev.rank = rank;
  c->dev.wait_ns = wg::kCommWaitNs;
  // data: 2 parities x world slots, each slot a multiple of 16 words
  c->dev.slot = (long long)((bytes - wg::kCommHeaderBytes) / (2 * (size_t)world * sizeof(unsigned long long))) / 16 * 16;
  for (int r = 0; r < world; r++) {
    uint8_t *b = static_cast<uint8_t *>(buffers[r]);
    c->dev.hdr[r] = reinterpret_cast<unsigned long long *>(b);
    c->dev.inbox[r] = reinterpret_cast<unsigned long long *>(b + wg::kCommHeaderBytes);
  }
  *out = c;
  return WG_OK;
}

int wg_comm_destroy(wg_ctx *ctx, wg_comm *comm) {
  if (!comm) return WG_OK;
  if (ctx) {
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  }
  int st = WG_OK;
  if (comm->tp) st = wg_tp_comm_release(ctx, comm);
  delete comm;
  return st;
}

int wg_comm_set_wait(wg_comm *comm, unsigned long long wait_ns) {
  if (!comm || wait_ns == 0) return WG_INVALID_ARGUMENT;
  comm->dev.wait_ns = wait_ns;
  return WG_OK;
}

int wg_comm_slot(const wg_comm *comm, size_t *floats) {
  if (!comm || !floats) return WG_INVALID_ARGUMENT;
  *floats = (size_t)comm->dev.slot;
  return WG_OK;
}

int wg_comm_reduce(wg_ctx *ctx, wg_comm *comm, int M, int N, float *out) {
  if (int st = begin(ctx)) return st;
  if (!comm || !out) return cfail(ctx, WG_INVALID_ARGUMENT, "wg_comm_reduce: null argument");
  if (comm->device != ctx->device) return cfail(ctx, WG_INVALID_ARGUMENT, "exchange and context devices differ");
  if (M <= 0 || N <= 0 || (size_t)M * N > (size_t)comm->dev.slot)
    return cfail(ctx, WG_INVALID_SHAPE, "wg_comm_reduce: %d x %d outputs (slot %lld floats)", M, N,
                 (long long)comm->dev.slot);
  cudaError_t e = wg::launch_comm_reduce(comm->dev, M, N, out, ctx->d_flags, ctx->stream, ctx->pdl);
  return e == cudaSuccess ? WG_OK : cuda_fail(ctx, e, "wg_comm_reduce");
}

int wg_comm_reduce_norm(wg_ctx *ctx, wg_comm *comm, int M, int K, const float *resid, const float *weight, float eps,
                        float *resid_out, void *x_out) {
  if (int st = begin(ctx)) return st;
  if (!comm || !resid || !weight || !x_out) return cfail(ctx, WG_INVALID_ARGUMENT, "wg_comm_reduce_norm: null argument");
  if (comm->device != ctx->device) return cfail(ctx, WG_INVALID_ARGUMENT, "exchange and context devices differ");
  if (M <= 0 || K <= 0 || K % 8 || (size_t)M * K > (size_t)comm->dev.slot)
    return cfail(ctx, WG_INVALID_SHAPE, "wg_comm_reduce_norm: %d x %d (K %% 8 == 0, slot %lld floats)", M, K,
                 (long long)comm->dev.slot);
  if (resid_out == resid) return cfail(ctx, WG_INVALID_ARGUMENT, "resid_out must not alias resid");
  cudaError_t e = wg::launch_addnorm(resid, nullptr, weight, eps, resid_out, x_out, M, K, &comm->dev, ctx->d_flags,
                                     ctx->stream, ctx->pdl);
  return e == cudaSuccess ? WG_OK : cuda_fail(ctx, e, "wg_comm_reduce_norm");
}

}  // extern "C"
