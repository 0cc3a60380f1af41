// The tensor-parallel group behind the C ABI (include/webgllm_comm.h,
// wg_tp_*): NCCL loaded on first use, the group's collectives on the
// context's stream, and the push exchange's set-up (IPC handles all-gathered
// through NCCL) so that no caller needs PyTorch or an MPI of its own.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <thread>
#include <vector>

#include "../../include/webgllm_comm.h"
#include "capi_internal.cuh"

static_assert(WG_TP_ID_BYTES == NCCL_UNIQUE_ID_BYTES, "group id size");

struct wg_tp {
  int device;
  int nranks, rank;
  ncclComm_t comm;
  int *d_word;  // the barrier's one-word all-reduce
  bool aborted;
};

namespace {

// The NCCL entry points this file uses, resolved from the loaded library.
struct Nccl {
  ncclResult_t (*get_version)(int *);
  ncclResult_t (*get_unique_id)(ncclUniqueId *);
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  ncclResult_t (*comm_abort)(ncclComm_t);
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t *);
  ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  const char *(*error_string)(ncclResult_t);
  bool ok;
  std::string why;
};

std::mutex g_nccl_lock;
Nccl g_nccl;
bool g_nccl_tried = false;

template <typename F>
bool resolve(void *h, const char *name, F *fn, std::string *why) {
  *fn = reinterpret_cast<F>(dlsym(h, name));
  if (!*fn) *why = std::string("NCCL lacks ") + name;
  return *fn != nullptr;
}

// Loads NCCL once: a copy already in the process (e.g. PyTorch's) is found
// by its soname first; WG_NCCL_LIBRARY names another file.
const Nccl &nccl() {
  std::lock_guard<std::mutex> guard(g_nccl_lock);
  if (g_nccl_tried) return g_nccl;
  g_nccl_tried = true;
  const char *path = getenv("WG_NCCL_LIBRARY");
  void *h = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    const char *e = dlerror();
    g_nccl.why = std::string("cannot load NCCL: ") + (e ? e : "dlopen failed");
    return g_nccl;
  }
  std::string why;
  g_nccl.ok = resolve(h, "ncclGetVersion", &g_nccl.get_version, &why) &&
              resolve(h, "ncclGetUniqueId", &g_nccl.get_unique_id, &why) &&
              resolve(h, "ncclCommInitRank", &g_nccl.comm_init_rank, &why) &&
              resolve(h, "ncclCommDestroy", &g_nccl.comm_destroy, &why) &&
              resolve(h, "ncclCommAbort", &g_nccl.comm_abort, &why) &&
              resolve(h, "ncclCommGetAsyncError", &g_nccl.comm_get_async_error, &why) &&
              resolve(h, "ncclAllReduce", &g_nccl.all_reduce, &why) &&
              resolve(h, "ncclAllGather", &g_nccl.all_gather, &why) &&
              resolve(h, "ncclGetErrorString", &g_nccl.error_string, &why);
  g_nccl.why = why;
  return g_nccl;
}

int tfail(wg_ctx *ctx, int status, const char *fmt, ...) {
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

int nccl_fail(wg_ctx *ctx, ncclResult_t r, const char *what) {
  const Nccl &n = nccl();
  const int st = r == ncclInvalidArgument || r == ncclInvalidUsage ? WG_INVALID_ARGUMENT : WG_CUDA_ERROR;
  return tfail(ctx, st, "%s: %s", what, n.ok ? n.error_string(r) : "NCCL error");
}

int begin(wg_ctx *ctx, const wg_tp *tp) {
  if (!ctx || !tp) return tfail(ctx, WG_INVALID_ARGUMENT, "null context or group");
  if (tp->device != ctx->device) return tfail(ctx, WG_INVALID_ARGUMENT, "group and context devices differ");
  if (tp->aborted) return tfail(ctx, WG_INVALID_ARGUMENT, "the group was aborted after a timeout");
  cudaError_t e = cudaSetDevice(ctx->device);
  return e == cudaSuccess ? WG_OK : tfail(ctx, wg::status_of(e), "cudaSetDevice: %s", cudaGetErrorString(e));
}

// Waits for ctx's stream for at most timeout_ms, watching the group for
// asynchronous errors; on timeout aborts the group.
int wait_stream(wg_ctx *ctx, wg_tp *tp, int timeout_ms, const char *what) {
  const Nccl &n = nccl();
  const auto t0 = std::chrono::steady_clock::now();
  const int limit = timeout_ms > 0 ? timeout_ms : 60000;
  while (true) {
    cudaError_t e = cudaStreamQuery(ctx->stream);
    if (e == cudaSuccess) return WG_OK;
    if (e != cudaErrorNotReady) return tfail(ctx, wg::status_of(e), "%s: %s", what, cudaGetErrorString(e));
    ncclResult_t async = ncclSuccess;
    if (n.comm_get_async_error(tp->comm, &async) == ncclSuccess && async != ncclSuccess &&
        async != ncclInProgress) {
      n.comm_abort(tp->comm);
      tp->aborted = true;
      return nccl_fail(ctx, async, what);
    }
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
    if (ms.count() > limit) {
      n.comm_abort(tp->comm);  // ends the group's kernels that wait for the missing rank
      tp->aborted = true;
      return tfail(ctx, WG_TIMEOUT, "%s: not every rank arrived within %d ms; the group was aborted", what, limit);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

}  // namespace

extern "C" {

int wg_tp_unique_id(void *id) {
  if (!id) return WG_INVALID_ARGUMENT;
  const Nccl &n = nccl();
  if (!n.ok) return WG_UNSUPPORTED;
  ncclUniqueId u;
  if (n.get_unique_id(&u) != ncclSuccess) return WG_CUDA_ERROR;
  memcpy(id, &u, sizeof u);
  return WG_OK;
}

int wg_tp_init(wg_ctx *ctx, int nranks, int rank, const void *id, wg_tp **out) {
  if (!ctx || !id || !out) return tfail(ctx, WG_INVALID_ARGUMENT, "wg_tp_init: null argument");
  *out = nullptr;
  if (nranks < 1 || nranks > wg::kCommMaxRanks || rank < 0 || rank >= nranks)
    return tfail(ctx, WG_INVALID_ARGUMENT, "wg_tp_init: rank %d of %d (at most %d ranks)", rank, nranks,
                 wg::kCommMaxRanks);
  const Nccl &n = nccl();
  if (!n.ok) return tfail(ctx, WG_UNSUPPORTED, "%s", n.why.c_str());
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return tfail(ctx, wg::status_of(e), "cudaSetDevice: %s", cudaGetErrorString(e));
  wg_tp *tp = new (std::nothrow) wg_tp{};
  if (!tp) return WG_OUT_OF_MEMORY;
  tp->device = ctx->device;
  tp->nranks = nranks;
  tp->rank = rank;
  if ((e = cudaMalloc(&tp->d_word, 256)) != cudaSuccess) {
    delete tp;
    return tfail(ctx, wg::status_of(e), "cudaMalloc: %s", cudaGetErrorString(e));
  }
  ncclUniqueId u;
  memcpy(&u, id, sizeof u);
  ncclResult_t r = n.comm_init_rank(&tp->comm, nranks, u, rank);
  if (r != ncclSuccess) {
    cudaFree(tp->d_word);
    delete tp;
    return nccl_fail(ctx, r, "ncclCommInitRank");
  }
  *out = tp;
  return WG_OK;
}

int wg_tp_destroy(wg_ctx *ctx, wg_tp *tp) {
  if (!tp) return WG_OK;
  if (ctx) {
    cudaSetDevice(ctx->device);
    if (ctx->stream && !tp->aborted) cudaStreamSynchronize(ctx->stream);
  }
  const Nccl &n = nccl();
  if (!tp->aborted && n.ok) n.comm_destroy(tp->comm);
  cudaFree(tp->d_word);
  delete tp;
  return WG_OK;
}

int wg_tp_info(const wg_tp *tp, int *nranks, int *rank) {
  if (!tp) return WG_INVALID_ARGUMENT;
  if (nranks) *nranks = tp->nranks;
  if (rank) *rank = tp->rank;
  return WG_OK;
}

int wg_tp_allreduce(wg_ctx *ctx, wg_tp *tp, void *buf, size_t count, int dtype, int op) {
  if (int st = begin(ctx, tp)) return st;
  if (!buf && count) return tfail(ctx, WG_INVALID_ARGUMENT, "wg_tp_allreduce: null buffer");
  ncclDataType_t t;
  switch (dtype) {
    case WG_TP_F32: t = ncclFloat32; break;
    case WG_TP_F16: t = ncclFloat16; break;
    case WG_TP_BF16: t = ncclBfloat16; break;
    case WG_TP_I64: t = ncclInt64; break;
    default: return tfail(ctx, WG_INVALID_ARGUMENT, "wg_tp_allreduce: unknown dtype %d", dtype);
  }
  if (op != WG_TP_SUM && op != WG_TP_MAX) return tfail(ctx, WG_INVALID_ARGUMENT, "wg_tp_allreduce: unknown op %d", op);
  if (count == 0) return WG_OK;
  ncclResult_t r = nccl().all_reduce(buf, buf, count, t, op == WG_TP_SUM ? ncclSum : ncclMax, tp->comm, ctx->stream);
  return r == ncclSuccess ? WG_OK : nccl_fail(ctx, r, "ncclAllReduce");
}

int wg_tp_barrier(wg_ctx *ctx, wg_tp *tp, int timeout_ms) {
  if (int st = begin(ctx, tp)) return st;
  ncclResult_t r = nccl().all_reduce(tp->d_word, tp->d_word, 1, ncclInt32, ncclSum, tp->comm, ctx->stream);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "barrier");
  return wait_stream(ctx, tp, timeout_ms, "wg_tp_barrier");
}

int wg_tp_comm(wg_ctx *ctx, wg_tp *tp, size_t bytes, wg_comm **out) {
  if (int st = begin(ctx, tp)) return st;
  if (!out) return tfail(ctx, WG_INVALID_ARGUMENT, "wg_tp_comm: null argument");
  *out = nullptr;
  const int W = tp->nranks, R = tp->rank;
  void *own = nullptr;
  unsigned char handle[WG_IPC_HANDLE_BYTES];
  if (int st = wg_ipc_alloc(ctx, bytes, &own, handle)) return st;
  // all-gather the handles: slot R of a device table, in place
  std::vector<unsigned char> all((size_t)W * WG_IPC_HANDLE_BYTES);
  unsigned char *d_all = nullptr;
  cudaError_t e = cudaMalloc(&d_all, all.size());
  int st = WG_OK;
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(d_all + (size_t)R * WG_IPC_HANDLE_BYTES, handle, WG_IPC_HANDLE_BYTES, cudaMemcpyHostToDevice,
                        ctx->stream);
  if (e != cudaSuccess) {
    st = tfail(ctx, wg::status_of(e), "wg_tp_comm: %s", cudaGetErrorString(e));
  } else {
    ncclResult_t r = nccl().all_gather(d_all + (size_t)R * WG_IPC_HANDLE_BYTES, d_all, WG_IPC_HANDLE_BYTES, ncclUint8,
                                       tp->comm, ctx->stream);
    if (r != ncclSuccess) st = nccl_fail(ctx, r, "ncclAllGather of the exchange handles");
    if (!st && (e = cudaMemcpyAsync(all.data(), d_all, all.size(), cudaMemcpyDeviceToHost, ctx->stream)) != cudaSuccess)
      st = tfail(ctx, wg::status_of(e), "wg_tp_comm: %s", cudaGetErrorString(e));
    if (!st) st = wait_stream(ctx, tp, 0, "wg_tp_comm");
  }
  if (d_all) cudaFree(d_all);
  std::vector<void *> ptrs(W, nullptr);
  ptrs[R] = own;
  for (int r = 0; r < W && !st; r++)
    if (r != R) st = wg_ipc_open(ctx, all.data() + (size_t)r * WG_IPC_HANDLE_BYTES, &ptrs[r]);
  wg_comm *c = nullptr;
  if (!st) st = wg_comm_init(ctx, W, R, ptrs.data(), bytes, &c);
  // every rank has mapped every buffer before anyone pushes
  if (!st) st = wg_tp_barrier(ctx, tp, 0);
  if (st) {
    if (c) delete c;
    for (int r = 0; r < W; r++)
      if (r != R && ptrs[r]) wg_ipc_close(ctx, ptrs[r]);
    wg_ipc_free(ctx, own);
    return st;
  }
  c->tp = tp;
  c->own = own;
  for (int r = 0; r < W; r++) c->opened[r] = r == R ? nullptr : ptrs[r];
  *out = c;
  return WG_OK;
}

}  // extern "C"

int wg_tp_comm_release(wg_ctx *ctx, wg_comm *comm) {
  // no rank still reads or writes a peer's buffer; then every mapping of
  // this rank's buffer is closed before it is freed
  int st = wg_tp_barrier(ctx, comm->tp, 0);
  for (int r = 0; r < comm->world; r++)
    if (comm->opened[r]) wg_ipc_close(ctx, comm->opened[r]);
  if (!st) st = wg_tp_barrier(ctx, comm->tp, 0);
  if (!st) wg_ipc_free(ctx, comm->own);  // after a failed barrier a peer may still map it: leak it
  comm->tp = nullptr;
  return st;
}
