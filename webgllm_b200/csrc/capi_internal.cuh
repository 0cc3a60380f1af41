// The C ABI's opaque types (include/webgllm_q4.h), shared by the files that
// implement its entry points.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "comm.cuh"
#include "common.cuh"
#include "q4_layout.cuh"

namespace wg {
constexpr size_t kReduceBytes = 64 * 1024;
}

struct wg_ctx {
  int device = 0;
  int num_sms = wg::kB200Sms;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  unsigned *d_flags = nullptr;  // device error flags (kFlag*)
  unsigned *d_count = nullptr;  // last-CTA counter of wg_head's argmax (rests at 0)
  unsigned long long *d_reduce = nullptr;  // wg_head's per-CTA argmax keys (kReduceBytes)
  uint8_t *staging = nullptr;   // device copy of a repack's source bytes
  size_t staging_bytes = 0;
  uint8_t *work = nullptr;      // matmul scratch: fp16 copy of x, split-K sums
  size_t work_bytes = 0;
  bool pdl = true;              // programmatic dependent launch for the GEMV
  int trigger_at = 1;           // GemvArgs::trigger_at (WG_GEMV_TRIGGER overrides)
  int gemv_wide = -1;           // -1: by shape; 0 / 1 forced (WG_GEMV_WIDE)
  int exact_rows = 16;          // WG_OPT_EXACT_ROWS: up to this many rows on the GEMV
  size_t norm_fuse_bytes = 64 << 10;  // largest row-statistics read a fused norm prologue makes per CTA
  unsigned long long *trace = nullptr;       // wg_trace buffer (device) or null
  unsigned long long trace_cap = 0;          // records that fit
  unsigned long long *d_trace_next = nullptr;  // device record counter
  unsigned launch_index = 0;
  std::string last_error;
};

// A tensor-parallel exchange (comm.cuh): this rank's view of every rank's
// buffer (the caller owns the buffers and their mappings).
struct wg_tp;
struct wg_comm {
  int device;
  int world, rank;
  size_t bytes;
  wg::CommDev dev;
  // set by wg_tp_comm, which owns the buffers: released by wg_comm_destroy
  wg_tp *tp = nullptr;
  void *own = nullptr;
  void *opened[wg::kCommMaxRanks] = {};
};

// Releases the buffers of a communicator made by wg_tp_comm (tp_nccl.cu).
int wg_tp_comm_release(wg_ctx *ctx, wg_comm *comm);

struct wg_q4mat {
  wg::Q4Dims d;
  int device;
  uint8_t *base;  // one allocation: nib | scl | zro
  uint32_t *nib;
  uint16_t *scl;
  uint8_t *zro;
  size_t bytes;
};


namespace wg {
struct GemvArgs;
// Whether a GEMV launch of these arguments goes to the wide kernel (capi.cu).
bool gemv_use_wide(const wg_ctx *ctx, const GemvArgs &a);
}  // namespace wg
