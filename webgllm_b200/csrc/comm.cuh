// Tensor-parallel exchange over NVLink peer memory (one-shot push
// all-reduce), device side.
//
// Every rank owns one exchange buffer that its peers map (CUDA IPC):
//   header (1 KB): flags[r] at byte 64 r (the last exchange rank r
//                  completed into this buffer), then this rank's own
//                  producer / consumer sequence numbers and two last-CTA
//                  counters;
//   data:          2 parities x world slots x slot floats.
// A row-parallel matmul whose partial sums must be added across ranks pushes
// them, inside its own epilogue, straight into slot [rank] of every rank's
// buffer (layout [n][token], so a warp's stores are contiguous), and its last
// CTA raises flags[rank] = s (a system-scope release store) in every rank's
// header. The consumer (comm_reduce_kernel) waits, with a time limit, until
// every flag reached its own next sequence number, sums the slots from its
// own memory and writes the fp32 result [token][n].
//
// Two parities suffice: a rank can only push exchange s + 2 after it
// consumed s + 1, which needed every peer's push of s + 1, which each peer
// issued after consuming s (stream order). So slot (s & 1) is free again.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "device_utils.cuh"

namespace wg {

constexpr int kCommMaxRanks = 8;
constexpr int kCommHeaderBytes = 1024;
// header words (u64 index)
constexpr int kCommFlag0 = 0;          // flags[r] at word 8 r
constexpr int kCommProdSeq = 64;       // byte 512
constexpr int kCommConsSeq = 72;       // byte 576
constexpr int kCommProdCount = 80;     // byte 640 (u32 counter in a u64 word)
constexpr int kCommConsCount = 88;     // byte 704

struct CommDev {
  float *inbox[kCommMaxRanks];              // data region of each rank's buffer
  unsigned long long *hdr[kCommMaxRanks];   // header of each rank's buffer
  int world, rank;
  long long slot;                           // floats per slot
};

__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Parity of the exchange this launch produces (read once, at entry: only
// the launch's last CTA advances the sequence, after every CTA is done).
__device__ __forceinline__ int push_parity(const CommDev &c) {
  return (int)((*(volatile unsigned long long *)(c.hdr[c.rank] + kCommProdSeq) + 1) & 1);
}

// Output (token, n) of an [M][N] partial into slot `rank` of every rank.
__device__ __forceinline__ void push_store(const CommDev &c, int parity, int n, int tok, int M, float v) {
  const long long off = ((long long)(parity * c.world + c.rank)) * c.slot + (long long)n * M + tok;
  for (int p = 0; p < c.world; p++) c.inbox[p][off] = v;
}

// End of a pushing launch, called by every thread of every CTA: once all
// CTAs' stores are visible system-wide, the last CTA raises flags[rank] in
// every rank's header.
__device__ __forceinline__ void push_signal(const CommDev &c) {
  __shared__ bool s_last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned *count = reinterpret_cast<unsigned *>(c.hdr[c.rank] + kCommProdCount);
    const unsigned total = gridDim.x * gridDim.y * gridDim.z;
    s_last = atomicAdd(count, 1u) == total - 1;
    if (s_last) {
      __threadfence_system();
      unsigned long long *seq = c.hdr[c.rank] + kCommProdSeq;
      const unsigned long long s = *seq + 1;
      *seq = s;
      *count = 0;
      for (int p = 0; p < c.world; p++) st_release_sys(c.hdr[p] + kCommFlag0 + 8 * c.rank, s);
    }
  }
  __syncthreads();
}

cudaError_t launch_comm_reduce(const CommDev &c, int M, int N, float *out, unsigned *flags, cudaStream_t s,
                               bool pdl);
// x fp16 [M][K] = rmsnorm(a + b) * w (and resid_out = a + b if not null);
// with comm, b is the sum of the next exchange's partials (b unused).
cudaError_t launch_addnorm(const float *a, const float *b, const float *w, float eps, float *resid_out, void *x,
                           int M, int K, const CommDev *comm, unsigned *flags, cudaStream_t s, bool pdl);

}  // namespace wg
