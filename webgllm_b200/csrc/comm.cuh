// Tensor-parallel exchange over NVLink peer memory (one-shot push
// all-reduce), device side.
//
// Every rank owns one exchange buffer that its peers map (CUDA IPC):
//   header (1 KB): this rank's producer / consumer sequence numbers and two
//                  last-CTA counters (local use only);
//   data:          2 parities x world slots x slot words of 64 bits.
// A row-parallel matmul whose partial sums must be added across ranks pushes
// them, inside its own epilogue, straight into slot [rank] of every rank's
// buffer (layout [n][token], so a warp's stores are contiguous). Each word
// carries its value and the exchange's sequence number (value bits low,
// sequence high) and is written with one 64-bit store, so the consumer needs
// no flag and no fence: it polls each word (with a time limit) until the
// word carries the sequence number it expects, then adds the values — the
// low-latency protocol of small all-reduces, one NVLink trip.
//
// Two parities suffice: a rank can only push exchange s + 2 after it
// consumed s + 1, which needed every peer's push of s + 1, which each peer
// issued after consuming s (stream order). So slot (s & 1) is free again;
// a stale word there carries s, never s + 2.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "device_utils.cuh"

namespace wg {

constexpr int kCommMaxRanks = 8;
constexpr int kCommHeaderBytes = 1024;
// header words (u64 index)
constexpr int kCommProdSeq = 64;       // byte 512
constexpr int kCommConsSeq = 72;       // byte 576
constexpr int kCommProdCount = 80;     // byte 640 (u32 counter in a u64 word)
constexpr int kCommConsCount = 88;     // byte 704
constexpr unsigned long long kCommWaitNs = 2000000000ull;  // default wait: 2 s, then give up and report

struct CommDev {
  unsigned long long *inbox[kCommMaxRanks];  // data region of each rank's buffer
  unsigned long long *hdr[kCommMaxRanks];    // header of each rank's buffer
  int world, rank;
  long long slot;                            // words per slot
  unsigned long long wait_ns;                // how long a consumer polls one word
};

// The sequence number of the exchange this launch produces. Only the
// previous pushing launch's last CTA advances it, so a launch reads it after
// its dependency wait (griddepcontrol.wait).
__device__ __forceinline__ unsigned push_seq(const CommDev &c) {
  return (unsigned)(*(volatile unsigned long long *)(c.hdr[c.rank] + kCommProdSeq) + 1);
}

// Output (token, n) of an [M][N] partial into slot `rank` of every rank.
__device__ __forceinline__ void push_store(const CommDev &c, unsigned seq, int n, int tok, int M, float v) {
  const long long off = ((long long)((seq & 1) * c.world + c.rank)) * c.slot + (long long)n * M + tok;
  const unsigned long long w = ((unsigned long long)seq << 32) | __float_as_uint(v);
  for (int p = 0; p < c.world; p++)
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(c.inbox[p] + off), "l"(w) : "memory");
}

// End of a pushing launch, called by every thread of every CTA: the last
// CTA advances this rank's producer sequence number.
__device__ __forceinline__ void push_signal(const CommDev &c) {
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned *count = reinterpret_cast<unsigned *>(c.hdr[c.rank] + kCommProdCount);
    const unsigned total = gridDim.x * gridDim.y * gridDim.z;
    if (atomicAdd(count, 1u) == total - 1) {
      unsigned long long *seq = c.hdr[c.rank] + kCommProdSeq;
      *seq = *seq + 1;
      *count = 0;
    }
  }
}

// The value of word `w` once it carries sequence number `e`: polls (relaxed,
// system scope) for at most wait_ns, then raises kFlagTimeout. Once the
// flag is up (this or an earlier wait ran out) no word is waited for again,
// so a launch whose peer never pushed ends after one wait_ns.
__device__ __forceinline__ float comm_wait_word(const unsigned long long *w, unsigned e, unsigned *flags,
                                                unsigned long long wait_ns) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(w) : "memory");
  if ((unsigned)(v >> 32) == e) return __uint_as_float((unsigned)v);
  if (*(volatile unsigned *)flags & kFlagTimeout) return 0.0f;
  const unsigned long long t0 = globaltimer();
  while (true) {
    __nanosleep(32);
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(w) : "memory");
    if ((unsigned)(v >> 32) == e) return __uint_as_float((unsigned)v);
    if (globaltimer() - t0 > wait_ns || (*(volatile unsigned *)flags & kFlagTimeout)) {
      raise_flag(flags, kFlagTimeout);
      return 0.0f;
    }
  }
}

cudaError_t launch_comm_reduce(const CommDev &c, int M, int N, float *out, unsigned *flags, cudaStream_t s,
                               bool pdl);
// x fp16 [M][K] = rmsnorm(a + b) * w (and resid_out = a + b if not null);
// with comm, b is the sum of the next exchange's partials (b unused).
cudaError_t launch_addnorm(const float *a, const float *b, const float *w, float eps, float *resid_out, void *x,
                           int M, int K, const CommDev *comm, unsigned *flags, cudaStream_t s, bool pdl);

}  // namespace wg
