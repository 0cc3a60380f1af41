// The consumer side of the push all-reduce (comm.cuh): wait for every rank's
// partial of the next exchange, then sum them from this rank's own buffer.
#include "comm.cuh"

namespace wg {

namespace {

constexpr int kReduceThreads = 256;
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s, then give up and report

__global__ void __launch_bounds__(kReduceThreads) comm_reduce_kernel(const CommDev c, int M, int N, float *out,
                                                                     unsigned *flags) {
  pdl_trigger();
  pdl_wait();  // this rank's own push (the previous kernel) is complete
  __shared__ unsigned long long s_e;
  __shared__ bool s_last;
  unsigned long long *hdr = c.hdr[c.rank];
  if (threadIdx.x == 0) {
    const unsigned long long e = *(volatile unsigned long long *)(hdr + kCommConsSeq) + 1;
    s_e = e;
    const unsigned long long t0 = globaltimer();
    for (int r = 0; r < c.world; r++) {
      while (ld_acquire_sys(hdr + kCommFlag0 + 8 * r) < e) {
        if (globaltimer() - t0 > kWaitNs) {  // a rank never pushed: report, carry on
          raise_flag(flags, kFlagTimeout);
          break;
        }
        __nanosleep(64);
      }
    }
  }
  __syncthreads();
  const int parity = (int)(s_e & 1);
  const float *base = c.inbox[c.rank] + (long long)parity * c.world * c.slot;
  const int total = M * N;
  for (int i = blockIdx.x * kReduceThreads + threadIdx.x; i < total; i += gridDim.x * kReduceThreads) {
    // slot layout [n][token]; out [token][n]
    const int n = i / M, tok = i - n * M;
    float v = 0.0f;
    for (int r = 0; r < c.world; r++) v += base[(long long)r * c.slot + i];
    out[(size_t)tok * N + n] = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned *count = reinterpret_cast<unsigned *>(hdr + kCommConsCount);
    s_last = atomicAdd(count, 1u) == gridDim.x - 1;
    if (s_last) {
      *(volatile unsigned long long *)(hdr + kCommConsSeq) = s_e;
      *count = 0;
    }
  }
}

}  // namespace

cudaError_t launch_comm_reduce(const CommDev &c, int M, int N, float *out, unsigned *flags, cudaStream_t s,
                               bool pdl) {
  const int total = M * N;
  int grid = (total + kReduceThreads * 4 - 1) / (kReduceThreads * 4);
  if (grid < 1) grid = 1;
  if (grid > 148) grid = 148;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kReduceThreads);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  if (pdl) {
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, comm_reduce_kernel, c, M, N, out, flags);
}

}  // namespace wg
