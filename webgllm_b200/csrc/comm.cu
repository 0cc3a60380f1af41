// The consumer side of the push all-reduce (comm.cuh): wait for every rank's
// partial of the next exchange (word by word), then sum them from this
// rank's own buffer.
#include <cooperative_groups.h>

#include "comm.cuh"

namespace wg {

namespace {

constexpr int kReduceThreads = 256;

__global__ void __launch_bounds__(kReduceThreads) comm_reduce_kernel(const CommDev c, int M, int N, float *out,
                                                                     unsigned *flags) {
  pdl_trigger();
  pdl_wait();  // this rank's own push (the previous kernel) is complete
  __shared__ unsigned s_e;
  unsigned long long *hdr = c.hdr[c.rank];
  if (threadIdx.x == 0) s_e = (unsigned)(*(volatile unsigned long long *)(hdr + kCommConsSeq) + 1);
  __syncthreads();
  const unsigned e = s_e;
  const unsigned long long *base = c.inbox[c.rank] + (long long)(e & 1) * c.world * c.slot;
  const int total = M * N;
  for (int i = blockIdx.x * kReduceThreads + threadIdx.x; i < total; i += gridDim.x * kReduceThreads) {
    // slot layout [n][token]; out [token][n]
    const int n = i / M, tok = i - n * M;
    float v = 0.0f;
    for (int r = 0; r < c.world; r++) v += comm_wait_word(base + (long long)r * c.slot + i, e, flags, c.wait_ns);
    out[(size_t)tok * N + n] = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned *count = reinterpret_cast<unsigned *>(hdr + kCommConsCount);
    if (atomicAdd(count, 1u) == gridDim.x - 1) {
      *(volatile unsigned long long *)(hdr + kCommConsSeq) = e;
      *count = 0;
    }
  }
}

// Residual add + RMS norm of M rows of K, one thread-block cluster of CL
// CTAs per row (each CTA a K/CL slice, its sum of squares shared through
// distributed shared memory): x fp16 = rmsnorm(a + b) * w, optional
// resid_out = a + b. With COMM, b is the sum over ranks of the next
// exchange's partials (layout [k][row]), each word waited for — the
// all-reduce, the residual add and the norm in one launch.
constexpr int kNormThreads = 256;
constexpr int kNormMaxPerThread = 16;  // K / CL / 256 values kept in registers

template <bool COMM>
__global__ void __launch_bounds__(kNormThreads) addnorm_kernel(const float *a, const float *b, const float *w,
                                                               float eps, float *resid_out, __half *x, int M, int K,
                                                               const CommDev c, unsigned *flags) {
  pdl_trigger();
  pdl_wait();
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int CL = (int)cluster.num_blocks(), cr = (int)cluster.block_rank();
  const int m = blockIdx.y;
  const int Kc = K / CL, k0 = cr * Kc;
  __shared__ float s_part[kNormThreads / 32];
  __shared__ float s_ss;
  __shared__ unsigned s_e;
  const unsigned long long *base = nullptr;
  if (COMM) {
    if (threadIdx.x == 0) s_e = (unsigned)(*(volatile unsigned long long *)(c.hdr[c.rank] + kCommConsSeq) + 1);
    __syncthreads();
    base = c.inbox[c.rank] + (long long)(s_e & 1) * c.world * c.slot;
  }
  float v[kNormMaxPerThread];
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < kNormMaxPerThread; j++) {
    const int k = k0 + threadIdx.x + j * kNormThreads;
    v[j] = 0.0f;
    if (threadIdx.x + j * kNormThreads < Kc) {
      float add = 0.0f;
      if (COMM) {
        for (int r = 0; r < c.world; r++) add += comm_wait_word(base + (long long)r * c.slot + (long long)k * M + m, s_e, flags, c.wait_ns);
      } else if (b) {
        add = b[(size_t)m * K + k];
      }
      v[j] = a[(size_t)m * K + k] + add;
      if (resid_out) resid_out[(size_t)m * K + k] = v[j];
      ss += v[j] * v[j];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int i = 0; i < kNormThreads / 32; i++) t += s_part[i];
    s_ss = t;
  }
  cluster.sync();
  float total = 0.0f;
  for (int r = 0; r < CL; r++) total += *cluster.map_shared_rank(&s_ss, r);
  const float inv = rsqrtf(total / (float)K + eps);
#pragma unroll
  for (int j = 0; j < kNormMaxPerThread; j++) {
    const int k = k0 + threadIdx.x + j * kNormThreads;
    if (threadIdx.x + j * kNormThreads < Kc) x[(size_t)m * K + k] = __float2half_rn(clamp_half(v[j] * inv * w[k]));
  }
  if (COMM) {
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long *hdr = c.hdr[c.rank];
      unsigned *count = reinterpret_cast<unsigned *>(hdr + kCommConsCount);
      if (atomicAdd(count, 1u) == gridDim.x * gridDim.y - 1) {
        *(volatile unsigned long long *)(hdr + kCommConsSeq) = s_e;
        *count = 0;
      }
    }
  }
  cluster.sync();  // peers may still read s_ss
}

}  // namespace

cudaError_t launch_addnorm(const float *a, const float *b, const float *w, float eps, float *resid_out, void *x,
                           int M, int K, const CommDev *comm, unsigned *flags, cudaStream_t s, bool pdl) {
  // cluster size: enough CTAs per row that each thread keeps at most
  // kNormMaxPerThread values, and K splits evenly
  int CL = 1;
  while ((K / CL) > kNormThreads * kNormMaxPerThread || (CL < 8 && K % (CL * 2) == 0 && K / (CL * 2) >= 1024)) CL *= 2;
  if (CL > 8 || K % CL) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)CL, (unsigned)M);
  cfg.blockDim = dim3(kNormThreads);
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  int n = 0;
  at[n].id = cudaLaunchAttributeClusterDimension;
  at[n].val.clusterDim.x = (unsigned)CL;
  at[n].val.clusterDim.y = 1;
  at[n].val.clusterDim.z = 1;
  n++;
  if (pdl) {
    at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[n].val.programmaticStreamSerializationAllowed = 1;
    n++;
  }
  cfg.attrs = at;
  cfg.numAttrs = n;
  CommDev c{};
  if (comm) c = *comm;
  __half *xh = reinterpret_cast<__half *>(x);
  return comm ? cudaLaunchKernelEx(&cfg, addnorm_kernel<true>, a, b, w, eps, resid_out, xh, M, K, c, flags)
              : cudaLaunchKernelEx(&cfg, addnorm_kernel<false>, a, b, w, eps, resid_out, xh, M, K, c, flags);
}

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
