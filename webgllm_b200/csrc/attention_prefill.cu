// Causal GQA attention for prompts (many query rows per sequence) on the
// tensor cores: the scores / attend passes of the reference's prefill
// (src/gpu/kernels.ts:2386-2579, run by forwardBatch for a prompt) as one
// flash-attention kernel.
//
// The decode kernel (decoder.cu, attention_kernel) serves one query row per
// CTA with CUDA-core dot products; for a prompt of P rows that re-reads each
// sequence's keys P times and runs the whole QK^T / PV work on the FMA pipe.
// Here a CTA takes 64 consecutive query rows of one (sequence, query head):
// - 4 warps, 16 query rows each; the warp's Q fragments (already RoPE'd and
//   scaled by 1/sqrt(Dh), fp16, from wg_rope_kv) stay in registers;
// - keys and values stream through shared memory in tiles of 64 positions
//   (cp.async, two buffers: the next tile loads while this one is used; rows
//   padded by 16 bytes so that ldmatrix reads hit distinct banks);
// - S = Q K^T with mma.sync.m16n8k16 (fp16 in, fp32 accumulate; K fragments
//   by ldmatrix), the causal mask on absolute positions, an online softmax
//   per row in registers (max and sum kept per thread, the 4 lanes of a row
//   combined by shuffles), then O += P V with P (rounded to fp16) taken
//   straight from the score registers as the A operand and V fragments by
//   ldmatrix.trans;
// - O / l written as fp16.
// Keys of a sequence are cache positions 0 .. pos0[b] + i for its i-th row
// (earlier calls' rows plus this call's, appended by wg_rope_kv).
#include <cuda_fp16.h>

#include "common.cuh"
#include "decoder_kernels.cuh"
#include "device_utils.cuh"

namespace wg {

namespace {

constexpr int kFaRows = 64;     // query rows per CTA (4 warps x 16)
constexpr int kFaKeys = 64;     // keys per tile
constexpr int kFaThreads = 128;

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_f16(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&h);
}

template <int Dh>
__global__ void __launch_bounds__(kFaThreads) flash_prefill_kernel(const __half *q, int rps, int H, int Hkv,
                                                                   const __half *k_cache, const __half *v_cache,
                                                                   int cache_len, const int *pos0, __half *out) {
  pdl_trigger();  // dependents may launch now; they wait for this grid to finish
  pdl_wait();     // q and the appended keys come from the previous kernel
  constexpr int kStride = Dh + 8;          // halves per shared-memory row
  constexpr int kTile = kFaKeys * kStride;  // halves per K (or V) buffer
  constexpr int kChunks = Dh / 8;           // 16-byte chunks per row
  constexpr float kLog2e = 1.4426950408889634f;
  extern __shared__ __align__(16) __half fa_smem[];
  __half *ks = fa_smem;              // [2][kFaKeys][kStride]
  __half *vs = fa_smem + 2 * kTile;  // [2][kFaKeys][kStride]

  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (H / Hkv);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int p0 = pos0[b];
  const int row_end = min(rps, (qb + 1) * kFaRows);  // this CTA's rows: [qb * 64, row_end)
  const int kend = max(0, min(p0 + row_end, cache_len));  // keys [0, kend)
  const int ntiles = (kend + kFaKeys - 1) / kFaKeys;
  const __half *kbase = k_cache + ((size_t)b * Hkv + hk) * cache_len * Dh;
  const __half *vbase = v_cache + ((size_t)b * Hkv + hk) * cache_len * Dh;

  auto load_tile = [&](int kt, int buf) {
    __half *kd = ks + buf * kTile, *vd = vs + buf * kTile;
    for (int i = tid; i < kFaKeys * kChunks; i += kFaThreads) {
      const int r = i / kChunks, c = i - r * kChunks;
      const int pos = kt * kFaKeys + r;
      if (pos < kend) {
        cp_async16(kd + r * kStride + c * 8, kbase + (size_t)pos * Dh + c * 8);
        cp_async16(vd + r * kStride + c * 8, vbase + (size_t)pos * Dh + c * 8);
      } else {  // past the keys: zeros (masked scores; P = 0 must not meet NaN)
        *reinterpret_cast<uint4 *>(kd + r * kStride + c * 8) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4 *>(vd + r * kStride + c * 8) = make_uint4(0, 0, 0, 0);
      }
    }
    cp_async_commit();
  };
  if (ntiles > 0) load_tile(0, 0);

  // this thread's two query rows (g and g + 8 of the warp's 16) and their
  // absolute positions; rows past the prompt read its last row (not stored)
  const int i0 = qb * kFaRows + warp * 16;
  const int ra = min(i0 + g, rps - 1), rb = min(i0 + g + 8, rps - 1);
  const int qpa = p0 + i0 + g, qpb = qpa + 8;
  uint32_t qf[Dh / 16][4];
  {
    const __half *qa = q + ((size_t)(b * rps + ra) * H + h) * Dh;
    const __half *qb_ = q + ((size_t)(b * rps + rb) * H + h) * Dh;
#pragma unroll
    for (int kk = 0; kk < Dh / 16; kk++) {
      qf[kk][0] = *reinterpret_cast<const uint32_t *>(qa + 16 * kk + 2 * t);
      qf[kk][1] = *reinterpret_cast<const uint32_t *>(qb_ + 16 * kk + 2 * t);
      qf[kk][2] = *reinterpret_cast<const uint32_t *>(qa + 16 * kk + 8 + 2 * t);
      qf[kk][3] = *reinterpret_cast<const uint32_t *>(qb_ + 16 * kk + 8 + 2 * t);
    }
  }
  float o[Dh / 8][4];
#pragma unroll
  for (int dt = 0; dt < Dh / 8; dt++) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.0f;
  float ma = -INFINITY, mb = -INFINITY, la = 0.0f, lb = 0.0f;  // running max / partial sums (log2 units)

  const int jm = lane >> 3, jr = lane & 7;  // ldmatrix: this lane addresses row jr of matrix jm
  for (int kt = 0; kt < ntiles; kt++) {
    const int buf = kt & 1;
    if (kt + 1 < ntiles) {
      load_tile(kt + 1, buf ^ 1);
      cp_async_wait_group<1>();
    } else {
      cp_async_wait_group<0>();
    }
    __syncthreads();
    const uint32_t kaddr = smem_u32(ks + buf * kTile), vaddr = smem_u32(vs + buf * kTile);

    // S = Q K^T for the warp's 16 rows x 64 keys (8 n-tiles of 8 keys)
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; nt++) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
#pragma unroll
    for (int np = 0; np < 4; np++) {  // keys 16 np .. 16 np + 15
#pragma unroll
      for (int kk = 0; kk < Dh / 16; kk++) {
        // matrices: (keys +0..7, dims 16kk..+7), (keys +0..7, dims +8..15),
        //           (keys +8..15, dims 16kk..+7), (keys +8..15, dims +8..15)
        const int key = 16 * np + 8 * (jm >> 1) + jr, dim = 16 * kk + 8 * (jm & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kaddr + (uint32_t)(key * kStride + dim) * 2, b0, b1, b2, b3);
        mma_f16(s[2 * np], qf[kk], b0, b1);
        mma_f16(s[2 * np + 1], qf[kk], b2, b3);
      }
    }
    // causal mask (only tiles that reach past a row's position)
    const int key0 = kt * kFaKeys;
    if (key0 + kFaKeys - 1 > p0 + i0) {
#pragma unroll
      for (int nt = 0; nt < 8; nt++) {
        const int k0 = key0 + 8 * nt + 2 * t;
        if (k0 > qpa) s[nt][0] = -INFINITY;
        if (k0 + 1 > qpa) s[nt][1] = -INFINITY;
        if (k0 > qpb) s[nt][2] = -INFINITY;
        if (k0 + 1 > qpb) s[nt][3] = -INFINITY;
      }
    }
    // online softmax (log2 domain)
    float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; nt++) {
      mxa = fmaxf(mxa, fmaxf(s[nt][0], s[nt][1]));
      mxb = fmaxf(mxb, fmaxf(s[nt][2], s[nt][3]));
    }
    mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
    mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
    mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
    mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
    const float mna = fmaxf(ma, mxa * kLog2e), mnb = fmaxf(mb, mxb * kLog2e);
    // a row with every key so far masked keeps max -inf: scale 1, weights 0
    const float ca = mna == -INFINITY ? 1.0f : exp2f(ma - mna);
    const float cb = mnb == -INFINITY ? 1.0f : exp2f(mb - mnb);
    const float sa = mna == -INFINITY ? 0.0f : mna, sb = mnb == -INFINITY ? 0.0f : mnb;
    ma = mna;
    mb = mnb;
    float suma = 0.0f, sumb = 0.0f;
#pragma unroll
    for (int nt = 0; nt < 8; nt++) {
      s[nt][0] = exp2f(s[nt][0] * kLog2e - sa);
      s[nt][1] = exp2f(s[nt][1] * kLog2e - sa);
      s[nt][2] = exp2f(s[nt][2] * kLog2e - sb);
      s[nt][3] = exp2f(s[nt][3] * kLog2e - sb);
      suma += s[nt][0] + s[nt][1];
      sumb += s[nt][2] + s[nt][3];
    }
    la = la * ca + suma;
    lb = lb * cb + sumb;
#pragma unroll
    for (int dt = 0; dt < Dh / 8; dt++) {
      o[dt][0] *= ca;
      o[dt][1] *= ca;
      o[dt][2] *= cb;
      o[dt][3] *= cb;
    }
    // O += P V: P (fp16) from the score registers, V fragments transposed
#pragma unroll
    for (int j = 0; j < 4; j++) {  // keys 16 j .. 16 j + 15
      const uint32_t pa[4] = {pack_h2(s[2 * j][0], s[2 * j][1]), pack_h2(s[2 * j][2], s[2 * j][3]),
                              pack_h2(s[2 * j + 1][0], s[2 * j + 1][1]), pack_h2(s[2 * j + 1][2], s[2 * j + 1][3])};
#pragma unroll
      for (int dp = 0; dp < Dh / 16; dp++) {
        // matrices: (keys +0..7, dims 16dp..+7), (keys +8..15, dims 16dp..+7),
        //           (keys +0..7, dims +8..15), (keys +8..15, dims +8..15)
        const int key = 16 * j + 8 * (jm & 1) + jr, dim = 16 * dp + 8 * (jm >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vaddr + (uint32_t)(key * kStride + dim) * 2, b0, b1, b2, b3);
        mma_f16(o[2 * dp], pa, b0, b1);
        mma_f16(o[2 * dp + 1], pa, b2, b3);
      }
    }
    __syncthreads();  // the buffer is refilled two tiles on
  }

  la += __shfl_xor_sync(0xffffffffu, la, 1);
  la += __shfl_xor_sync(0xffffffffu, la, 2);
  lb += __shfl_xor_sync(0xffffffffu, lb, 1);
  lb += __shfl_xor_sync(0xffffffffu, lb, 2);
  const float ia = la > 0.0f ? 1.0f / la : 0.0f, ib = lb > 0.0f ? 1.0f / lb : 0.0f;
  const bool va = i0 + g < rps, vb = i0 + g + 8 < rps;
  __half *oa = out + ((size_t)(b * rps + i0 + g) * H + h) * Dh;
  __half *ob = out + ((size_t)(b * rps + i0 + g + 8) * H + h) * Dh;
#pragma unroll
  for (int dt = 0; dt < Dh / 8; dt++) {
    if (va) *reinterpret_cast<uint32_t *>(oa + 8 * dt + 2 * t) = pack_h2(o[dt][0] * ia, o[dt][1] * ia);
    if (vb) *reinterpret_cast<uint32_t *>(ob + 8 * dt + 2 * t) = pack_h2(o[dt][2] * ib, o[dt][3] * ib);
  }
}

template <int Dh>
cudaError_t launch_fa(const void *q, int rps, int batch, int H, int Hkv, const void *k_cache, const void *v_cache,
                      int cache_len, const int *pos0, void *out, cudaStream_t s, bool pdl) {
  const size_t smem = (size_t)4 * kFaKeys * (Dh + 8) * sizeof(__half);
  auto kern = flash_prefill_kernel<Dh>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((rps + kFaRows - 1) / kFaRows), (unsigned)H, (unsigned)batch);
  cfg.blockDim = dim3(kFaThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  if (pdl) {
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kern, reinterpret_cast<const __half *>(q), rps, H, Hkv,
                            reinterpret_cast<const __half *>(k_cache), reinterpret_cast<const __half *>(v_cache),
                            cache_len, pos0, reinterpret_cast<__half *>(out));
}

}  // namespace

bool flash_prefill_supported(int rps, int Dh) { return rps >= kFaPrefillMinRows && (Dh == 64 || Dh == 128); }

cudaError_t launch_flash_prefill(const void *q, int rps, int batch, int H, int Hkv, int Dh, const void *k_cache,
                                 const void *v_cache, int cache_len, const int *pos0, void *out, cudaStream_t s,
                                 bool pdl) {
  if (H % Hkv || !flash_prefill_supported(rps, Dh)) return cudaErrorInvalidValue;
  return Dh == 64 ? launch_fa<64>(q, rps, batch, H, Hkv, k_cache, v_cache, cache_len, pos0, out, s, pdl)
                  : launch_fa<128>(q, rps, batch, H, Hkv, k_cache, v_cache, cache_len, pos0, out, s, pdl);
}

}  // namespace wg
