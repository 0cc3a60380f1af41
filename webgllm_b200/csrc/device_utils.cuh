// Device helpers shared by the Q4 kernels: mbarriers with bounded waits,
// bulk async copies (the TMA engine, one destination CTA), fp16 bit tricks.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "common.cuh"

namespace wg {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// ---- mbarriers -------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Makes mbarrier initialisation visible to the async proxy (bulk copies).
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One try: the thread may be suspended (not spinning, not issuing) for a
// system-dependent time while the phase is incomplete. (With a 1 ms
// suspend-time hint every pipeline measured slower on B200: the Q4 GEMM at
// M = 1024, 4096^2, 39.9 vs 37.4 us a launch; the M = 1 GEMV chain 3.89 vs
// 3.82 us.)
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for phase `parity` of `bar` for at most ~`limit_cycles` SM cycles.
// On timeout raises kFlagTimeout in `flags` and returns false: the caller
// carries on with whatever is in shared memory and the host reports
// WG_TIMEOUT; nothing spins forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, unsigned *flags,
                                                  long long limit_cycles = 2000000000LL) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > limit_cycles) {
      raise_flag(flags, kFlagTimeout);
      return false;
    }
  }
  return true;
}

// ---- bulk async copy global -> shared (the TMA engine, one destination CTA)

// `bytes` a multiple of 16, both addresses 16-byte aligned.
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---- programmatic dependent launch ----------------------------------------

// 16-byte asynchronous global -> shared copy (cp.async, bypassing L1), and
// the wait for all of this thread's outstanding ones.
__device__ __forceinline__ void cp_async16(void *dst_smem, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Bulk prefetch of [p, p + bytes) into L2 (a hint; 16-byte aligned, bytes a
// multiple of 16).
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

// ---- tracing (wg_trace) ----------------------------------------------------

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned smid() {
  unsigned r;
  asm volatile("mov.u32 %0, %smid;" : "=r"(r));
  return r;
}

// One record: six timestamps, the SM id, (launch << 32 | cta).
__device__ __forceinline__ void trace_record(unsigned long long *buf, unsigned long long *next,
                                             unsigned long long cap, const unsigned long long ts[6],
                                             unsigned launch, unsigned cta) {
  const unsigned long long i = atomicAdd(next, 1ull);
  if (i >= cap) return;
  unsigned long long *r = buf + i * 8;
#pragma unroll
  for (int k = 0; k < 6; k++) r[k] = ts[k];
  r[6] = smid();
  r[7] = ((unsigned long long)launch << 32) | cta;
}

// ---- fp16 helpers ----------------------------------------------------------

// (a & b) | c
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t hmul2_u(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

// Zero-point constants of one row's block: lo = 1024 + z (subtracted from
// 1024 + q, exact), hi = -(64 + z) (added to (1024 + 16 q) / 16, exact),
// both as half2.
__device__ __forceinline__ uint32_t zp_lo(uint32_t z) { return (0x6400u | z) * 0x00010001u; }
__device__ __forceinline__ uint32_t zp_hi(uint32_t z) { return (0xD400u | (z << 4)) * 0x00010001u; }
constexpr uint32_t kZpLo8 = 0x64086408u;  // 1032.0h x2
constexpr uint32_t kZpHi8 = 0xD480D480u;  // -72.0h x2

// One word of codes (q4_layout.cuh) -> (q - z) as exact fp16 pairs:
//   P[0] = (row g, e 0-1), P[1] = (row g, e 2-3),
//   P[2] = (row g+8, e 0-1), P[3] = (row g+8, e 2-3).
__device__ __forceinline__ void unpack_codes(uint32_t w, uint32_t lo_g, uint32_t hi_g, uint32_t lo_g8,
                                             uint32_t hi_g8, uint32_t P[4]) {
  const uint32_t kMagic = 0x64006400u;      // 1024.0h x2
  const uint32_t kSixteenth = 0x2C002C00u;  // 0.0625h x2
  const uint32_t w8 = w >> 8;
  P[0] = hsub2_u(and_or(w, 0x000F000Fu, kMagic), lo_g);
  P[1] = hfma2_u(and_or(w, 0x00F000F0u, kMagic), kSixteenth, hi_g);
  P[2] = hsub2_u(and_or(w8, 0x000F000Fu, kMagic), lo_g8);
  P[3] = hfma2_u(and_or(w8, 0x00F000F0u, kMagic), kSixteenth, hi_g8);
}

// One word of codes -> the raw pairs (1024 + q) (e 0-1 of each row, from the
// low nibbles) and (64 + q) (e 2-3, from the high nibbles: the exponent of
// 64.0h puts mantissa bits 4-7 at weight 1), exact fp16, in P's order; the
// offsets (1024 + z, 64 + z) are subtracted by a second MMA against the same
// activations (tile_mma).
__device__ __forceinline__ void unpack_codes_raw(uint32_t w, uint32_t P[4]) {
  const uint32_t w8 = w >> 8;
  P[0] = and_or(w, 0x000F000Fu, 0x64006400u);
  P[1] = and_or(w, 0x00F000F0u, 0x54005400u);
  P[2] = and_or(w8, 0x000F000Fu, 0x64006400u);
  P[3] = and_or(w8, 0x00F000F0u, 0x54005400u);
}

__device__ __forceinline__ float clamp_half(float v) { return fminf(fmaxf(v, -65504.0f), 65504.0f); }

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(clamp_half(a), clamp_half(b));
  return *reinterpret_cast<uint32_t *>(&h);
}

// Eight activations of any dtype as fp16 (saturating like packH2), 16 bytes.
__device__ __forceinline__ uint4 load_x8_f16(const void *x, int dtype, size_t off) {
  uint4 v;
  if (dtype == WG_F16) {
    v = *reinterpret_cast<const uint4 *>(reinterpret_cast<const __half *>(x) + off);
  } else if (dtype == WG_F32) {
    const float4 *p = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(x) + off);
    const float4 f0 = p[0], f1 = p[1];
    v.x = pack_half2(f0.x, f0.y);
    v.y = pack_half2(f0.z, f0.w);
    v.z = pack_half2(f1.x, f1.y);
    v.w = pack_half2(f1.z, f1.w);
  } else {
    const uint4 raw = *reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(x) + off);
    const __nv_bfloat162 *b = reinterpret_cast<const __nv_bfloat162 *>(&raw);
    const float2 f0 = __bfloat1622float2(b[0]), f1 = __bfloat1622float2(b[1]);
    const float2 f2 = __bfloat1622float2(b[2]), f3 = __bfloat1622float2(b[3]);
    v.x = pack_half2(f0.x, f0.y);
    v.y = pack_half2(f1.x, f1.y);
    v.z = pack_half2(f2.x, f2.y);
    v.w = pack_half2(f3.x, f3.y);
  }
  return v;
}

__device__ __forceinline__ void store_out(void *y, int dtype, size_t off, float v) {
  if (dtype == WG_F32) reinterpret_cast<float *>(y)[off] = v;
  else if (dtype == WG_F16) reinterpret_cast<__half *>(y)[off] = __float2half_rn(clamp_half(v));
  else reinterpret_cast<__nv_bfloat16 *>(y)[off] = __float2bfloat16_rn(v);
}

}  // namespace wg
