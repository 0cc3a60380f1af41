// The Q4 decode GEMV (M <= 32 rows of activations): y = x . W^T.
//
// Replaces the reference's split matmul (src/engine.ts:5241-5391 dispatching
// matmulSplitRgba4, src/gpu/kernels.ts:744-895, or matmul({split: true}),
// kernels.ts:163-296) and its consumers' slice reduction (pf,
// kernels.ts:69-79): the K-slices are summed on chip, not written as fp16
// partials.
//
// Design (HBM-bound: 0.5625 bytes of weights per multiply-add at M = 1):
// - A CTA of 8 warps owns one 16-row tile column (16 outputs) and a range of
//   K tiles (all of K unless K is large, then a thread-block cluster splits
//   it). Its first thread starts bulk asynchronous copies (the TMA engine) of
//   the whole range's codes and scales into shared memory, in chunks of 8
//   tiles with one mbarrier each, before anything waits: weight streaming
//   needs no registers and does not depend on the kernel that produced x.
// - The CTA then triggers its dependents (programmatic dependent launch) and
//   only afterwards waits for x's producer, so in a chain of matmuls the next
//   one's weight copies are in flight while this one finishes. The kernel
//   keeps to a fraction of an SM (<= 64 registers a thread, modest shared
//   memory) so that the next kernel's CTAs can be resident at the same time.
// - Codes become exact fp16 (q - z) in registers (q4_layout.cuh), x is staged
//   once as fp16 in shared memory, and mma.m16n8k16 (fp32 accumulate)
//   multiplies each 32-weight block into a fresh accumulator that is scaled
//   by the block's scale in fp32: the reference's per-block arithmetic
//   d * (sum q*a - z * sum a) (kernels.ts:182-217) without its fp16
//   partials.
// - The 8 warps' partial tiles are summed in shared memory; across a cluster
//   through distributed shared memory (no atomics, no global scratch).
#include <cooperative_groups.h>

#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "device_utils.cuh"
#include "q4_kernels.cuh"

namespace cg = cooperative_groups;

namespace wg {

namespace {

// Codes unpacked to raw (1024 + q) / (64 + q) pairs with the offsets taken
// off by a second MMA (5 instead of 9 instructions a word, one more MMA a K
// step; up to 16 rows), or to exact (q - z) pairs. Measured on B200 (64-launch
// graphs): raw is slower — M = 1 at 4096^2 4.18 -> 4.67 us, M = 16 8.6 ->
// 9.9 us, config-4 decode step 3.19 -> 3.34 ms: the second mma.sync costs
// more tensor-pipe time (one per ~10 cycles a sub-partition) than the four
// ALU instructions it saves. Kept off.
constexpr bool kRawUnpack = false;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
// Up to 16 tiles a warp: K up to 8192 in one CTA at one row (the smem budget
// lowers it for more rows). A K split across a cluster costs its two cluster
// barriers and the remote reads (~1.5 us a launch on B200) and is only used
// where the range does not fit.
constexpr int kMaxTilesPerWarp = 16;
constexpr int kMaxTilesPerCta = kWarps * kMaxTilesPerWarp;
constexpr int kSmemBudget = 100 * 1024;  // per CTA, so that two kernels' CTAs fit an SM
constexpr int kMaxSmem = 200 * 1024;

struct GemvSmem {
  int nib, scl, zro, x, red, bar, total;
  int tpw;       // tiles per warp
  int x_stride;  // halves per staged token row (per warp)
  int x_warp;    // halves per warp's x slice
};

__host__ __device__ inline int align_to(int v, int a) { return (v + a - 1) / a * a; }

// Shared memory of one CTA with a K range of `ktc` tiles (the planned range:
// every CTA of a grid uses the same layout, so that the cluster reduction
// can address a peer's `part` at its own offset).
__host__ __device__ inline GemvSmem gemv_smem(int M, int ktc, int NG, bool zeros) {
  GemvSmem s;
  s.tpw = (ktc + kWarps - 1) / kWarps;
  s.nib = 0;
  s.scl = s.nib + ktc * kTileNibBytes;
  s.zro = s.scl + ktc * kTileSclBytes;
  s.x = align_to(s.zro + (zeros ? ktc * kTileZroBytes : 0), 128);
  // +16 halves (32 bytes) per row: the 8-byte fragment loads of 8 rows by 4
  // threads hit 32 distinct banks.
  s.x_stride = s.tpw * kTileK + 16;
  s.x_warp = M * s.x_stride;
  s.red = align_to(s.x + kWarps * s.x_warp * 2, 128);
  s.bar = align_to(s.red + (kWarps * NG * 128 + 128 * NG) * 4, 8);
  s.total = s.bar + 2 * kWarps * 8;  // a weight and an x barrier per warp
  return s;
}

__device__ __forceinline__ void mma_16816(float d[4], const uint32_t a0, const uint32_t a1,
                                          const uint32_t a2, const uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One 16 x 64 tile: four K steps of mma.m16n8k16 per token group, two
// 32-weight blocks each scaled in fp32 into acc.
// SPLIT: the block's two 16-wide K steps accumulate separately (two
// independent MMAs, then added), for kernels with few warps to hide the MMA
// latency; otherwise they chain into one accumulator.
template <int NG, bool ZEROS, bool SPLIT = false>
__device__ __forceinline__ void tile_mma(const uint8_t *s_nib, const uint8_t *s_scl, const uint8_t *s_zro,
                                         const __half *xt, int stride, int M, int lane, float acc[NG][4]) {
  const int g = lane >> 2;
  const uint4 wv = *reinterpret_cast<const uint4 *>(s_nib + lane * 16);
  const uint2 sv = *reinterpret_cast<const uint2 *>(s_scl + g * 8);
  uint32_t zv = 0;
  if (ZEROS) zv = *reinterpret_cast<const uint32_t *>(s_zro + g * 4);
  const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
  for (int bsel = 0; bsel < 2; bsel++) {
    uint32_t lo_g = kZpLo8, hi_g = kZpHi8, lo_g8 = kZpLo8, hi_g8 = kZpHi8;
    if (ZEROS) {
      const uint32_t zz = zv >> (16 * bsel);
      lo_g = zp_lo(zz & 15u);
      hi_g = zp_hi(zz & 15u);
      lo_g8 = zp_lo((zz >> 8) & 15u);
      hi_g8 = zp_hi((zz >> 8) & 15u);
    }
    float blk[2][NG][4];
#pragma unroll
    for (int js = 0; js < 2; js++)
#pragma unroll
      for (int ng = 0; ng < NG; ng++)
#pragma unroll
        for (int e = 0; e < 4; e++) blk[js][ng][e] = 0.0f;
#pragma unroll
    for (int js = 0; js < 2; js++) {
      const int j = 2 * bsel + js;
      uint32_t P[4];
      if (kRawUnpack && NG <= 2)
        unpack_codes_raw(w[j], P);
      else
        unpack_codes(w[j], lo_g, hi_g, lo_g8, hi_g8, P);
#pragma unroll
      for (int ng = 0; ng < NG; ng++) {
        const int tok = ng * 8 + g;
        uint2 b = make_uint2(0, 0);
        if (tok < M) b = *reinterpret_cast<const uint2 *>(xt + (size_t)tok * stride + 16 * j);
        // fragment k {2t,2t+1 | 2t+8,2t+9} <-> K offset {4t,4t+1 | 4t+2,4t+3}
        mma_16816(blk[SPLIT ? js : 0][ng], P[0], P[2], P[1], P[3], b.x, b.y);
        // raw codes: minus (1024 + z) x on e 0-1 and (64 + z) x on e 2-3
        if (kRawUnpack && NG <= 2) mma_16816(blk[SPLIT ? js : 0][ng], lo_g ^ 0x80008000u, lo_g8 ^ 0x80008000u, hi_g, hi_g8, b.x, b.y);
      }
    }
    const uint32_t sp = bsel ? sv.y : sv.x;
    const float2 sc = __half22float2(*reinterpret_cast<const __half2 *>(&sp));
#pragma unroll
    for (int ng = 0; ng < NG; ng++) {
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float v = SPLIT ? blk[0][ng][e] + blk[1][ng][e] : blk[0][ng][e];
        acc[ng][e] = fmaf(e < 2 ? sc.x : sc.y, v, acc[ng][e]);
      }
    }
  }
}

// Barrier `id` (1..15) over the `threads` threads (a multiple of 32) of the
// warps that reach it.
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

// The final value of output row n (tile nt, row r) for token tok: stored,
// pushed to the exchange, or (SwiGLU pairs, only rows r < 8 of a tile,
// given the paired up value) activated into y [M][N/2].
__device__ __forceinline__ void emit(const GemvArgs &a, unsigned parity, int nt, int r, int tok, float v) {
  const int n = nt * kTileRows + r;
  if (n >= a.N || tok >= a.M) return;
  if (a.push_on)
    push_store(a.push, parity, n, tok, a.M, v);
  else
    store_out(a.y, a.y_dtype, (size_t)tok * a.N + n, v);
}
__device__ __forceinline__ void emit_pair(const GemvArgs &a, int nt, int r, int tok, float gate, float up) {
  const int f = nt * (kTileRows / 2) + r;  // feature: tile nt holds gate / up rows of features 8nt .. 8nt+7
  if (nt * kTileRows + r >= a.N || tok >= a.M) return;
  store_out(a.y, a.y_dtype, (size_t)tok * (a.N / 2) + f, silu_mul(gate, up));
}

// The residual epilogue (kEpiResidual): y fp32 [M][N] += v, returning the
// new value (0 for padding rows and tokens past M, which add nothing to the
// statistics).
__device__ __forceinline__ float emit_residual(const GemvArgs &a, int nt, int r, int tok, float v) {
  const int n = nt * kTileRows + r;
  if (n >= a.N || tok >= a.M) return 0.0f;
  float *y = reinterpret_cast<float *>(a.y) + (size_t)tok * a.N + n;
  v += *y;
  *y = v;
  return v;
}

// Tile nt's statistics from sq[r * 8 + tok] = (new residual)^2 of its 16
// rows (one token group): stats[nt][tok] = the sum over r, in order. Called
// by threads 0 .. M-1 after a barrier.
__device__ __forceinline__ void emit_stats(const GemvArgs &a, int nt, int tok, const float *sq) {
  float t = 0.0f;
#pragma unroll
  for (int r = 0; r < kTileRows; r++) t += sq[r * 8 + tok];
  a.stats[(size_t)nt * a.M + tok] = t;
}

// Eight consecutive x values (row m, columns k..k+7) as fp16, made by the
// prologue: (residual + b) * inv * w for the norm, silu(gate) * up for SwiGLU.
// The norm of eight values: fp16((v * inv) * w), the one place this
// arithmetic is written (every staging path gives the same bits).
__device__ __forceinline__ uint4 norm_x8(float4 v0, float4 v1, float4 w0, float4 w1, float inv) {
  float f[8];
  f[0] = v0.x * inv * w0.x; f[1] = v0.y * inv * w0.y; f[2] = v0.z * inv * w0.z; f[3] = v0.w * inv * w0.w;
  f[4] = v1.x * inv * w1.x; f[5] = v1.y * inv * w1.y; f[6] = v1.z * inv * w1.z; f[7] = v1.w * inv * w1.w;
  return make_uint4(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]), pack_half2(f[4], f[5]), pack_half2(f[6], f[7]));
}

template <int PRO>
__device__ __forceinline__ uint4 prologue_x8(const Prologue &p, int K, int m, int k, float inv) {
  float f[8];
  if (PRO == kProRmsNorm) {
    const float4 *r = reinterpret_cast<const float4 *>(p.a + (size_t)m * K + k);
    float4 v0 = r[0], v1 = r[1];
    if (p.b) {
      const float4 *b = reinterpret_cast<const float4 *>(p.b + (size_t)m * K + k);
      v0 = add4(v0, b[0]);
      v1 = add4(v1, b[1]);
    }
    const float4 w0 = reinterpret_cast<const float4 *>(p.w + k)[0], w1 = reinterpret_cast<const float4 *>(p.w + k)[1];
    return norm_x8(v0, v1, w0, w1, inv);
  } else {
    const float4 *g = reinterpret_cast<const float4 *>(p.a + (size_t)m * 2 * K + k);
    const float4 *u = reinterpret_cast<const float4 *>(p.a + (size_t)m * 2 * K + K + k);
    const float4 g0 = g[0], g1 = g[1], u0 = u[0], u1 = u[1];
    f[0] = silu_mul(g0.x, u0.x); f[1] = silu_mul(g0.y, u0.y); f[2] = silu_mul(g0.z, u0.z); f[3] = silu_mul(g0.w, u0.w);
    f[4] = silu_mul(g1.x, u1.x); f[5] = silu_mul(g1.y, u1.y); f[6] = silu_mul(g1.z, u1.z); f[7] = silu_mul(g1.w, u1.w);
  }
  return make_uint4(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]), pack_half2(f[4], f[5]), pack_half2(f[6], f[7]));
}

// The norm prologue's row statistics: inv[m] = 1 / sqrt(mean((residual +
// b)^2) + eps) over all of K, for every row (all threads of the CTA), and
// the residual sum written out by a grid-strided share of every CTA.
template <int NW = kWarps>
__device__ void rmsnorm_rows(const Prologue &p, int M, int K, float *s_part, float *s_inv) {
  constexpr int kThreads = NW * 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K4 = K / 4;
  if (p.stats) {
    // the producer's per-tile sums of squares (a fixed order: deterministic)
    static_assert(NW >= kProMaxTokens, "a warp per row");
    if (warp < M) {
      float t = 0.0f;
      for (int i = lane; i < K / kTileRows; i += 32) t += p.stats[(size_t)i * M + warp];
      t = warp_sum_f(t);
      if (lane == 0) s_inv[warp] = rsqrtf(t / (float)K + p.eps);
    }
    __syncthreads();
    return;
  }
  for (int m = 0; m < M; m++) {
    const float4 *r = reinterpret_cast<const float4 *>(p.a + (size_t)m * K);
    const float4 *b = p.b ? reinterpret_cast<const float4 *>(p.b + (size_t)m * K) : nullptr;
    float ss = 0.0f;
#pragma unroll 4
    for (int i = threadIdx.x; i < K4; i += kThreads) {
      float4 v = r[i];
      if (b) v = add4(v, b[i]);
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = warp_sum_f(ss);
    if (lane == 0) s_part[warp * kProMaxTokens + m] = ss;
  }
  if (p.out) {
    const int ncta = gridDim.x * gridDim.y, cta = blockIdx.y * gridDim.x + blockIdx.x;
    const float4 *r = reinterpret_cast<const float4 *>(p.a);
    const float4 *b = reinterpret_cast<const float4 *>(p.b);
    float4 *o = reinterpret_cast<float4 *>(p.out);
    for (int i = cta * kThreads + threadIdx.x; i < M * K4; i += ncta * kThreads) o[i] = b ? add4(r[i], b[i]) : r[i];
  }
  __syncthreads();
  if (threadIdx.x < M) {
    float t = 0.0f;
    for (int w = 0; w < NW; w++) t += s_part[w * kProMaxTokens + threadIdx.x];
    s_inv[threadIdx.x] = rsqrtf(t / (float)K + p.eps);
  }
  __syncthreads();
}

template <int NG, bool ZEROS, int PRO>
__global__ void __launch_bounds__(kThreads, NG == 1 ? 4 : 2) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = lane & 3;
  const int nt = blockIdx.y;
  const int crank = blockIdx.x;
  const int kt0 = crank * a.kt_per_cta;
  const int kt1 = min(a.KT, kt0 + a.kt_per_cta);
  const int ktc = kt1 - kt0;  // >= 1 (plan_gemv)
  const GemvSmem L = gemv_smem(a.M, a.kt_per_cta, NG, ZEROS);
  // This warp's tiles: [wt0, wt1) of the CTA's range, contiguous in memory.
  const int wt0 = min(ktc, warp * L.tpw);
  const int wt1 = min(ktc, wt0 + L.tpw);
  const int nw = wt1 - wt0;
  uint8_t *s_nib = smem + L.nib;
  uint8_t *s_scl = smem + L.scl;
  uint8_t *s_zro = smem + L.zro;
  __half *xw = reinterpret_cast<__half *>(smem + L.x) + warp * L.x_warp;
  float *red = reinterpret_cast<float *>(smem + L.red);
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem + L.bar) + warp;
  uint64_t *xbar = reinterpret_cast<uint64_t *>(smem + L.bar) + kWarps + warp;
  // fp16 x without a prologue arrives by bulk copy (one per row), else by
  // loads and stores that convert or compute it
  const bool x_bulk = PRO == kProNone && a.x_dtype == WG_F16;
  __shared__ unsigned long long ts[6];  // tracing stamps (thread 0)
  if (a.trace && threadIdx.x == 0) ts[0] = globaltimer();

  // 1. Each warp starts the copies of its own tiles (the TMA engine, one
  //    mbarrier a warp): weights depend on nothing the previous kernel
  //    writes, so this happens before any wait.
  if (lane == 0 && nw > 0) {
    mbar_init(bar, 1);
    if (x_bulk) mbar_init(xbar, 1);
    fence_mbar_init();
    const size_t tile = (size_t)nt * a.KT + kt0 + wt0;
    mbar_expect_tx(bar, nw * (kTileNibBytes + kTileSclBytes + (ZEROS ? kTileZroBytes : 0)));
    bulk_g2s(s_nib + wt0 * kTileNibBytes, reinterpret_cast<const uint8_t *>(a.nib) + tile * kTileNibBytes,
             nw * kTileNibBytes, bar);
    bulk_g2s(s_scl + wt0 * kTileSclBytes, reinterpret_cast<const uint8_t *>(a.scl) + tile * kTileSclBytes,
             nw * kTileSclBytes, bar);
    if (ZEROS)
      bulk_g2s(s_zro + wt0 * kTileZroBytes, a.zro + tile * kTileZroBytes, nw * kTileZroBytes, bar);
  }
  __syncwarp();
  if (a.trace && threadIdx.x == 0) ts[1] = globaltimer();

  // 2. Wait for the kernel that wrote x. The next kernel in the stream is
  //    let in (programmatic dependent launch) at a.trigger_at: 0 here, 1 once
  //    x is staged, 2 after the multiplies. Later is better when its weight
  //    copies would otherwise queue ahead of this kernel's x loads at the
  //    SMs.
  if (a.trigger_at == 0) pdl_trigger();
  pdl_wait();
  if (a.trace && threadIdx.x == 0) ts[2] = globaltimer();
  // The exchange's sequence number, read only after the wait: the previous
  // pushing launch advances it from its last CTA, and that launch is
  // complete only once every kernel this one waits on is.
  const unsigned parity = a.push_on ? push_seq(a.push) : 0u;

  // 3. Each warp stages its own K slice of x[0..M) as fp16 (no CTA barrier,
  //    except for the norm prologue's row statistics).
  const int M = a.M;
  const int stride = L.x_stride;
  __shared__ float s_inv[PRO == kProRmsNorm ? kProMaxTokens : 1];
  if constexpr (PRO == kProRmsNorm) {
    __shared__ float s_part[kWarps * kProMaxTokens];
    rmsnorm_rows(a.pro, M, a.K, s_part, s_inv);
  }
  if (x_bulk) {
    // this warp's K slice of every row: one bulk copy per row (16-byte
    // aligned: K is a multiple of 32, the slice starts at a tile), the
    // partial last tile's columns past K zeroed (padding weights are 0, but
    // 0 * NaN is not)
    if (nw > 0) {
      const int kbase = (kt0 + wt0) * kTileK;
      const int kcols = min(a.K - kbase, nw * kTileK);  // a multiple of 32
      if (lane == 0) {
        mbar_expect_tx(xbar, (uint32_t)(M * kcols * 2));
        for (int m = 0; m < M; m++)
          bulk_g2s(xw + (size_t)m * stride, reinterpret_cast<const __half *>(a.x) + (size_t)m * a.K + kbase,
                   kcols * 2, xbar);
      }
      const int tail = nw * kTileK - kcols;
      for (int i = lane; i < M * tail; i += 32) {
        const int m = i / tail;
        xw[(size_t)m * stride + kcols + (i - m * tail)] = __float2half_rn(0.0f);
      }
      mbar_wait_bounded(xbar, 0, a.flags);
    }
  } else {
    // Up to 4 loads in flight per lane before any store (one L2 round trip
    // for every 128 chunks). Entry idx = m * 128 + c (token m, chunk c of 8
    // K values; a warp has at most 128 chunks), so that shifts, not
    // divisions, split it.
    static_assert(kMaxTilesPerWarp * (kTileK / 8) == 128, "128 chunks per warp at most");
    const int chunks = nw * (kTileK / 8);
    const int kbase = (kt0 + wt0) * kTileK;
    for (int base = 0; base < M * 128; base += 4 * 32) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int idx = base + u * 32 + lane;
        const int m = idx >> 7, c = idx & 127;
        const int k = kbase + c * 8;
        v[u] = make_uint4(0, 0, 0, 0);
        if (m < M && c < chunks && k < a.K) {
          if constexpr (PRO == kProNone)
            v[u] = load_x8_f16(a.x, a.x_dtype, (size_t)m * a.K + k);
          else
            v[u] = prologue_x8<PRO>(a.pro, a.K, m, k, PRO == kProRmsNorm ? s_inv[m] : 0.0f);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int idx = base + u * 32 + lane;
        const int m = idx >> 7, c = idx & 127;
        if (m < M && c < chunks) *reinterpret_cast<uint4 *>(xw + (size_t)m * stride + c * 8) = v[u];
      }
    }
  }
  __syncwarp();
  if (a.trigger_at == 1) pdl_trigger();
  if (a.trace && threadIdx.x == 0) ts[3] = globaltimer();

  // 4. Tensor-core steps over this warp's tiles.
  float acc[NG][4];
#pragma unroll
  for (int ng = 0; ng < NG; ng++)
#pragma unroll
    for (int e = 0; e < 4; e++) acc[ng][e] = 0.0f;
  if (nw > 0) {
    mbar_wait_bounded(bar, 0, a.flags);
#pragma unroll 2
    for (int i = 0; i < nw; i++) {
      const int ti = wt0 + i;
      tile_mma<NG, ZEROS>(s_nib + ti * kTileNibBytes, s_scl + ti * kTileSclBytes, s_zro + ti * kTileZroBytes,
                          xw + i * kTileK + 4 * t, stride, M, lane, acc);
    }
  }

  if (a.trigger_at == 2) pdl_trigger();

  // 5. Sum the warps' fragments: red[warp][ng][e][lane], then one output
  //    (row r, token) per thread.
  float *part = red + kWarps * NG * 128;
#pragma unroll
  for (int ng = 0; ng < NG; ng++)
#pragma unroll
    for (int e = 0; e < 4; e++) red[((warp * NG + ng) * 4 + e) * 32 + lane] = acc[ng][e];
  __syncthreads();
  if (a.trace && threadIdx.x == 0) ts[4] = globaltimer();
  constexpr int kOut = 16 * 8 * NG;
  const int C = a.cluster;
  auto warp_sum_at = [&](int r, int tok) {  // sum over the 8 warps of output (r, tok)
    const int ng = tok >> 3, tk = tok & 7;
    const int ln = 4 * (r & 7) + (tk >> 1);
    const int e = ((r >> 3) << 1) | (tk & 1);
    float s = 0.0f;
#pragma unroll
    for (int w2 = 0; w2 < kWarps; w2++) s += red[((w2 * NG + ng) * 4 + e) * 32 + ln];
    return s;
  };
  if (C > 1 || a.epi == kEpiNone) {
    for (int o = threadIdx.x; o < kOut; o += kThreads) {
      const int r = o / (8 * NG), tok = o - r * (8 * NG);
      const float s = warp_sum_at(r, tok);
      if (C > 1)
        part[o] = s;
      else
        emit(a, parity, nt, r, tok, s);
    }
  } else {
    for (int o = threadIdx.x; o < kOut / 2; o += kThreads) {
      const int r = o / (8 * NG), tok = o - r * (8 * NG);
      emit_pair(a, nt, r, tok, warp_sum_at(r, tok), warp_sum_at(r + 8, tok));
    }
  }

  // 6. With a K split, rank c sums outputs o = c (mod C) over the cluster's
  //    CTAs through distributed shared memory and writes them.
  if (C > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const int nout = a.epi == kEpiNone ? kOut : kOut / 2;
    for (int o = crank + C * (int)threadIdx.x; o < nout; o += C * kThreads) {
      const int r = o / (8 * NG), tok = o - r * (8 * NG);
      float s = 0.0f, u = 0.0f;
      for (int c = 0; c < C; c++) {
        const float *pc = cluster.map_shared_rank(part, c);
        s += pc[o];
        if (a.epi != kEpiNone) u += pc[o + kOut / 2];  // row r + 8: index + 8 * 8NG
      }
      if (a.epi == kEpiNone)
        emit(a, parity, nt, r, tok, s);
      else
        emit_pair(a, nt, r, tok, s, u);
    }
    cluster.sync();
  }

  // 7. No copy may still be writing this CTA's shared memory when it exits
  //    (only possible after a timed-out wait).
  if (lane == 0 && nw > 0) {
    mbar_wait_bounded(bar, 0, a.flags);
    if (x_bulk) mbar_wait_bounded(xbar, 0, a.flags);
  }
  if (a.push_on) push_signal(a.push);
  if (a.trace && threadIdx.x == 0) {
    ts[5] = globaltimer();
    trace_record(a.trace, a.trace_next, a.trace_cap, ts, a.launch_index, blockIdx.y * gridDim.x + blockIdx.x);
  }
}

template <int NG, bool ZEROS, int PRO = kProNone>
cudaError_t launch_t(const GemvArgs &a, cudaStream_t stream, bool pdl) {
  const GemvSmem L = gemv_smem(a.M, a.kt_per_cta, NG, ZEROS);
  auto kern = gemv_kernel<NG, ZEROS, PRO>;
  // Function attributes once per instantiation (not per launch: launches may
  // be captured into a CUDA graph).
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  if (L.total > kMaxSmem) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.cluster, (unsigned)a.NT, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)L.total;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int n = 0;
  if (a.cluster > 1) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = (unsigned)a.cluster;
    attrs[n].val.clusterDim.y = 1;
    attrs[n].val.clusterDim.z = 1;
    n++;
  }
  if (pdl) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    n++;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

// The prologue on its own, one CTA per row: x fp16 [M][K] for the GEMM path
// (and the residual sum, as in the fused form).
__global__ void __launch_bounds__(kThreads) prologue_kernel(const Prologue p, int K, __half *x) {
  __shared__ float s_part[kWarps * kProMaxTokens];
  __shared__ float s_inv;
  const int m = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float inv = 0.0f;
  if (p.kind == kProRmsNorm) {
    const float4 *r = reinterpret_cast<const float4 *>(p.a + (size_t)m * K);
    const float4 *b = p.b ? reinterpret_cast<const float4 *>(p.b + (size_t)m * K) : nullptr;
    float4 *o = p.out ? reinterpret_cast<float4 *>(p.out + (size_t)m * K) : nullptr;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < K / 4; i += kThreads) {
      float4 v = r[i];
      if (b) v = add4(v, b[i]);
      if (o) o[i] = v;
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = warp_sum_f(ss);
    if (lane == 0) s_part[warp] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.0f;
      for (int w = 0; w < kWarps; w++) t += s_part[w];
      s_inv = rsqrtf(t / (float)K + p.eps);
    }
    __syncthreads();
    inv = s_inv;
  }
  for (int k = threadIdx.x * 8; k < K; k += kThreads * 8) {
    const uint4 v = p.kind == kProRmsNorm ? prologue_x8<kProRmsNorm>(p, K, m, k, inv)
                                          : prologue_x8<kProSwiglu>(p, K, m, k, 0.0f);
    *reinterpret_cast<uint4 *>(x + (size_t)m * K + k) = v;
  }
}

// ---- the wide GEMV: x staged once per CTA, tile columns streamed ---------
//
// For matrices with many 16-row tile columns (or several activation rows),
// the kernel above re-stages x in every CTA of a multi-wave grid: at M = 8
// and N = 28672 that is 8x the weight bytes in L2 reads. Here a grid of about
// one CTA per SM (or cluster of C CTAs when x does not fit: C splits K) keeps
// its x slice resident in shared memory for the whole launch and walks tile
// columns g, g + G, g + 2G, ...; a column's K range is contiguous in each
// plane, so one thread streams whole columns (two or three bulk async
// copies each) through a ring of S stages with one mbarrier per stage, and
// the copies of the next columns are in flight while the 16 warps multiply
// this one (each warp a slice of its K tiles). Per column the warps'
// fragments are summed in shared memory; with a K split, the per-column sums
// stay in shared memory and the cluster reduces them once at the end.

constexpr int kWideXBudget = 96 * 1024;   // x slice per CTA
constexpr int kWideMaxTokens = 32;        // rows (4 token groups of 8)
constexpr int kWideSmemMax = 200 * 1024;
// The two-group column walk (gemv_wide_kernel) wants an even stage count:
// it may use up to this much (the attribute is set to it for every launch).
constexpr int kWideSmemMaxGroups = 224 * 1024;
constexpr int kWWarps = 16;                // warps of a wide CTA (one CTA per SM)
constexpr int kWThreads = kWWarps * 32;

struct WideSmem {
  int x, stage, bars, red, part, total;
  int xstride, stage_bytes;
};

__host__ __device__ inline WideSmem wide_smem(int M, int ktc, int S, int J, int C, bool zeros) {
  WideSmem w;
  const int NG = (M + 7) / 8;
  w.xstride = ktc * kTileK + 16;
  w.stage_bytes = align_to(ktc * (kTileNibBytes + kTileSclBytes + (zeros ? kTileZroBytes : 0)), 128);
  w.x = 0;
  w.stage = align_to(w.x + M * w.xstride * 2, 128);
  w.bars = align_to(w.stage + S * w.stage_bytes, 8);
  w.red = align_to(w.bars + (S + 1) * 8, 16);  // + the x barrier
  w.part = w.red + kWWarps * NG * 128 * 4;
  w.total = w.part + (C > 1 ? J * NG * 128 * 4 : 0);
  return w;
}

template <int NG, bool ZEROS, int PRO>
__global__ void __launch_bounds__(kWThreads, 1) gemv_wide_kernel(const GemvArgs a) {
  if (NG != 1 && a.epi == kEpiResidual) return;  // one token group only (the host checks it too)
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = lane & 3;
  const int C = a.cluster, crank = blockIdx.x;
  const int G = gridDim.y, g = blockIdx.y;
  const int S = a.stages;
  const int kt0 = crank * a.kt_per_cta;
  const int kt1 = min(a.KT, kt0 + a.kt_per_cta);
  const int ktc = kt1 - kt0;
  const int J = (a.NT - g + G - 1) / G;  // columns of this CTA: g, g + G, ...
  const WideSmem L = wide_smem(a.M, a.kt_per_cta, S, a.part_cols, C, ZEROS);
  const int tpw = (a.kt_per_cta + kWWarps - 1) / kWWarps;
  const int wt0 = min(ktc, warp * tpw), wt1 = min(ktc, wt0 + tpw);  // this warp's K tiles
  __half *xs = reinterpret_cast<__half *>(smem + L.x);
  uint8_t *stages = smem + L.stage;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
  uint64_t *xbar = bars + S;
  // fp16 x without a prologue arrives by bulk copy, one per row
  const bool x_bulk = PRO == kProNone && a.x_dtype == WG_F16;
  float *red = reinterpret_cast<float *>(smem + L.red);
  float *part = reinterpret_cast<float *>(smem + L.part);
  const int nib_b = ktc * kTileNibBytes, scl_b = ktc * kTileSclBytes;
  __shared__ unsigned long long ts[6];  // tracing stamps (thread 0)
  if (a.trace && threadIdx.x == 0) ts[0] = globaltimer();

  // column g + j*G (this CTA's K range) into stage st (j % S, or the warp
  // groups' own rings: the first S columns land in stage j either way)
  auto issue_to = [&](int j, int st) {
    uint8_t *dst = stages + st * L.stage_bytes;
    const size_t tile = (size_t)(g + j * G) * a.KT + kt0;
    mbar_expect_tx(&bars[st], nib_b + scl_b + (ZEROS ? ktc * kTileZroBytes : 0));
    bulk_g2s(dst, reinterpret_cast<const uint8_t *>(a.nib) + tile * kTileNibBytes, nib_b, &bars[st]);
    bulk_g2s(dst + nib_b, reinterpret_cast<const uint8_t *>(a.scl) + tile * kTileSclBytes, scl_b, &bars[st]);
    if (ZEROS) bulk_g2s(dst + nib_b + scl_b, a.zro + tile * kTileZroBytes, ktc * kTileZroBytes, &bars[st]);
  };
  auto issue = [&](int j) { issue_to(j, j % S); };

  // 1. Weight copies of the first column: they depend on nothing the
  //    previous kernel writes. The other first S columns follow x: copies
  //    issued ahead of x's would delay it by their bytes at this SM's share
  //    of HBM (measured on B200, M = 8 chains with fp16 x: 6144x4096 7.14 ->
  //    6.46 us, 28672x4096 19.8 -> 18.2 us, 4096x14336 15.8 -> 14.5 us; the
  //    norm prologue's x in the config-4 decode step, wg_trace: gate|up
  //    6.7 -> 5.4 us a CTA, the step 1.2 % shorter).
  if (threadIdx.x == 0) {
    for (int st = 0; st <= S; st++) mbar_init(&bars[st], 1);  // stages and x
    fence_mbar_init();
    if (J > 0) issue(0);
  }
  __syncthreads();
  if (a.trace && threadIdx.x == 0) ts[1] = globaltimer();

  // 2. x (or its prologue) for this CTA's K range, once.
  pdl_wait();
  if (a.trace && threadIdx.x == 0) ts[2] = globaltimer();
  // read after the wait, as in gemv_kernel
  const unsigned parity = a.push_on ? push_seq(a.push) : 0u;
  const int M = a.M;
  __shared__ float s_inv[kProMaxTokens];
  if constexpr (PRO == kProRmsNorm) {
    __shared__ float s_part[kWWarps * kProMaxTokens];
    rmsnorm_rows<kWWarps>(a.pro, M, a.K, s_part, s_inv);
  }
  if (x_bulk) {
    const int kbase = kt0 * kTileK;
    const int kcols = min(a.K - kbase, ktc * kTileK);  // a multiple of 32
    if (threadIdx.x == 0) {
      mbar_expect_tx(xbar, (uint32_t)(M * kcols * 2));
      for (int m = 0; m < M; m++)
        bulk_g2s(xs + (size_t)m * L.xstride, reinterpret_cast<const __half *>(a.x) + (size_t)m * a.K + kbase,
                 kcols * 2, xbar);
      for (int j = 1; j < min(S, J); j++) issue(j);  // the rest of the first S columns, after x
    }
    // the partial last tile reads zeros past K
    const int tail = ktc * kTileK - kcols;
    for (int i = threadIdx.x; i < M * tail; i += kWThreads) {
      const int m = i / tail;
      xs[(size_t)m * L.xstride + kcols + (i - m * tail)] = __float2half_rn(0.0f);
    }
    mbar_wait_bounded(xbar, 0, a.flags);
  } else if (PRO == kProRmsNorm && !a.wide_norm_rows) {
    // The norm: the weight is the same for every row, so a thread takes one
    // chunk of 8 columns for the rows, loading its 8 weights once and four
    // rows' residuals at a time (10 loads in flight), instead of the weights
    // again with every row.
    constexpr int kRowsAtOnce = 4;
    const int chunks = ktc * (kTileK / 8);
    const int kbase = kt0 * kTileK;
    for (int c = threadIdx.x; c < chunks; c += kWThreads) {
      const int k = kbase + c * 8;
      if (k >= a.K) {  // the partial last tile: zeros past K
        for (int m = 0; m < M; m++) *reinterpret_cast<uint4 *>(xs + (size_t)m * L.xstride + c * 8) = make_uint4(0, 0, 0, 0);
        continue;
      }
      const float4 w0 = reinterpret_cast<const float4 *>(a.pro.w + k)[0];
      const float4 w1 = reinterpret_cast<const float4 *>(a.pro.w + k)[1];
      for (int m0 = 0; m0 < M; m0 += kRowsAtOnce) {
        float4 v[kRowsAtOnce][2];
#pragma unroll
        for (int i = 0; i < kRowsAtOnce; i++)
          if (m0 + i < M) {
            const float4 *r = reinterpret_cast<const float4 *>(a.pro.a + (size_t)(m0 + i) * a.K + k);
            v[i][0] = r[0];
            v[i][1] = r[1];
            if (a.pro.b) {
              const float4 *b = reinterpret_cast<const float4 *>(a.pro.b + (size_t)(m0 + i) * a.K + k);
              v[i][0] = add4(v[i][0], b[0]);
              v[i][1] = add4(v[i][1], b[1]);
            }
          }
#pragma unroll
        for (int i = 0; i < kRowsAtOnce; i++)
          if (m0 + i < M)
            *reinterpret_cast<uint4 *>(xs + (size_t)(m0 + i) * L.xstride + c * 8) =
                norm_x8(v[i][0], v[i][1], w0, w1, s_inv[m0 + i]);
      }
    }
  } else {
    // entry idx = m << sh | c (token m, chunk c of 8 K values, 2^sh >=
    // chunks): shifts, not divisions, split it
    const int chunks = ktc * (kTileK / 8);
    const int kbase = kt0 * kTileK;
    int sh = 0;
    while ((1 << sh) < chunks) sh++;
    for (int base = 0; base < (M << sh); base += 4 * kWThreads) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int idx = base + u * kWThreads + threadIdx.x;
        const int m = idx >> sh, c = idx & ((1 << sh) - 1);
        const int k = kbase + c * 8;
        v[u] = make_uint4(0, 0, 0, 0);
        if (m < M && c < chunks && k < a.K) {
          if constexpr (PRO == kProNone)
            v[u] = load_x8_f16(a.x, a.x_dtype, (size_t)m * a.K + k);
          else
            v[u] = prologue_x8<PRO>(a.pro, a.K, m, k, PRO == kProRmsNorm ? s_inv[m] : 0.0f);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int idx = base + u * kWThreads + threadIdx.x;
        const int m = idx >> sh, c = idx & ((1 << sh) - 1);
        if (m < M && c < chunks) *reinterpret_cast<uint4 *>(xs + (size_t)m * L.xstride + c * 8) = v[u];
      }
    }
  }
  // x made by a prologue (loads, not a copy): the rest of the first S
  // columns once its loads are done
  if (!x_bulk && threadIdx.x == 0)
    for (int j = 1; j < min(S, J); j++) issue(j);
  __syncthreads();
  if (a.trigger_at <= 1) pdl_trigger();
  if (a.trace && threadIdx.x == 0) ts[3] = globaltimer();

  // 3. Columns. With a K split, the per-column sums wait in `part` (Jc
  //    columns at a time) and the cluster reduces them a chunk at a time:
  //    rank c takes entries c, c + C, ... of the chunk.
  constexpr int kOut = 16 * 8 * NG;
  const int Jc = a.part_cols;
  __shared__ float sq[2][128];  // kEpiResidual: a column's squared new residuals, per warp group
  auto flush = [&](int j0, int j1) {  // columns [j0, j1), all CTAs of the cluster together
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (a.epi == kEpiResidual) {
      // whole columns per rank (column jj to rank jj mod C), so that a
      // column's statistics sum in one CTA
      for (int jj = crank; jj < j1 - j0; jj += C) {
        const int nt = g + (j0 + jj) * G;
        for (int o = threadIdx.x; o < kOut; o += kWThreads) {
          const int r = o / (8 * NG), tok = o - r * (8 * NG);
          float sum = 0.0f;
          for (int c = 0; c < C; c++) sum += cluster.map_shared_rank(part, c)[jj * kOut + o];
          const float v = emit_residual(a, nt, r, tok, sum);
          sq[0][o] = v * v;
        }
        __syncthreads();
        if ((int)threadIdx.x < M) emit_stats(a, nt, threadIdx.x, sq[0]);
        __syncthreads();
      }
      cluster.sync();
      return;
    }
    const int per = a.epi == kEpiNone ? kOut : kOut / 2;  // outputs per column
    for (int idx = crank + C * (int)threadIdx.x; idx < (j1 - j0) * per; idx += C * kWThreads) {
      const int jj = idx / per, o = idx - jj * per;
      const int r = o / (8 * NG), tok = o - r * (8 * NG);
      float sum = 0.0f, up = 0.0f;
      for (int c = 0; c < C; c++) {
        const float *pc = cluster.map_shared_rank(part, c) + jj * kOut;
        sum += pc[o];
        if (a.epi != kEpiNone) up += pc[o + kOut / 2];  // row r + 8: index + 8 * 8NG
      }
      if (a.epi == kEpiNone)
        emit(a, parity, g + (j0 + jj) * G, r, tok, sum);
      else
        emit_pair(a, g + (j0 + jj) * G, r, tok, sum, up);
    }
    cluster.sync();
  };
  if (a.wide_groups) {
    // (planned with an even S, and with a K split only when `part` holds
    // every column of the walk.) Two independent
    // groups of 8 warps take alternate columns (group 0 the even ones), each
    // with its own named barrier, its half of `red` and its own ring of S / 2
    // stages (group q: stages q, q + 2, ...): a group's barriers wait for 8
    // warps, not 16, one group's barrier and reduction overlap the other
    // group's multiplies, and every stage is filled and drained by one group
    // in column order, so a parity wait is never two phases behind. The
    // group refills the stage it has just drained with its column j + S.
    const int grp = warp >> 3, gw = warp & 7, gtid = threadIdx.x & 255;
    const int Sg = S >> 1;
    const int gtpw = (ktc + 7) / 8;
    const int gt0 = min(ktc, gw * gtpw), gt1 = min(ktc, gt0 + gtpw);
    float *gred = red + grp * (8 * NG * 128);
    int l = 0;  // the group's column count
    for (int j = grp; j < J; j += 2, l++) {
      float acc[NG][4];
#pragma unroll
      for (int ng = 0; ng < NG; ng++)
#pragma unroll
        for (int e = 0; e < 4; e++) acc[ng][e] = 0.0f;
      const int st = grp + 2 * (l % Sg);
      mbar_wait_bounded(&bars[st], (l / Sg) & 1, a.flags);
      const uint8_t *sb = stages + st * L.stage_bytes;
#pragma unroll 2
      for (int i = gt0; i < gt1; i++)
        tile_mma<NG, ZEROS, NG == 1>(sb + i * kTileNibBytes, sb + nib_b + i * kTileSclBytes,
                                     sb + nib_b + scl_b + i * kTileZroBytes, xs + i * kTileK + 4 * t, L.xstride, M,
                                     lane, acc);
#pragma unroll
      for (int ng = 0; ng < NG; ng++)
#pragma unroll
        for (int e = 0; e < 4; e++) gred[((gw * NG + ng) * 4 + e) * 32 + lane] = acc[ng][e];
      named_bar_sync(1 + grp, 256);
      if (gtid == 0 && j + S < J) issue_to(j + S, st);  // the group's next column for this stage
      const int nt = g + j * G;
      auto gsum_at = [&](int r, int tok) {
        const int ng = tok >> 3, tk = tok & 7;
        const int ln = 4 * (r & 7) + (tk >> 1);
        const int e = ((r >> 3) << 1) | (tk & 1);
        float sum = 0.0f;
#pragma unroll
        for (int w2 = 0; w2 < 8; w2++) sum += gred[((w2 * NG + ng) * 4 + e) * 32 + ln];
        return sum;
      };
      if (C > 1) {  // every output of the column waits for the cluster reduction
        for (int o = gtid; o < kOut; o += 256) {
          const int r = o / (8 * NG), tok = o - r * (8 * NG);
          part[j * kOut + o] = gsum_at(r, tok);
        }
      } else if (a.epi == kEpiNone) {
        for (int o = gtid; o < kOut; o += 256) {
          const int r = o / (8 * NG), tok = o - r * (8 * NG);
          emit(a, parity, nt, r, tok, gsum_at(r, tok));
        }
      } else if (a.epi == kEpiResidual) {
        for (int o = gtid; o < kOut; o += 256) {
          const int r = o / (8 * NG), tok = o - r * (8 * NG);
          const float v = emit_residual(a, nt, r, tok, gsum_at(r, tok));
          sq[grp][o] = v * v;
        }
        named_bar_sync(1 + grp, 256);
        if (gtid < M) emit_stats(a, nt, gtid, sq[grp]);
      } else {
        for (int o = gtid; o < kOut / 2; o += 256) {
          const int r = o / (8 * NG), tok = o - r * (8 * NG);
          emit_pair(a, nt, r, tok, gsum_at(r, tok), gsum_at(r + 8, tok));
        }
      }
      named_bar_sync(1 + grp, 256);  // the group's half of red (and sq) is reused next
    }
    // No copy may still be writing shared memory at exit (only possible
    // after a timed-out wait): the group's last use of each of its stages.
    if (gtid == 0)
      for (int q = max(0, l - Sg); q < l; q++) mbar_wait_bounded(&bars[grp + 2 * (q % Sg)], (q / Sg) & 1, a.flags);
    // With a K split: one cluster reduction of all J columns (planned only
    // when `part` holds them all). Every thread of every CTA of the cluster
    // gets here: the CTAs of a cluster share g, hence J.
    if (C > 1) flush(0, J);
  } else
  for (int j = 0; j < J; j++) {
    float acc[NG][4];
#pragma unroll
    for (int ng = 0; ng < NG; ng++)
#pragma unroll
      for (int e = 0; e < 4; e++) acc[ng][e] = 0.0f;
    const int st = j % S;
    mbar_wait_bounded(&bars[st], (j / S) & 1, a.flags);
    const uint8_t *sb = stages + st * L.stage_bytes;
#pragma unroll 2
    for (int i = wt0; i < wt1; i++)
      tile_mma<NG, ZEROS, NG == 1>(sb + i * kTileNibBytes, sb + nib_b + i * kTileSclBytes,
                         sb + nib_b + scl_b + i * kTileZroBytes, xs + i * kTileK + 4 * t, L.xstride, M, lane, acc);
#pragma unroll
    for (int ng = 0; ng < NG; ng++)
#pragma unroll
      for (int e = 0; e < 4; e++) red[((warp * NG + ng) * 4 + e) * 32 + lane] = acc[ng][e];
    __syncthreads();
    if (threadIdx.x == 0 && j + S < J) issue(j + S);  // every warp is done with the stage
    const int nt = g + j * G;
    auto warp_sum_at = [&](int r, int tok) {
      const int ng = tok >> 3, tk = tok & 7;
      const int ln = 4 * (r & 7) + (tk >> 1);
      const int e = ((r >> 3) << 1) | (tk & 1);
      float sum = 0.0f;
#pragma unroll
      for (int w2 = 0; w2 < kWWarps; w2++) sum += red[((w2 * NG + ng) * 4 + e) * 32 + ln];
      return sum;
    };
    if (C > 1 || a.epi == kEpiNone) {
      for (int o = threadIdx.x; o < kOut; o += kWThreads) {
        const int r = o / (8 * NG), tok = o - r * (8 * NG);
        const float sum = warp_sum_at(r, tok);
        if (C > 1)
          part[(j % Jc) * kOut + o] = sum;
        else
          emit(a, parity, nt, r, tok, sum);
      }
    } else if (a.epi == kEpiResidual) {
      for (int o = threadIdx.x; o < kOut; o += kWThreads) {
        const int r = o / (8 * NG), tok = o - r * (8 * NG);
        const float v = emit_residual(a, nt, r, tok, warp_sum_at(r, tok));
        sq[0][o] = v * v;
      }
      __syncthreads();
      if ((int)threadIdx.x < M) emit_stats(a, nt, threadIdx.x, sq[0]);
    } else {
      for (int o = threadIdx.x; o < kOut / 2; o += kWThreads) {
        const int r = o / (8 * NG), tok = o - r * (8 * NG);
        emit_pair(a, nt, r, tok, warp_sum_at(r, tok), warp_sum_at(r + 8, tok));
      }
    }
    __syncthreads();  // red is reused by the next column
    if (C > 1 && (j % Jc == Jc - 1 || j == J - 1)) flush(j - j % Jc, j + 1);
  }
  if (a.trigger_at == 2) pdl_trigger();
  if (a.trace && threadIdx.x == 0) ts[4] = globaltimer();
  // No copy may still be writing shared memory at exit (only possible after
  // a timed-out wait).
  if (threadIdx.x == 0) {
    if (x_bulk) mbar_wait_bounded(xbar, 0, a.flags);
    if (!a.wide_groups)
      for (int j = max(0, J - S); j < J; j++) mbar_wait_bounded(&bars[j % S], (j / S) & 1, a.flags);
  }
  if (a.push_on) push_signal(a.push);
  if (a.trace && threadIdx.x == 0) {
    ts[5] = globaltimer();
    trace_record(a.trace, a.trace_next, a.trace_cap, ts, a.launch_index, blockIdx.y * gridDim.x + blockIdx.x);
  }
}

// Clusters of C CTAs with `smem` bytes each that fit on the GPU at once
// (clusters must sit within one GPC, so this can be below num_sms / C).
int wide_max_clusters(int C, int smem, int num_sms) {
  static std::mutex lock;
  static std::map<std::pair<int, int>, int> cache;
  std::lock_guard<std::mutex> guard(lock);
  const auto key = std::make_pair(C, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  auto kern = gemv_wide_kernel<1, false, kProNone>;
  int n = 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kWideSmemMaxGroups) == cudaSuccess &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)C, (unsigned)(num_sms / C > 0 ? num_sms / C : 1), 1);
    cfg.blockDim = dim3(kWThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = (unsigned)C;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();  // a failed query leaves no sticky error
  if (n <= 0) n = num_sms / C > 0 ? num_sms / C : 1;
  cache[key] = n;
  return n;
}

template <int NG, bool ZEROS, int PRO>
cudaError_t launch_wide_t(const GemvArgs &a, cudaStream_t stream, bool pdl) {
  const int G = a.groups;
  const WideSmem L = wide_smem(a.M, a.kt_per_cta, a.stages, a.part_cols, a.cluster, ZEROS);
  auto kern = gemv_wide_kernel<NG, ZEROS, PRO>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kWideSmemMaxGroups);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  if (L.total > (a.wide_groups ? kWideSmemMaxGroups : kWideSmemMax)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.cluster, (unsigned)G, 1);
  cfg.blockDim = dim3(kWThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)L.total;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int n = 0;
  if (a.cluster > 1) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = (unsigned)a.cluster;
    attrs[n].val.clusterDim.y = 1;
    attrs[n].val.clusterDim.z = 1;
    n++;
  }
  if (pdl) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    n++;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace

cudaError_t launch_prologue(const Prologue &p, int M, int K, void *x_f16, cudaStream_t stream, bool pdl) {
  if (K % 8 || (p.kind != kProRmsNorm && p.kind != kProSwiglu)) return cudaErrorInvalidValue;
  // the norm: a cluster of CTAs per row (comm.cu)
  if (p.kind == kProRmsNorm) return launch_addnorm(p.a, p.b, p.w, p.eps, p.out, x_f16, M, K, nullptr, nullptr, stream, pdl);
  prologue_kernel<<<M, kThreads, 0, stream>>>(p, K, reinterpret_cast<__half *>(x_f16));
  return cudaGetLastError();
}

bool plan_gemv(GemvArgs &a, int num_sms) {
  if (a.M < 1 || a.M > kGemvMaxTokens) return false;
  const int NG = (a.M + 7) / 8;
  const bool zeros = a.zro != nullptr;
  // Largest K range per CTA within the shared-memory budget and the chunk
  // count.
  int max_ktc = kMaxTilesPerCta;
  while (max_ktc > 1 && gemv_smem(a.M, max_ktc, NG, zeros).total > kSmemBudget) max_ktc--;
  int C = (a.KT + max_ktc - 1) / max_ktc;
  // Few row tiles, where WG_GEMV_SPLIT_PCT allows it: split K further (up
  // to a portable cluster of 8) until the grid covers the SMs `ctas_per_sm`
  // times, keeping at least one tile per warp. WG_GEMV_CTAS_PER_SM overrides
  // the target (tuning).
  static int ctas_per_sm = -1, split_pct = -1;
  if (ctas_per_sm < 0) {
    const char *e = getenv("WG_GEMV_CTAS_PER_SM");
    ctas_per_sm = e ? atoi(e) : 1;
    if (ctas_per_sm < 1) ctas_per_sm = 1;
    // Split K for a small grid only below this % of the target (tuning;
    // default 0: never). Measured on B200 (M = 1, chains of 16 as a CUDA
    // graph): 2048 x 2048 in clusters of 2 over 256 CTAs 3.89 us a launch,
    // unsplit over 128 CTAs 2.45 us: the cluster reduction's ~1.5 us outweighs
    // the halved multiplies, and the weights are in shared memory before the
    // dependency release either way.
    const char *f = getenv("WG_GEMV_SPLIT_PCT");
    split_pct = f ? atoi(f) : 0;
  }
  if ((long)a.NT * 100 < (long)split_pct * ctas_per_sm * num_sms)
    while (C < 8 && a.NT * C < ctas_per_sm * num_sms && (a.KT + C) / (C + 1) >= kWarps) C++;
  if (C > 16) return false;
  const int ktc = (a.KT + C - 1) / C;
  C = (a.KT + ktc - 1) / ktc;
  a.kt_per_cta = ktc;
  a.cluster = C;
  return true;
}

// Clusters of several CTAs: four fewer than the occupancy query allows, then
// the fewest that give each cluster the same number of columns. The query's
// count of co-resident clusters is more than the hardware places behind a
// previous kernel's tail (wg_trace of the config-4 decode step, clusters of
// 3 after the gate|up GEMV on all 148 SMs: of 45 planned, 43 placed and the
// last two ran as a second wave, the down projection 29 us a layer; of 43,
// one or two late in most layers, 26 us; of 37 (this reserve) none late,
// 19.8 us; the step 2.91 -> 2.67 ms). Single CTAs keep one an SM (each SM's
// share of HBM bounds a CTA with more columns).
static int wide_balance(int NT, int G, int C) {
  if (C == 1) return G;
  if (G > 8) G -= 4;
  const int J = (NT + G - 1) / G;
  return (NT + J - 1) / J;
}

bool plan_gemv_wide(GemvArgs &a, int num_sms) {
  if (a.M < 1 || a.M > kWideMaxTokens || (a.pro.kind != kProNone && a.M > kProMaxTokens)) return false;
  const bool zeros = a.zro != nullptr;
  int C = 1;
  while (a.M * ((a.KT + C - 1) / C) * kTileK * 2 > kWideXBudget) C++;
  if (C > 8) return false;
  const int ktc = (a.KT + C - 1) / C;
  C = (a.KT + ktc - 1) / ktc;
  // stages: as many as fit (with the largest column count a CTA can get)
  int G = num_sms / C;
  if (G < 1) G = 1;
  if (G > a.NT) G = a.NT;
  // stages, then the columns whose K-split sums wait for a cluster reduction
  // (a few at least; the rest go in later chunks)
  int S = 4;
  while (S > 1 && wide_smem(a.M, ktc, S, 4, C, zeros).total > kWideSmemMax) S--;
  if (wide_smem(a.M, ktc, S, 1, C, zeros).total > kWideSmemMax) return false;
  // Without a K split, two warp groups walk alternate columns through
  // their own stage rings (an even S). WG_GEMV_WIDE_GROUPS (comparison): 0
  // off, 1 within the 200 KB budget, 2 (default) within 224 KB — measured
  // on B200: M = 8 at 28672x4096 25.2 us (off), 23.6 (1: two stages), 20.6
  // (2: four stages).
  static int groups_on = -1;
  if (groups_on < 0) {
    const char *e = getenv("WG_GEMV_WIDE_GROUPS");
    groups_on = e ? atoi(e) : 2;
  }
  static int norm_rows = -1;
  if (norm_rows < 0) {
    const char *e = getenv("WG_WIDE_NORM_ROWS");
    norm_rows = e && e[0] == '1' ? 1 : 0;
  }
  a.wide_norm_rows = norm_rows;
  a.wide_groups = 0;
  if (groups_on && C == 1) {
    const int budget = groups_on == 2 ? kWideSmemMaxGroups : kWideSmemMax;
    int S2 = 4;
    while (S2 > 2 && wide_smem(a.M, ktc, S2, 1, C, zeros).total > budget) S2 -= 2;
    if (wide_smem(a.M, ktc, S2, 1, C, zeros).total <= budget) {
      S = S2;
      a.wide_groups = 1;
    }
  }
  int Jc = (a.NT + G - 1) / G * 2;
  while (Jc > 1 && wide_smem(a.M, ktc, S, Jc, C, zeros).total > kWideSmemMax) Jc--;
  // one wave: no more clusters than fit at once
  const int fit = wide_max_clusters(C, wide_smem(a.M, ktc, S, Jc, C, zeros).total, num_sms);
  if (G > fit) G = fit;
  int J = (a.NT + G - 1) / G;
  G = wide_balance(a.NT, G, C);
  J = (a.NT + G - 1) / G;
  if (Jc > J) Jc = J;
  // With a K split the group walk keeps every column's partial sums in
  // `part` and reduces them across the cluster once, after the walk: only
  // when all J columns fit (the cluster count, hence J, depends on the
  // shared memory it is planned with). Not yet for the tensor-parallel push
  // exchange (its K-split launches keep the per-chunk walk, the one measured
  // on several GPUs).
  if (groups_on && C > 1 && !a.push_on) {
    const int budget = groups_on == 2 ? kWideSmemMaxGroups : kWideSmemMax;
    const int Gmax = min(num_sms / C > 0 ? num_sms / C : 1, a.NT);
    const int Jest = (a.NT + Gmax - 1) / Gmax;
    int S2 = 4;
    while (S2 > 2 && wide_smem(a.M, ktc, S2, Jest, C, zeros).total > budget) S2 -= 2;
    const int smem2 = wide_smem(a.M, ktc, S2, Jest, C, zeros).total;
    if (smem2 <= budget) {
      const int G2 = wide_balance(a.NT, min(Gmax, wide_max_clusters(C, smem2, num_sms)), C);
      const int J2 = (a.NT + G2 - 1) / G2;
      if (J2 <= Jest) {
        S = S2;
        G = G2;
        J = J2;
        Jc = J2;
        a.wide_groups = 1;
      }
    }
  }
  a.kt_per_cta = ktc;
  a.cluster = C;
  a.groups = G;
  a.stages = S;
  a.part_cols = Jc;
  return true;
}

cudaError_t launch_gemv_wide(const GemvArgs &a, cudaStream_t stream, bool pdl) {
  const bool z = a.zro != nullptr;
  const int NG = (a.M + 7) / 8;
  if (a.pro.kind != kProNone && NG != 1) return cudaErrorInvalidValue;
  switch (a.pro.kind) {
    case kProNone:
      switch (NG) {
        case 1: return z ? launch_wide_t<1, true, kProNone>(a, stream, pdl) : launch_wide_t<1, false, kProNone>(a, stream, pdl);
        case 2: return z ? launch_wide_t<2, true, kProNone>(a, stream, pdl) : launch_wide_t<2, false, kProNone>(a, stream, pdl);
        case 3: return z ? launch_wide_t<3, true, kProNone>(a, stream, pdl) : launch_wide_t<3, false, kProNone>(a, stream, pdl);
        case 4: return z ? launch_wide_t<4, true, kProNone>(a, stream, pdl) : launch_wide_t<4, false, kProNone>(a, stream, pdl);
        default: return cudaErrorInvalidValue;
      }
    case kProRmsNorm:
      return z ? launch_wide_t<1, true, kProRmsNorm>(a, stream, pdl) : launch_wide_t<1, false, kProRmsNorm>(a, stream, pdl);
    case kProSwiglu:
      return z ? launch_wide_t<1, true, kProSwiglu>(a, stream, pdl) : launch_wide_t<1, false, kProSwiglu>(a, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemv(const GemvArgs &a, cudaStream_t stream, bool pdl) {
  const int NG = (a.M + 7) / 8;
  const bool z = a.zro != nullptr;
  if (a.pro.kind != kProNone) {
    if (a.M > kProMaxTokens) return cudaErrorInvalidValue;
    if (a.pro.kind == kProRmsNorm)
      return z ? launch_t<1, true, kProRmsNorm>(a, stream, pdl) : launch_t<1, false, kProRmsNorm>(a, stream, pdl);
    if (a.pro.kind == kProSwiglu)
      return z ? launch_t<1, true, kProSwiglu>(a, stream, pdl) : launch_t<1, false, kProSwiglu>(a, stream, pdl);
    return cudaErrorInvalidValue;
  }
  switch (NG) {
    case 1: return z ? launch_t<1, true>(a, stream, pdl) : launch_t<1, false>(a, stream, pdl);
    case 2: return z ? launch_t<2, true>(a, stream, pdl) : launch_t<2, false>(a, stream, pdl);
    case 3: return z ? launch_t<3, true>(a, stream, pdl) : launch_t<3, false>(a, stream, pdl);
    case 4: return z ? launch_t<4, true>(a, stream, pdl) : launch_t<4, false>(a, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace wg
