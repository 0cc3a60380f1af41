// The kernels around the Q4 matmuls in a decoder layer: embedding, fused residual add + RMS norm, qk-norm + RoPE + KV-cache append,
// causal GQA attention over fp16 caches, SwiGLU, LFM2's gated short
// convolution with an fp16 rolling state, the fp16 output head and argmax.
//
// Activation layout: row-major [rows][features]; the residual stream is fp32
// (the reference keeps it in f32 textures), matmul inputs fp16. Positions
// come from a device counter so that a decode step can be replayed from a
// CUDA graph without re-recording.
#include <cooperative_groups.h>

#include <cstdlib>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "decoder_kernels.cuh"
#include "tma.cuh"
#include "device_utils.cuh"

namespace wg {

namespace cg = cooperative_groups;

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum over a block of blockDim.x (multiple of 32, <= 1024) threads.
__device__ float block_sum(float v, float *red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.0f;
  for (int i = 0; i < nw; i++) s += red[i];
  return s;
}

// ---- embedding (src/gpu/kernels.ts:1092, embed pass engine.ts:8961) ------

__global__ void embed_kernel(const int32_t *ids, int rows, const __half *table, int V, int D, float *out) {
  pdl_trigger();  // dependents may launch now; they wait for this grid to finish
  pdl_wait();     // inputs come from the previous kernel
  const int r = blockIdx.x;
  int id = ids[r];
  if (id < 0 || id >= V) id = 0;
  const __half *src = table + (size_t)id * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) out[(size_t)r * D + d] = __half2float(src[d]);
}

// ---- residual add + RMS norm (addNormed engine.ts:5695; RMS kernels
//      kernels.ts:1158-1372; fusedAdd native.ts:33) ---------------------------

__global__ void rmsnorm_kernel(float *x, const float *add, const float *w, float eps, int D, void *out,
                               int out_dtype) {
  pdl_trigger();  // dependents may launch now; they wait for this grid to finish
  pdl_wait();     // inputs come from the previous kernel
  __shared__ float red[32];
  const int r = blockIdx.x;
  float *xr = x + (size_t)r * D;
  float ss = 0.0f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float v = xr[d];
    if (add) {
      v += add[(size_t)r * D + d];
      xr[d] = v;
    }
    ss += v * v;
  }
  const float inv = rsqrtf(block_sum(ss, red) / (float)D + eps);
  for (int d = threadIdx.x; d < D; d += blockDim.x)
    store_out(out, out_dtype, (size_t)r * D + d, xr[d] * inv * w[d]);
}

// ---- qk-norm + RoPE + KV append (headPrep kernels.ts:2196-2322) -----------
// qkv: [rows][(H + 2 Hkv) Dh] = q | k | v. One CTA per (row, head among
// H + Hkv), Dh/2 threads: thread j rotates the pair (j, j + Dh/2) by
// pos * theta^(-2j/Dh) (rotate-half). Queries leave scaled by 1/sqrt(Dh).

__global__ void rope_kv_kernel(const float *qkv, int rps, int H, int Hkv, int Dh, const int *pos0, float theta,
                               const float *q_norm, const float *k_norm, float eps, __half *q_out,
                               __half *k_cache, __half *v_cache, int cache_len, unsigned *flags) {
  pdl_trigger();  // dependents may launch now; they wait for this grid to finish
  pdl_wait();     // inputs come from the previous kernel
  __shared__ float red[32];
  const int r = blockIdx.x, h = blockIdx.y;  // h < H: query head; else kv head h - H
  const int half = Dh / 2, j = threadIdx.x;
  const int seq = r / rps;  // sequence of this row (rps rows per sequence)
  const int pos = pos0[seq] + (r - seq * rps);
  const size_t row = (size_t)r * (H + 2 * Hkv) * Dh;
  k_cache += (size_t)seq * Hkv * cache_len * Dh;
  v_cache += (size_t)seq * Hkv * cache_len * Dh;
  const bool is_q = h < H;
  const int hk = h - H;
  const float *src = qkv + row + (size_t)(is_q ? h : H + hk) * Dh;
  float a = src[j], b = src[j + half];
  const float *nw = is_q ? q_norm : k_norm;
  if (nw) {
    const float inv = rsqrtf(block_sum(a * a + b * b, red) / (float)Dh + eps);
    a *= inv * nw[j];
    b *= inv * nw[j + half];
  }
  const float freq = powf(theta, -2.0f * (float)j / (float)Dh);
  float sn, cs;
  sincosf((float)pos * freq, &sn, &cs);
  const float ra = a * cs - b * sn, rb = b * cs + a * sn;
  if (is_q) {
    const float scale = rsqrtf((float)Dh);
    __half *q = q_out + ((size_t)r * H + h) * Dh;
    q[j] = __float2half_rn(ra * scale);
    q[j + half] = __float2half_rn(rb * scale);
  } else {
    if (pos < 0 || pos >= cache_len) {
      if (j == 0) raise_flag(flags, kFlagBadArgument);
      return;
    }
    __half *k = k_cache + ((size_t)hk * cache_len + pos) * Dh;
    k[j] = __float2half_rn(ra);
    k[j + half] = __float2half_rn(rb);
    const float *vs = qkv + row + (size_t)(H + Hkv + hk) * Dh;
    __half *v = v_cache + ((size_t)hk * cache_len + pos) * Dh;
    v[j] = __float2half_rn(vs[j]);
    v[j + half] = __float2half_rn(vs[j + half]);
  }
}

// ---- causal GQA attention (scores / attend kernels.ts:2386-2579) -----------
// A (query row, KV head) pair is served by HS x CL CTAs: its G query heads
// split over HS CTAs (each owns whole softmax rows), and, for caches longer
// than kAttnSliceKeys positions, its keys 0..pos split over a thread-block
// cluster of CL CTAs ("flash decoding"; CTA c takes the c-th slice). CL,
// then HS, are as large as keeps the grid within about one wave.
// Per slice, tiles of 128 keys (64 for Dh = 256) of K and V are staged in
// shared memory with cp.async (all copies in flight at once; the first
// tile's while the queries are made; K and V rows padded by 16 bytes so
// that row-strided fragment reads hit distinct banks). Both products run on
// the tensor cores (mma.m16n8k16, fp32 sums), the G query heads as the rows
// of A (rows >= G zero): scores S = Q K^T, warp w taking key blocks w, w +
// 4, ... of 8 keys (q and K are fp16 values: the products are exact); an
// online softmax keeps (max, sum) per head in fp32; then O += P V, warp w
// owning head dims [w Dh / 4, (w + 1) Dh / 4) in registers across tiles,
// with P split as fp16 hi + lo (two MMAs: fp32-level precision) and V read
// by ldmatrix.trans from the key-major tile. The key slices are merged
// at the cluster's leader: every CTA pushes (max, sum, acc) into the
// leader's shared memory (distributed shared memory stores), one cluster
// barrier, and the leader writes the outputs. No global scratch: one launch
// per step and nothing to allocate.

constexpr int kAttnCluster = 8;  // largest cluster
constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnMaxGroup = 16;
constexpr int kAttnSliceKeys = 128;  // cache positions per CTA before the keys are split over a cluster

// Keys per tile: 128 (one tile covers a decode step's slice up to 1024
// positions) while shared memory allows, 64 for Dh = 256.
__host__ __device__ constexpr int attn_tile(int Dh) { return Dh <= 128 ? 128 : 64; }

// Shared memory of one attention CTA. q, corr, m, l and acc live for the
// whole kernel; k, v, p and red are per-tile scratch. gather receives the
// cluster's (m, l, acc) slices at the leader: its own slots when they fit
// (the CTAs push without a first barrier), else overlaid on the scratch
// (alias: one more cluster barrier, so that no push lands on a tile still in
// use).
constexpr size_t kAttnGatherBudget = 200 * 1024;
struct AttnSmem {
  size_t q, corr, m, l, acc, k, v, p, red, gather, total;  // byte offsets
  bool alias;
  __host__ __device__ AttnSmem(int Dh, int G) {
    const int kAttnTile = attn_tile(Dh);
    const size_t gpad = ((size_t)G * 4 + 15) / 16 * 16;  // every region 16-byte aligned
    size_t o = 0;
    q = o;
    o += (size_t)G * Dh * 4;
    corr = o;
    o += gpad;
    m = o;
    o += gpad;
    l = o;
    o += gpad;
    acc = o;
    o += (size_t)G * Dh * 4;
    k = o;
    o += (size_t)kAttnTile * (Dh + 8) * 2;
    v = o;
    o += (size_t)kAttnTile * (Dh + 8) * 2;
    p = o;
    o += (size_t)G * (kAttnTile + 8) * 4;
    red = o;
    const size_t gbytes = (size_t)kAttnCluster * (2 * G + G * Dh) * 4;
    alias = o + gbytes > kAttnGatherBudget;
    gather = alias ? k : o;
    total = alias ? (k + gbytes > o ? k + gbytes : o) : o + gbytes;
  }
};

// DPL consecutive halves from shared memory as floats.
template <int DPL>
__device__ __forceinline__ void load_halves(const __half *p, float v[DPL]) {
  if constexpr (DPL == 1) {
    v[0] = __half2float(*p);
  } else if constexpr (DPL == 2) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(p));
    v[0] = f.x;
    v[1] = f.y;
  } else if constexpr (DPL == 4) {
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
    v[0] = a.x, v[1] = a.y, v[2] = b.x, v[3] = b.y;
  } else {
    const uint4 u = *reinterpret_cast<const uint4 *>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

// With ROPE (decode: one row per sequence), the kernel also does
// rope_kv_kernel's work: every CTA turns its heads' q rows of qkv into
// rotated, scaled fp16 queries itself, and the CTA whose key slice holds the
// new position computes that key and value, appends them to the caches and
// patches them into its shared-memory tile — one launch instead of two.
struct RopeArgs {
  const float *qkv;  // [rows][(H + 2 Hkv) Dh]
  float theta;
  const float *q_norm, *k_norm;  // or null
  float eps;
  unsigned *flags;
  // wg_trace (any attention launch): a record per CTA of entry, cache
  // prefetch issued, dependency release, queries made, the last tile's P.V
  // done, exit (the cluster leader after the merge)
  TraceSink tr;
};

// q / k rows of qkv for one head, as rope_kv_kernel computes them: optional
// RMS norm over Dh, rotate-half RoPE at position pos, scale; lane l holds
// dims l + 32 i (i < DPL), so the rotate-half pairs (i, i + DPL/2) sit in
// one lane. Values are rounded to fp16 as the separate kernel stores them.
// The rotation of the lane's pairs at one position: cs / sn of
// pos * theta^(-2j / Dh), j = lane + 32 i (computed once per thread: every
// head of the row shares it).
template <int DPL>
__device__ __forceinline__ void rope_angles(float theta, int pos, int lane, float *cs, float *sn) {
  constexpr int Dh = 32 * DPL;
#pragma unroll
  for (int i = 0; i < DPL / 2; i++) {
    const int j = lane + 32 * i;
    const float freq = powf(theta, -2.0f * (float)j / (float)Dh);
    sincosf((float)pos * freq, &sn[i], &cs[i]);
  }
}

template <int DPL>
__device__ __forceinline__ void rope_head(const float *src, const float *nw, float eps, const float *cs,
                                          const float *sn, float scale, int lane, float out[DPL]) {
  constexpr int Dh = 32 * DPL;
  float v[DPL];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < DPL; i++) {
    v[i] = src[lane + 32 * i];
    ss += v[i] * v[i];
  }
  if (nw) {
    const float inv = rsqrtf(warp_sum(ss) / (float)Dh + eps);
#pragma unroll
    for (int i = 0; i < DPL; i++) v[i] *= inv * nw[lane + 32 * i];
  }
#pragma unroll
  for (int i = 0; i < DPL / 2; i++) {  // pairs (j, j + Dh/2), j = lane + 32 i
    const float a = v[i], b = v[i + DPL / 2];
    out[i] = __half2float(__float2half_rn((a * cs[i] - b * sn[i]) * scale));
    out[i + DPL / 2] = __half2float(__float2half_rn((b * cs[i] + a * sn[i]) * scale));
  }
}

__device__ __forceinline__ void attn_mma(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t half2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

// Four 8x8 fp16 matrices from shared memory, transposed (B fragments of a
// key-major tile); lane l gives the address of row l & 7 of matrix l >> 3.
__device__ __forceinline__ void ldsm_x4_trans(uint32_t r[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2_trans(uint32_t r[2], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(smem_u32(p)));
}

// A fragment rows g and g + 8 (g < 16), columns c, c + 1 and c + 8, c + 9
// of a row-major fp32 matrix with `rows` valid rows, as fp16 pairs (hi) and
// the remainders (lo): value = hi + lo to ~2^-22 relative.
__device__ __forceinline__ void a_frag_split(const float *m, int stride, int rows, int g, int c, uint32_t hi[4],
                                             uint32_t lo[4]) {
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int row = g + 8 * (i & 1), col = c + 8 * (i >> 1);
    float2 v = make_float2(0.0f, 0.0f);
    if (row < rows) v = *reinterpret_cast<const float2 *>(m + (size_t)row * stride + col);
    const __half2 h = __float22half2_rn(v);
    const float2 hf = __half22float2(h);
    hi[i] = half2_bits(h);
    lo[i] = half2_bits(__float22half2_rn(make_float2(v.x - hf.x, v.y - hf.y)));
  }
}

template <int DPL, bool ROPE>  // head dims per lane: Dh = 32 * DPL
__global__ void __launch_bounds__(kAttnThreads)
    attention_kernel(const __half *q, int rps, int H, int Hkv, __half *k_cache, __half *v_cache, int cache_len,
                     const int *pos0, __half *out, const RopeArgs ra) {
  pdl_trigger();  // dependents may launch now; they wait for this grid to finish
  __shared__ unsigned long long tstamp[6];
  const bool tracing = ra.tr.buf != nullptr;
  if (tracing && threadIdx.x == 0) tstamp[0] = globaltimer();
  // While the previous kernel finishes: an L2 prefetch of this CTA's slice
  // of the caches (rows written by earlier steps; a prefetch is only a hint
  // and L2 is where writes land, so a position read early or a row still
  // being written cannot make anything stale).
  if (threadIdx.x == 0) {
    const int r = blockIdx.z, bq = r / rps, CLx = (int)gridDim.x;
    const int Lg = max(0, min(pos0[bq] + (r - bq * rps) + 1, cache_len));
    const int pg = (Lg + CLx - 1) / CLx;
    const int a0 = min(Lg, (int)blockIdx.x * pg), a1 = min(Lg, a0 + pg);
    if (a1 > a0) {
      const int Dh = 32 * DPL, hkx = blockIdx.y / (gridDim.y / Hkv);
      const size_t row0 = ((size_t)bq * Hkv + hkx) * cache_len + a0;
      prefetch_l2(k_cache + row0 * Dh, (uint32_t)(a1 - a0) * Dh * 2);
      prefetch_l2(v_cache + row0 * Dh, (uint32_t)(a1 - a0) * Dh * 2);
    }
  }
  if (tracing && threadIdx.x == 0) tstamp[1] = globaltimer();
  pdl_wait();     // inputs come from the previous kernel
  if (tracing && threadIdx.x == 0) tstamp[2] = globaltimer();
  constexpr int Dh = 32 * DPL;
  constexpr int kHalfDpl = DPL / 2 > 0 ? DPL / 2 : 1;  // rotate-half pairs per lane (ROPE: DPL >= 2)
  constexpr int kAttnTile = attn_tile(Dh);
  constexpr int kPerLane = kAttnTile / 32;  // scores per lane in the softmax
  constexpr int vecs = Dh / 8;  // 16-byte vectors per key row
  constexpr int kstride = Dh + 8;        // K and V rows (halves)
  constexpr int pstride = kAttnTile + 8;  // P rows (floats)
  constexpr int kDw = Dh / kAttnWarps;    // head dims of a warp's P.V (DPL blocks of 8)
  extern __shared__ __align__(16) unsigned char smem[];
  cg::cluster_group cluster = cg::this_cluster();
  // grid: x the cluster's key slices, y KV head x HS head groups, z rows
  const int HS = gridDim.y / Hkv;
  const int G = H / Hkv / HS;        // query heads of this CTA
  const int qh0 = blockIdx.y * G;    // its first query head
  const AttnSmem lay(Dh, G);
  float *sq = reinterpret_cast<float *>(smem + lay.q);
  __half *sk = reinterpret_cast<__half *>(smem + lay.k);
  __half *sv = reinterpret_cast<__half *>(smem + lay.v);
  float *sp = reinterpret_cast<float *>(smem + lay.p);
  float *scorr = reinterpret_cast<float *>(smem + lay.corr);
  float *sm = reinterpret_cast<float *>(smem + lay.m);
  float *sl = reinterpret_cast<float *>(smem + lay.l);
  float *sacc = reinterpret_cast<float *>(smem + lay.acc);
  float *sgather = reinterpret_cast<float *>(smem + lay.gather);

  const int c = (int)cluster.block_rank();
  const int CL = (int)cluster.num_blocks();
  const int hk = blockIdx.y / HS, r = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bseq = r / rps;  // sequence of this query row (rps rows per sequence)
  const int L = max(0, min(pos0[bseq] + (r - bseq * rps) + 1, cache_len));
  const int per = (L + CL - 1) / CL;
  const int t0 = min(L, c * per), t1 = min(L, t0 + per);

  const __half *kb = k_cache + ((size_t)bseq * Hkv + hk) * cache_len * Dh;
  const __half *vb = v_cache + ((size_t)bseq * Hkv + hk) * cache_len * Dh;
  auto issue_tile = [&](int tt, int nt) {  // every copy of the tile in flight at once
    for (int i = tid; i < nt * vecs; i += kAttnThreads) {
      const int t = i / vecs, e = i - t * vecs;
      cp_async16(sk + t * kstride + e * 8, kb + (size_t)(tt + t) * Dh + e * 8);
      cp_async16(sv + t * kstride + e * 8, vb + (size_t)(tt + t) * Dh + e * 8);
    }
  };
  // the first tile's keys and values load while the queries are made
  if (t0 < t1) issue_tile(t0, min(kAttnTile, t1 - t0));

  // queries of the group (already scaled by 1/sqrt(Dh))
  const int pnew = pos0[bseq] + (r - bseq * rps);  // this row's position (ROPE: its new key)
  const bool owner = ROPE && t0 <= pnew && pnew < t1;  // this CTA's slice holds the new key
  float knew[DPL], vnew[DPL];
  if constexpr (ROPE) {
    const float *row = ra.qkv + (size_t)r * (H + 2 * Hkv) * Dh;
    float cs[kHalfDpl], sn[kHalfDpl];
    rope_angles<DPL>(ra.theta, pnew, lane, cs, sn);
    for (int g = warp; g < G; g += kAttnWarps) {
      float qv[DPL];
      rope_head<DPL>(row + (size_t)(qh0 + g) * Dh, ra.q_norm, ra.eps, cs, sn, rsqrtf((float)Dh), lane, qv);
#pragma unroll
      for (int i = 0; i < DPL; i++) sq[g * Dh + lane + 32 * i] = qv[i];
    }
    if (pnew < 0 || pnew >= cache_len) {
      if (c == 0 && tid == 0) raise_flag(ra.flags, kFlagBadArgument);
    } else if (owner && warp == 0) {
      rope_head<DPL>(row + (size_t)(H + hk) * Dh, ra.k_norm, ra.eps, cs, sn, 1.0f, lane, knew);
      const float *vs = row + (size_t)(H + Hkv + hk) * Dh;
      __half *kc = k_cache + (((size_t)bseq * Hkv + hk) * cache_len + pnew) * Dh;
      __half *vc = v_cache + (((size_t)bseq * Hkv + hk) * cache_len + pnew) * Dh;
      const bool writer = blockIdx.y % HS == 0;  // one head group appends to the caches
#pragma unroll
      for (int i = 0; i < DPL; i++) {
        vnew[i] = __half2float(__float2half_rn(vs[lane + 32 * i]));
        if (writer) {
          kc[lane + 32 * i] = __float2half_rn(knew[i]);
          vc[lane + 32 * i] = __float2half_rn(vnew[i]);
        }
      }
    }
  } else {
    const __half *qg = q + ((size_t)r * H + qh0) * Dh;
    for (int i = tid; i < G * Dh; i += kAttnThreads) sq[i] = __half2float(qg[i]);
  }
  for (int g = tid; g < G; g += kAttnThreads) {
    sm[g] = -INFINITY;
    sl[g] = 0.0f;
  }
  for (int i = tid; i < G * Dh; i += kAttnThreads) sacc[i] = 0.0f;
  if (tracing && tid == 0) tstamp[3] = globaltimer();

  const int gq = lane >> 2, tq = lane & 3;  // MMA fragment row group / column pair
  uint32_t qa[Dh / 16][4];  // A fragments of the queries (heads x dims), made at the first tile
  float o[DPL][4];          // this warp's dims of O: heads gq, gq + 8 x 8 dims per block
#pragma unroll
  for (int b = 0; b < DPL; b++)
#pragma unroll
    for (int e = 0; e < 4; e++) o[b][e] = 0.0f;
  for (int tt = t0; tt < t1; tt += kAttnTile) {
    const int nt = min(kAttnTile, t1 - tt);
    const int kch = (nt + 15) >> 4;  // 16-key chunks of P.V
    if (tt != t0) {
      __syncthreads();  // previous tile fully consumed
      issue_tile(tt, nt);
    }
    // V rows past the tile's keys up to the chunk's end: zero (their P is
    // 0, and 0 times a stale NaN would not be)
    for (int i = tid; i < (kch * 16 - nt) * (Dh / 2); i += kAttnThreads) {
      const int t = nt + i / (Dh / 2), e = i - (t - nt) * (Dh / 2);
      reinterpret_cast<uint32_t *>(sv + t * kstride)[e] = 0u;
    }
    cp_async_wait_all();
    __syncthreads();
    if (owner && tt <= pnew && pnew < tt + nt) {  // the new key's row: not in the cache when the tile was read
      if (warp == 0) {
#pragma unroll
        for (int i = 0; i < DPL; i++) {
          sk[(pnew - tt) * kstride + lane + 32 * i] = __float2half_rn(knew[i]);
          sv[(pnew - tt) * kstride + lane + 32 * i] = __float2half_rn(vnew[i]);
        }
      }
      __syncthreads();
    }
    if (tt == t0) {
#pragma unroll
      for (int kc = 0; kc < Dh / 16; kc++) {
#pragma unroll
        for (int i = 0; i < 4; i++) {  // q values are fp16 already: exact
          const int row = gq + 8 * (i & 1), col = kc * 16 + 2 * tq + 8 * (i >> 1);
          const float2 v = row < G ? *reinterpret_cast<const float2 *>(sq + row * Dh + col) : make_float2(0.f, 0.f);
          qa[kc][i] = half2_bits(__float22half2_rn(v));
        }
      }
    }
    // scores: S[head][key] at sp[head * pstride + key]; keys >= nt -> -inf
    {
      const int nblk = (nt + 7) >> 3;
      for (int nb = warp; nb < nblk; nb += kAttnWarps) {
        float c4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const __half *kr = sk + (nb * 8 + gq) * kstride + 2 * tq;
#pragma unroll
        for (int kc = 0; kc < Dh / 16; kc++)
          attn_mma(c4, qa[kc], *reinterpret_cast<const uint32_t *>(kr + kc * 16),
                   *reinterpret_cast<const uint32_t *>(kr + kc * 16 + 8));
        const int key = nb * 8 + 2 * tq;
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int g = gq + 8 * (i >> 1), t = key + (i & 1);
          if (g < G) sp[g * pstride + t] = t < nt ? c4[i] : -INFINITY;
        }
      }
      const int rest = kAttnTile - 8 * nblk;
      for (int i = tid; i < G * rest; i += kAttnThreads) {
        const int g = i / rest;
        sp[g * pstride + 8 * nblk + (i - g * rest)] = -INFINITY;
      }
    }
    __syncthreads();
    // per head: new max, rescale factor, probabilities (one warp per head)
    for (int g = warp; g < G; g += kAttnWarps) {
      float *pg = sp + g * pstride;
      float sv_[kPerLane];
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < kPerLane; j++) {
        sv_[j] = pg[lane + 32 * j];
        mx = fmaxf(mx, sv_[j]);
      }
      for (int o2 = 16; o2 > 0; o2 >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o2));
      const float mold = sm[g], mnew = fmaxf(mold, mx);
      float psum = 0.0f;
#pragma unroll
      for (int j = 0; j < kPerLane; j++) {
        const float pj = expf(sv_[j] - mnew);
        pg[lane + 32 * j] = pj;
        psum += pj;
      }
      const float ps = warp_sum(psum);
      if (lane == 0) {
        const float corr = mold == -INFINITY ? 0.0f : expf(mold - mnew);
        sl[g] = sl[g] * corr + ps;
        sm[g] = mnew;
        scorr[g] = corr;
      }
    }
    __syncthreads();
    // O = O * corr + P V over this warp's dims
    {
      const float c_lo = gq < G ? scorr[gq] : 0.0f, c_hi = gq + 8 < G ? scorr[gq + 8] : 0.0f;
#pragma unroll
      for (int b = 0; b < DPL; b++) {
        o[b][0] *= c_lo;
        o[b][1] *= c_lo;
        o[b][2] *= c_hi;
        o[b][3] *= c_hi;
      }
      const int d0 = warp * kDw;
      for (int kc = 0; kc < kch; kc++) {
        uint32_t phi[4], plo[4];
        a_frag_split(sp, pstride, G, gq, kc * 16 + 2 * tq, phi, plo);
        const __half *vr = sv + (kc * 16 + (lane & 15)) * kstride + d0 + (lane >> 4) * 8;
        if constexpr (DPL == 1) {
          uint32_t b[2];
          ldsm_x2_trans(b, sv + (kc * 16 + (lane & 15)) * kstride + d0);
          attn_mma(o[0], phi, b[0], b[1]);
          attn_mma(o[0], plo, b[0], b[1]);
        } else {
#pragma unroll
          for (int b2 = 0; b2 < DPL; b2 += 2) {
            uint32_t b[4];
            ldsm_x4_trans(b, vr + b2 * 8);
            attn_mma(o[b2], phi, b[0], b[1]);
            attn_mma(o[b2], plo, b[0], b[1]);
            attn_mma(o[b2 + 1], phi, b[2], b[3]);
            attn_mma(o[b2 + 1], plo, b[2], b[3]);
          }
        }
      }
    }
  }
  if (tracing && tid == 0) tstamp[4] = globaltimer();
  // this warp's dims of O into sacc for the merge
#pragma unroll
  for (int b = 0; b < DPL; b++)
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int g = gq + 8 * (i >> 1), d = warp * kDw + b * 8 + 2 * tq + (i & 1);
      if (g < G) sacc[g * Dh + d] = o[b][i];
    }
  __syncthreads();
  // merge the slices at the leader (rank 0): every CTA with keys pushes its
  // (m, l, acc) into the leader's gather slots (stores to distributed shared
  // memory: no round trip), one cluster barrier, and the leader combines them
  // from its own shared memory while the others exit.
  if (lay.alias) cluster.sync();  // the gather overlays tiles a peer may still read
  if (t0 < t1) {
    float *gl = cluster.map_shared_rank(sgather, 0);
    for (int g = tid; g < G; g += kAttnThreads) {
      gl[c * G + g] = sm[g];
      gl[(kAttnCluster + c) * G + g] = sl[g];
    }
    float *ga = gl + 2 * kAttnCluster * G + (size_t)c * G * Dh;
    for (int i = tid; i < G * Dh / 4; i += kAttnThreads)
      reinterpret_cast<float4 *>(ga)[i] = reinterpret_cast<const float4 *>(sacc)[i];
  }
  cluster.sync();
  const unsigned cta_id = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
  if (c != 0) {  // nothing reads this CTA's shared memory any more
    if (tracing && tid == 0) {
      tstamp[5] = globaltimer();
      trace_record(ra.tr.buf, ra.tr.next, ra.tr.cap, tstamp, ra.tr.launch_index, cta_id);
    }
    return;
  }
  // weights of each slice per head: w[j][g] = exp(m_j - M) / sum_j' l_j' exp(m_j' - M)
  // (slices without keys carry none; the weights go to the probability tile,
  // or to q's slots when the gather overlays the tiles; corr holds the
  // per-head sums)
  const int nslices = min(CL, (L + per - 1) / max(per, 1));  // slices holding keys
  float *wts = sp;  // G * kAttnCluster floats of the probability tile (free now)
  if (lay.alias) wts = reinterpret_cast<float *>(smem + lay.q);  // q is free too
  for (int g = tid; g < G; g += kAttnThreads) {
    float M = -INFINITY;
    for (int j = 0; j < nslices; j++) M = fmaxf(M, sgather[j * G + g]);
    float lsum = 0.0f;
    for (int j = 0; j < nslices; j++) {
      const float w = M == -INFINITY ? 0.0f : expf(sgather[j * G + g] - M);
      wts[j * G + g] = w;
      lsum += sgather[(kAttnCluster + j) * G + g] * w;
    }
    scorr[g] = lsum > 0.0f ? 1.0f / lsum : 0.0f;
  }
  __syncthreads();
  const float *gacc = sgather + 2 * kAttnCluster * G;
  for (int i = tid; i < G * Dh; i += kAttnThreads) {
    const int g = i / Dh;
    float a = 0.0f;
    for (int j = 0; j < nslices; j++) a += gacc[(size_t)j * G * Dh + i] * wts[j * G + g];
    out[((size_t)r * H + qh0) * Dh + i] = __float2half_rn(a * scorr[g]);
  }
  if (tracing && tid == 0) {
    tstamp[5] = globaltimer();
    trace_record(ra.tr.buf, ra.tr.next, ra.tr.cap, tstamp, ra.tr.launch_index, cta_id);
  }
}

// ---- SwiGLU (REDUCE_SWIGLU kernels.ts:1066-1077) ---------------------------

__global__ void swiglu_kernel(const float *gu, int rows, int I, void *out, int out_dtype) {
  pdl_trigger();  // dependents may launch now; they wait for this grid to finish
  pdl_wait();     // inputs come from the previous kernel
  const size_t n = (size_t)rows * I;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / I, c = i - r * I;
    const float g = gu[r * 2 * I + c], u = gu[r * 2 * I + I + c];
    store_out(out, out_dtype, i, g / (1.0f + expf(-g)) * u);
  }
}

// gate|up rows interleaved by 8 per 16-row tile (the SwiGLU-pairs packing):
// out[r][8t + i] = silu(gu[r][16t + i]) * gu[r][16t + 8 + i].
__global__ void swiglu_pairs_kernel(const float *gu, int rows, int I, void *out, int out_dtype) {
  pdl_trigger();
  pdl_wait();
  const size_t n = (size_t)rows * I;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / I, f = i - r * I;
    const size_t col = (f / 8) * 16 + (f % 8);
    const float g = gu[r * 2 * I + col], u = gu[r * 2 * I + col + 8];
    store_out(out, out_dtype, i, g / (1.0f + expf(-g)) * u);
  }
}

// ---- gated short conv (shortConv / convState kernels.ts:1380-1437) --------
// bcx [rows][3D] = B | C | x; y_t = B_t x_t; out_t = C_t * sum_k w[c][k]
// y_{t - (W-1-k)}; y before the batch comes from the fp16 state [W-1][D]
// (oldest first), which then holds the batch's last W-1 values of y.
// Every output is independent, so the grid covers (channel block, row
// block); each thread takes one channel over kConvRows rows, loading all of
// them before use. Only the threads of row block 0 touch the state: they
// read the old state first and write the new one last (recomputing the
// batch's last W-1 values of y from bcx), so no other thread races with
// them, and blocks > 0 only look back into bcx (kConvRows >= W - 1).

constexpr int kMaxConvWidth = 8;
constexpr int kConvRows = 16;

__global__ void short_conv_kernel(const float *bcx, int rows, int cps, int D, int W, const float *w, __half *state,
                                  void *out, int out_dtype, __half *prefixes, int slot0, int slots) {
  pdl_trigger();  // dependents may launch now; they wait for this grid to finish
  pdl_wait();     // inputs come from the previous kernel
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= D) return;
  // this block's sequence (rows consecutive rows each) and its row chunk
  const int seq = blockIdx.y / cps, chunk = blockIdx.y - seq * cps;
  bcx += (size_t)seq * rows * 3 * D;
  state += (size_t)seq * (W - 1) * D;
  out = reinterpret_cast<uint8_t *>(out) + (size_t)seq * rows * D * (out_dtype == WG_F32 ? 4 : 2);
  const int r0 = chunk * kConvRows;
  const int nr = min(kConvRows, rows - r0);
  // y over rows r0 - (W-1) .. r0 + nr - 1
  float y[kConvRows + kMaxConvWidth - 1];
  float cg_[kConvRows];
#pragma unroll
  for (int i = 0; i < kConvRows + kMaxConvWidth - 1; i++) {
    const int t = r0 - (W - 1) + i;
    if (i >= nr + W - 1) break;
    if (t >= 0) {
      const float *row = bcx + (size_t)t * 3 * D;
      y[i] = row[c] * row[2 * D + c];
    } else {
      y[i] = __half2float(state[(size_t)(W - 1 + t) * D + c]);  // only row block 0 gets here
    }
  }
#pragma unroll
  for (int i = 0; i < kConvRows; i++)
    if (i < nr) cg_[i] = bcx[(size_t)(r0 + i) * 3 * D + D + c];
  float wk[kMaxConvWidth];
#pragma unroll
  for (int k = 0; k < kMaxConvWidth; k++) wk[k] = k < W ? w[(size_t)c * W + k] : 0.0f;
#pragma unroll
  for (int i = 0; i < kConvRows; i++) {
    if (i >= nr) break;
    float a = 0.0f;
#pragma unroll
    for (int k = 0; k < kMaxConvWidth; k++)
      if (k < W) a += wk[k] * y[i + k];
    store_out(out, out_dtype, (size_t)(r0 + i) * D + c, cg_[i] * a);
  }
  if (prefixes && chunk == 0 && W > 1) {
    // the state after each prefix of p = 1 .. rows rows (convPrefixes,
    // src/gpu/kernels.ts:1504): row i is y at t = p - (W-1) + i, the old
    // state for t < 0; into slot slot0 + p - 1 of this sequence (written
    // before the state itself is replaced)
    __half *pf = prefixes + (size_t)seq * slots * (W - 1) * D;
    for (int pp = 1; pp <= rows && slot0 + pp - 1 < slots; pp++) {
      for (int i = 0; i < W - 1; i++) {
        const int t = pp - (W - 1) + i;
        float v;
        if (t < 0) {
          v = __half2float(state[(size_t)(W - 1 + t) * D + c]);
        } else {
          const float *row = bcx + (size_t)t * 3 * D;
          v = row[c] * row[2 * D + c];
        }
        pf[((size_t)(slot0 + pp - 1) * (W - 1) + i) * D + c] = __float2half_rn(v);
      }
    }
  }
  if (chunk == 0 && W > 1) {
    // new state: y at rows rows-(W-1) .. rows-1 (old state for negative rows)
    float ns[kMaxConvWidth];
#pragma unroll
    for (int i = 0; i < kMaxConvWidth - 1; i++) {
      if (i >= W - 1) break;
      const int t = rows - (W - 1) + i;
      if (t < 0) {
        ns[i] = __half2float(state[(size_t)(W - 1 + t) * D + c]);
      } else {
        const float *row = bcx + (size_t)t * 3 * D;
        ns[i] = row[c] * row[2 * D + c];
      }
    }
#pragma unroll
    for (int i = 0; i < kMaxConvWidth - 1; i++)
      if (i < W - 1) state[(size_t)i * D + c] = __float2half_rn(ns[i]);
  }
}

// ---- fp16 output head + argmax (head engine.ts:8557, pick :8352) -----------
// logits[r][v] = x[r] . W[v]; warp per vocab row, 16-byte loads issued
// eight at a time, x staged in shared memory as fp32. With `amax`, each warp also
// keeps its best (logit, index) per row, each CTA publishes its best, and
// the last CTA to finish (a counter it resets) reduces them: the greedy
// token without a second launch.

constexpr int kHeadMaxRows = 8;
constexpr int kHeadCtasPerSm = 3;
constexpr int kHeadThreads = 256;
constexpr int kHeadUnroll = 8;  // 16-byte loads in flight per lane (a 4 KB row per warp)

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  // larger logit first, then the lower index (-0 counts as +0)
  unsigned u = __float_as_uint(v == 0.0f ? 0.0f : v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned)(0xffffffffu - (unsigned)idx);
}

// Head input: x fp16 [rows][D] as given, or (with `nrm`) the final norm of
// the residual stream, rmsnorm(a + b) * weight rounded to fp16 as the
// separate norm pass would store it.
struct HeadNorm {
  const float *a, *b, *w;
  float eps;
};

template <bool NORM, int kHeadMaxRows>  // kHeadMaxRows: 1 (decode) or 8
__global__ void __launch_bounds__(kHeadThreads, kHeadCtasPerSm)
    head_kernel(const __half *x, HeadNorm nrm, int rows, int row_stride, int D, const __half *W, int V,
                int vocab_offset, float *logits, int32_t *amax, unsigned long long *keys, unsigned long long *part,
                unsigned *count) {
  pdl_trigger();  // dependents may launch now; they wait for this grid to finish
  pdl_wait();     // inputs come from the previous kernel
  extern __shared__ float xs[];  // [rows][D]
  __shared__ unsigned long long s_key[kHeadThreads / 32][8];
  __shared__ bool s_last;
  if (NORM) {
    __shared__ float red[32];
    for (int r = 0; r < rows; r++) {
      float ss = 0.0f;
      const size_t src = (size_t)r * row_stride * D;
      for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float v = nrm.a[src + i];
        if (nrm.b) v += nrm.b[src + i];
        xs[r * D + i] = v;
        ss += v * v;
      }
      const float inv = rsqrtf(block_sum(ss, red) / (float)D + nrm.eps);
      for (int i = threadIdx.x; i < D; i += blockDim.x)
        xs[r * D + i] = __half2float(__float2half_rn(clamp_half(xs[r * D + i] * inv * nrm.w[i])));
    }
  } else {
    for (int i = threadIdx.x; i < rows * D; i += blockDim.x) {
      const int r = i / D;
      xs[i] = __half2float(x[(size_t)r * row_stride * D + (i - r * D)]);
    }
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  const int nvec = D / 8;
  float bv[kHeadMaxRows];
  int bi[kHeadMaxRows];
#pragma unroll
  for (int r = 0; r < kHeadMaxRows; r++) {
    bv[r] = -INFINITY;
    bi[r] = 0x7fffffff;
  }
  for (int v = blockIdx.x * warps + warp; v < V; v += gridDim.x * warps) {
    const uint4 *wr = reinterpret_cast<const uint4 *>(W + (size_t)v * D);
    float acc[kHeadMaxRows];
#pragma unroll
    for (int r = 0; r < kHeadMaxRows; r++) acc[r] = 0.0f;
    constexpr int U = kHeadMaxRows > 1 ? kHeadUnroll / 2 : kHeadUnroll;  // registers for 8 rows
    for (int c0 = lane; c0 < nvec; c0 += 32 * U) {
      uint4 u[U];
#pragma unroll
      for (int j = 0; j < U; j++)
        if (c0 + 32 * j < nvec) u[j] = __ldcs(wr + c0 + 32 * j);  // read once: stream past L2
#pragma unroll
      for (int j = 0; j < U; j++) {
        const int c = c0 + 32 * j;
        if (c >= nvec) break;
        const __half2 *hp = reinterpret_cast<const __half2 *>(&u[j]);
        float wf[8];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float2 f = __half22float2(hp[i]);
          wf[2 * i] = f.x;
          wf[2 * i + 1] = f.y;
        }
#pragma unroll
        for (int r = 0; r < kHeadMaxRows; r++) {
          if (r >= rows) break;
          const float4 *xr = reinterpret_cast<const float4 *>(xs + r * D + c * 8);
          const float4 x0 = xr[0], x1 = xr[1];
          acc[r] += wf[0] * x0.x + wf[1] * x0.y + wf[2] * x0.z + wf[3] * x0.w + wf[4] * x1.x + wf[5] * x1.y +
                    wf[6] * x1.z + wf[7] * x1.w;
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kHeadMaxRows; r++) {
      if (r >= rows) break;
      const float sres = warp_sum(acc[r]);
      if (lane == 0) logits[(size_t)r * V + v] = sres;
      if (sres > bv[r]) {  // v grows along a warp's walk: ties keep the lower index
        bv[r] = sres;
        bi[r] = v;
      }
    }
  }
  if (!amax && !keys) return;
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < kHeadMaxRows; r++)
      if (r < rows) s_key[warp][r] = argmax_key(bv[r], vocab_offset + bi[r]);
  }
  __syncthreads();
  if (threadIdx.x < rows) {
    unsigned long long k = 0;
    for (int w = 0; w < warps; w++) k = max(k, s_key[w][threadIdx.x]);
    part[(size_t)blockIdx.x * rows + threadIdx.x] = k;
    __threadfence();
  }
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(count, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // The last CTA: every thread takes a share of the CTAs' keys, per row.
  for (int r = 0; r < rows; r++) {
    unsigned long long k = 0;
    for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) k = max(k, __ldcg(part + (size_t)b * rows + r));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) k = max(k, __shfl_xor_sync(0xffffffffu, k, o));
    if (lane == 0) s_key[warp][0] = k;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long kk = 0;
      for (int w = 0; w < warps; w++) kk = max(kk, s_key[w][0]);
      if (amax) amax[r] = (int32_t)(0xffffffffu - (unsigned)(kk & 0xffffffffu));
      if (keys) keys[r] = kk ^ 0x8000000000000000ull;  // signed-orderable: an int64 MAX picks it
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) *count = 0;  // ready for the next launch (stream order)
}

// The head on tensor cores (D % 128 == 0): W streams through a ring of
// shared-memory stages filled by TMA (one thread issues 2-D tiled copies of
// 128 vocabulary rows x 64 dims, 16 KB, 128-byte swizzled), so the bytes in
// flight cost no registers and the first stages are requested before the
// wait for the previous kernel (W depends on none). 16 compute warps in two
// groups of 8 take alternate stages of a 128-row block (group g the stages
// s = g mod 2), warp w of a group 16 of its rows, reading A fragments with
// ldmatrix from the swizzled stage and x (fp16, 8 rows, zero past `rows`)
// from shared memory; mma.m16n8k16 with fp32 sums. At the end of a block the
// second group's sums meet the first's in shared memory and the first
// writes the logits and keeps each token's best (row, value); then the
// greedy pick as in head_kernel. A CTA per SM, blocks strided over the CTAs.

constexpr int kHtWarps = 16;                    // compute warps; warp 16 issues the copies
constexpr int kHtThreads = (kHtWarps + 1) * 32;
constexpr int kHtStages = 8;
constexpr int kHtRows = 128;                    // vocabulary rows of a block
constexpr int kHtStageBytes = kHtRows * 128;    // 128 rows x 64 fp16 dims

struct HeadSmem {
  size_t ring, x, red, bar, total;
  __host__ __device__ explicit HeadSmem(int D) {
    ring = 0;  // 1024-aligned (128-byte swizzle atoms)
    x = ring + (size_t)kHtStages * kHtStageBytes;
    red = x + (size_t)8 * (D + 8) * 2;
    bar = red + (size_t)2 * 8 * 32 * 4 * 4;
    total = bar + (size_t)2 * kHtStages * 8;
  }
};

__device__ __forceinline__ void mma_f16_16816(float c[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t r[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

template <bool NORM>
__global__ void __launch_bounds__(kHtThreads, 1)
    head_tma_kernel(const __grid_constant__ CUtensorMap tm_w, const __half *x, HeadNorm nrm, int rows,
                    int row_stride, int D, int V, int vocab_offset, float *logits, int32_t *amax,
                    unsigned long long *keys, unsigned long long *part, unsigned *count, unsigned *flags) {
  pdl_trigger();  // dependents may launch now; they wait for this grid to finish
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const HeadSmem L(D);
  uint8_t *ring = smem + L.ring;
  __half *xh = reinterpret_cast<__half *>(smem + L.x);  // [8][D + 8]
  float *sred = reinterpret_cast<float *>(smem + L.red);  // [2 block parities][8 warps][32 lanes][4]
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bar);
  uint64_t *empty = full + kHtStages;
  __shared__ unsigned long long s_key[kHtWarps + 1][8];
  __shared__ bool s_last;
  __shared__ float red[32];
  __shared__ int aborted;
  __shared__ int issued;
  const int xstride = D + 8;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int KS = D / 64;  // stages a block (even: D % 128 == 0)
  const int nblocks = (V + kHtRows - 1) / kHtRows;
  const int my_blocks = (int)blockIdx.x < nblocks ? (nblocks - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total = my_blocks * KS;  // stages this CTA consumes

  if (threadIdx.x == 0) {
    aborted = 0;
    issued = 0;
    for (int i = 0; i < kHtStages; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kHtWarps / 2);  // the 8 warps of the stage's group
    }
    fence_mbar_init();
  }
  __syncthreads();
  const bool producer = warp == kHtWarps && lane == 0;
  auto issue = [&](int q) {
    const int slot = q % kHtStages, bi = q / KS, s = q - bi * KS;
    const int row0 = ((int)blockIdx.x + bi * (int)gridDim.x) * kHtRows;
    mbar_expect_tx(&full[slot], kHtStageBytes);
    tma_load_2d(ring + (size_t)slot * kHtStageBytes, &tm_w, s * 64, row0, &full[slot]);
  };
  // the first stages: W depends on no earlier kernel
  int q_next = 0;
  if (producer) {
    prefetch_tensormap(&tm_w);
    for (; q_next < min(kHtStages, total); q_next++) issue(q_next);
  }

  pdl_wait();  // x / the residual come from the previous kernel; logits may still be read by it
  for (int r = 0; r < 8; r++) {
    if (r >= rows) {
      for (int i = threadIdx.x; i < D; i += blockDim.x) xh[r * xstride + i] = __float2half_rn(0.0f);
      continue;
    }
    const size_t src = (size_t)r * row_stride * D;
    if (NORM) {
      float ss = 0.0f;
      for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float v = nrm.a[src + i];
        if (nrm.b) v += nrm.b[src + i];
        ss += v * v;
      }
      const float inv = rsqrtf(block_sum(ss, red) / (float)D + nrm.eps);
      for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float v = nrm.a[src + i];
        if (nrm.b) v += nrm.b[src + i];
        xh[r * xstride + i] = __float2half_rn(clamp_half(v * inv * nrm.w[i]));
      }
    } else {
      for (int i = threadIdx.x; i < D; i += blockDim.x) xh[r * xstride + i] = x[src + i];
    }
  }
  __syncthreads();

  float bv[2] = {-INFINITY, -INFINITY};
  int bi_[2] = {0x7fffffff, 0x7fffffff};
  if (warp == kHtWarps) {
    // the rest of the stages, each once the group that read its slot is done
    if (producer) {
      for (; q_next < total; q_next++) {
        const int slot = q_next % kHtStages;
        if (aborted || !mbar_wait_bounded(&empty[slot], ((q_next / kHtStages) & 1) ^ 1, flags)) {
          aborted = 1;
          break;
        }
        issue(q_next);
      }
      issued = q_next;
    }
  } else {
    const int grp = warp >> 3, wr = warp & 7;
    const int gq = lane >> 2, tq = lane & 3;
    const int arow = 16 * wr + (lane & 15);  // this lane's ldmatrix row of the stage
    const __half *xg = xh + gq * xstride + 2 * tq;
    for (int bi = 0; bi < my_blocks; bi++) {
      float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int s = grp; s < KS; s += 2) {
        const int q = bi * KS + s, slot = q % kHtStages;
        if (!aborted && !mbar_wait_bounded(&full[slot], (q / kHtStages) & 1, flags)) aborted = 1;
        const uint8_t *st = ring + (size_t)slot * kHtStageBytes + arow * 128;
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
          const int chunk = 2 * kk + (lane >> 4);
          uint32_t a[4];
          ldsm_x4(a, st + ((chunk ^ (arow & 7)) << 4));
          const int k0 = s * 64 + kk * 16;
          const uint32_t b0 = *reinterpret_cast<const uint32_t *>(xg + k0);
          const uint32_t b1 = *reinterpret_cast<const uint32_t *>(xg + k0 + 8);
          mma_f16_16816(c, a[0], a[1], a[2], a[3], b0, b1);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
      }
      // the two groups' sums of this block meet; group 0 writes them
      float *rb = sred + ((size_t)((bi & 1) * 8 + wr) * 32 + lane) * 4;
      if (grp == 1) {
#pragma unroll
        for (int e = 0; e < 4; e++) rb[e] = c[e];
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kHtWarps * 32) : "memory");
      if (grp == 0) {
        const int v0 = ((int)blockIdx.x + bi * (int)gridDim.x) * kHtRows + 16 * wr;
        // c0, c1: row v0 + gq, tokens 2tq, 2tq + 1; c2, c3: row v0 + gq + 8
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const int v = v0 + gq + 8 * h;
          if (v >= V) continue;
#pragma unroll
          for (int q2 = 0; q2 < 2; q2++) {
            const int tok = 2 * tq + q2;
            if (tok >= rows) continue;
            const float val = c[2 * h + q2] + rb[2 * h + q2];
            logits[(size_t)tok * V + v] = val;
            if (val > bv[q2]) {  // v grows along a lane's walk: ties keep the lower index
              bv[q2] = val;
              bi_[q2] = v;
            }
          }
        }
      }
    }
  }
  // No copy may still be writing this CTA's shared memory when it exits
  // (only possible after a timed-out wait): the producer waits for the last
  // copy issued into each slot.
  if (producer && aborted)
    for (int q = issued > kHtStages ? issued - kHtStages : 0; q < issued; q++)
      mbar_wait_bounded(&full[q % kHtStages], (q / kHtStages) & 1, flags);

  if (!amax && !keys) return;
  // best per token: lanes with the same tq (gq = 0..7) hold tokens 2tq, 2tq + 1
  unsigned long long k0 = argmax_key(bv[0], vocab_offset + bi_[0]);
  unsigned long long k1 = argmax_key(bv[1], vocab_offset + bi_[1]);
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    k0 = max(k0, __shfl_xor_sync(0xffffffffu, k0, o));
    k1 = max(k1, __shfl_xor_sync(0xffffffffu, k1, o));
  }
  if ((lane >> 2) == 0) {
    s_key[warp][2 * (lane & 3)] = k0;
    s_key[warp][2 * (lane & 3) + 1] = k1;
  }
  __syncthreads();
  if (threadIdx.x < rows) {
    unsigned long long k = 0;
    for (int w = 0; w <= kHtWarps; w++) k = max(k, s_key[w][threadIdx.x]);
    part[(size_t)blockIdx.x * rows + threadIdx.x] = k;
    __threadfence();
  }
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(count, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int r = 0; r < rows; r++) {
    unsigned long long k = 0;
    for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) k = max(k, __ldcg(part + (size_t)b * rows + r));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) k = max(k, __shfl_xor_sync(0xffffffffu, k, o));
    if (lane == 0) s_key[warp][0] = k;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long kk = 0;
      for (int w = 0; w <= kHtWarps; w++) kk = max(kk, s_key[w][0]);
      if (amax) amax[r] = (int32_t)(0xffffffffu - (unsigned)(kk & 0xffffffffu));
      if (keys) keys[r] = kk ^ 0x8000000000000000ull;  // signed-orderable: an int64 MAX picks it
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) *count = 0;  // ready for the next launch (stream order)
}

// Per row: the index of the largest logit, the lowest index on ties.
__global__ void argmax_kernel(const float *logits, int V, int32_t *out) {
  pdl_trigger();  // dependents may launch now; they wait for this grid to finish
  pdl_wait();     // inputs come from the previous kernel
  __shared__ float sv[32];
  __shared__ int si[32];
  const int r = blockIdx.x;
  const float *lr = logits + (size_t)r * V;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float x = lr[v];
    if (x > best || (x == best && v < bi)) {
      best = x;
      bi = v;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sv[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x >> 5); i++)
      if (sv[i] > best || (sv[i] == best && si[i] < bi)) {
        best = sv[i];
        bi = si[i];
      }
    out[r] = bi == 0x7fffffff ? 0 : bi;
  }
}

// Token ids from packed (logit, index) keys (after a max-reduction of the
// keys across vocabulary shards).
__global__ void pick_keys_kernel(const unsigned long long *keys, int rows, int32_t *ids) {
  pdl_trigger();
  pdl_wait();
  for (int i = threadIdx.x; i < rows; i += blockDim.x)
    ids[i] = (int32_t)(0xffffffffu - (unsigned)((unsigned long long)keys[i] & 0xffffffffu));
}

// Greedy speculative decoding, acceptance (one thread per sequence): the
// draft proposed d_1..d_k (drafts[b][j] = d_{j+1}); the target's picks at the
// k + 1 verified rows are g_0..g_k (picks[j][b] = g_j, its token for the
// position after row j). Accept the longest prefix with d_{j+1} == g_j, emit
// it and g_n (the target's own token after it), and rewind both models'
// positions to just past what was kept: the target's verify forward advanced
// its position by k + 1; rows past the kept prefix stay in the caches but lie
// beyond the positions, so the next rows overwrite them.
__global__ void spec_accept_kernel(const int32_t *drafts, const int32_t *picks, int batch, int k, int32_t *pos_t,
                                   int32_t *pos_d, int32_t *next_t, int32_t *next_d, int32_t *out, int out_cap,
                                   int32_t *out_len, int32_t *accepted) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  int n = 0;
  while (n < k && drafts[b * k + n] == picks[n * batch + b]) n++;
  const int32_t last = picks[n * batch + b];
  int len = out_len[b];
  for (int i = 0; i < n && len < out_cap; i++) out[(size_t)b * out_cap + len++] = drafts[b * k + i];
  if (len < out_cap) out[(size_t)b * out_cap + len++] = last;
  out_len[b] = len;
  accepted[b] += n;
  const int32_t p = pos_t[b] - (k + 1) + n + 1;
  pos_t[b] = p;
  pos_d[b] = p;
  next_t[b] = last;
  next_d[b] = last;
}

__global__ void add_i32_kernel(int32_t *p, int n, int delta) {
  pdl_trigger();  // dependents may launch now; they wait for this grid to finish
  pdl_wait();     // inputs come from the previous kernel
  for (int i = threadIdx.x; i < n; i += blockDim.x) p[i] += delta;
}

// Launch with programmatic dependent launch when `pdl`: the kernel may start
// while the previous one in the stream finishes (every kernel here waits
// for it with griddepcontrol.wait before reading anything).
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                     Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  if (pdl) {
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace

cudaError_t launch_embed(const int32_t *ids, int rows, const void *table, int V, int D, float *out, cudaStream_t s,
                         bool pdl) {
  return launch_k(embed_kernel, dim3(rows), dim3(256), 0, s, pdl, ids, rows, reinterpret_cast<const __half *>(table),
                  V, D, out);
}

cudaError_t launch_rmsnorm(float *x, const float *add, const float *w, float eps, int rows, int D, void *out,
                           int out_dtype, cudaStream_t s, bool pdl) {
  const int threads = D >= 1024 ? 1024 : ((D + 31) / 32) * 32;
  return launch_k(rmsnorm_kernel, dim3(rows), dim3(threads), 0, s, pdl, x, add, w, eps, D, out, out_dtype);
}

cudaError_t launch_rope_kv(const float *qkv, int rows, int batch, int H, int Hkv, int Dh, const int *pos0,
                           float theta, const float *q_norm, const float *k_norm, float eps, void *q_out,
                           void *k_cache, void *v_cache, int cache_len, unsigned *flags, cudaStream_t s, bool pdl) {
  return launch_k(rope_kv_kernel, dim3(rows, H + Hkv), dim3(Dh / 2), 0, s, pdl, qkv, rows / batch, H, Hkv, Dh, pos0,
                  theta, q_norm,
                  k_norm, eps, reinterpret_cast<__half *>(q_out), reinterpret_cast<__half *>(k_cache),
                  reinterpret_cast<__half *>(v_cache), cache_len, flags);
}

template <int DPL, bool ROPE>
cudaError_t launch_attention_t(const void *q, int rows, int rps, int H, int Hkv, const void *k_cache,
                               const void *v_cache, int cache_len, const int *pos0, void *out, int num_sms,
                               cudaStream_t s, bool pdl, const RopeArgs &ra) {
  // Work split of each (row, KV head) pair, within about one wave of CTAs:
  // first its keys over a cluster of CL CTAs, until a slice of the cache is
  // at most kAttnSliceKeys positions (the split that divides each CTA's K / V
  // bytes; slices merged through distributed shared memory), then its G
  // query heads over HS CTAs with the CTAs left (each owns whole softmax
  // rows: nothing more to merge, the K / V tile is read again from L2).
  const int G = H / Hkv;
  const long long pairs = (long long)rows * Hkv;
  auto per_sm = [](size_t smem) { return smem <= 100 * 1024 ? 2 : 1; };
  const long long wave = (long long)num_sms * per_sm(AttnSmem(32 * DPL, G).total);
  int CL = 1;
  while (CL < kAttnCluster && (long long)CL * kAttnSliceKeys < cache_len && pairs * CL * 2 <= wave) CL *= 2;
  int HS = 1;
  for (int hs = G; hs > 1; hs--)
    if (G % hs == 0 && pairs * CL * hs <= (long long)num_sms * per_sm(AttnSmem(32 * DPL, G / hs).total)) {
      HS = hs;
      break;
    }
  const AttnSmem lay(32 * DPL, G / HS);
  const size_t smem = lay.total;
  auto kern = attention_kernel<DPL, ROPE>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)CL, (unsigned)(Hkv * HS), (unsigned)rows);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
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
  return cudaLaunchKernelEx(&cfg, kern, reinterpret_cast<const __half *>(q), rps, H, Hkv,
                            reinterpret_cast<__half *>(const_cast<void *>(k_cache)),
                            reinterpret_cast<__half *>(const_cast<void *>(v_cache)), cache_len, pos0,
                            reinterpret_cast<__half *>(out), ra);
}

cudaError_t launch_attention(const void *q, int rows, int batch, int H, int Hkv, int Dh, const void *k_cache,
                             const void *v_cache, int cache_len, const int *pos0, void *out, int num_sms,
                             cudaStream_t s, bool pdl, const TraceSink &tr) {
  if (H % Hkv || H / Hkv > kAttnMaxGroup) return cudaErrorInvalidValue;
  const int rps = rows / batch;
  static const bool no_flash = getenv("WG_NO_FLASH_PREFILL") != nullptr;  // the CUDA-core kernel (comparison)
  if (flash_prefill_supported(rps, Dh) && !no_flash)
    return launch_flash_prefill(q, rps, batch, H, Hkv, Dh, k_cache, v_cache, cache_len, pos0, out, s, pdl);
  RopeArgs ra{};
  ra.tr = tr;
  switch (Dh) {
    case 32:
      return launch_attention_t<1, false>(q, rows, rps, H, Hkv, k_cache, v_cache, cache_len, pos0, out, num_sms, s,
                                          pdl, ra);
    case 64:
      return launch_attention_t<2, false>(q, rows, rps, H, Hkv, k_cache, v_cache, cache_len, pos0, out, num_sms, s,
                                          pdl, ra);
    case 128:
      return launch_attention_t<4, false>(q, rows, rps, H, Hkv, k_cache, v_cache, cache_len, pos0, out, num_sms, s,
                                          pdl, ra);
    case 256:
      return launch_attention_t<8, false>(q, rows, rps, H, Hkv, k_cache, v_cache, cache_len, pos0, out, num_sms, s,
                                          pdl, ra);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_rope_attention(const float *qkv, int batch, int H, int Hkv, int Dh, const int *pos0, float theta,
                                  const float *q_norm, const float *k_norm, float eps, void *k_cache, void *v_cache,
                                  int cache_len, void *out, unsigned *flags, int num_sms, cudaStream_t s, bool pdl,
                                  const TraceSink &tr) {
  if (H % Hkv || H / Hkv > kAttnMaxGroup) return cudaErrorInvalidValue;
  const RopeArgs ra{qkv, theta, q_norm, k_norm, eps, flags, tr};
  switch (Dh) {
    case 64:
      return launch_attention_t<2, true>(nullptr, batch, 1, H, Hkv, k_cache, v_cache, cache_len, pos0, out, num_sms,
                                         s, pdl, ra);
    case 128:
      return launch_attention_t<4, true>(nullptr, batch, 1, H, Hkv, k_cache, v_cache, cache_len, pos0, out, num_sms,
                                         s, pdl, ra);
    case 256:
      return launch_attention_t<8, true>(nullptr, batch, 1, H, Hkv, k_cache, v_cache, cache_len, pos0, out, num_sms,
                                         s, pdl, ra);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_swiglu(const float *gu, int rows, int I, void *out, int out_dtype, cudaStream_t s, bool pdl) {
  const size_t n = (size_t)rows * I;
  const size_t blocks = (n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096;
  return launch_k(swiglu_kernel, dim3((unsigned)(blocks ? blocks : 1)), dim3(256), 0, s, pdl, gu, rows, I, out,
                  out_dtype);
}

cudaError_t launch_swiglu_pairs(const float *gu, int rows, int I, void *out, int out_dtype, cudaStream_t s,
                                bool pdl) {
  const size_t n = (size_t)rows * I;
  const size_t blocks = (n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096;
  return launch_k(swiglu_pairs_kernel, dim3((unsigned)(blocks ? blocks : 1)), dim3(256), 0, s, pdl, gu, rows, I, out,
                  out_dtype);
}

cudaError_t launch_short_conv(const float *bcx, int rows, int batch, int D, int W, const float *w, void *state,
                              void *out, int out_dtype, void *prefixes, int slot0, int slots, cudaStream_t s,
                              bool pdl) {
  if (W < 1 || W > kMaxConvWidth) return cudaErrorInvalidValue;
  const int rps = rows / batch, cps = (rps + kConvRows - 1) / kConvRows;
  const dim3 grid((D + 127) / 128, batch * cps);
  return launch_k(short_conv_kernel, grid, dim3(128), 0, s, pdl, bcx, rps, cps, D, W, w,
                  reinterpret_cast<__half *>(state), out, out_dtype, reinterpret_cast<__half *>(prefixes), slot0,
                  slots);
}

// The rollback of speculative accept (accept, src/engine.ts:8063-8085): per
// sequence, kept = pos_after - pos_before tokens of the last draft batch were
// kept; unless that is all `slots` of them, the state becomes the saved
// state after the kept prefix.
__global__ void conv_restore_kernel(const __half *prefixes, int slots, int D, int W, const int32_t *pos_before,
                                    const int32_t *pos_after, __half *state) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.y;
  const int kept = pos_after[b] - pos_before[b];
  if (kept < 1 || kept >= slots) return;
  const size_t n = (size_t)(W - 1) * D;
  const __half *src = prefixes + ((size_t)b * slots + kept - 1) * n;
  __half *dst = state + (size_t)b * n;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

cudaError_t launch_conv_restore(const void *prefixes, int slots, int batch, int D, int W, const int32_t *pos_before,
                                const int32_t *pos_after, void *state, cudaStream_t s, bool pdl) {
  if (W < 2 || W > kMaxConvWidth || slots < 1) return cudaErrorInvalidValue;
  const int n = (W - 1) * D;
  const dim3 grid((n + 255) / 256 < 64 ? (n + 255) / 256 : 64, batch);
  return launch_k(conv_restore_kernel, grid, dim3(256), 0, s, pdl, reinterpret_cast<const __half *>(prefixes), slots,
                  D, W, pos_before, pos_after, reinterpret_cast<__half *>(state));
}

cudaError_t launch_head(const void *x, const float *na, const float *nb, const float *nw, float eps, int rows,
                        int row_stride, int D, const void *W, int V, int vocab_offset, float *logits, int32_t *amax,
                        unsigned long long *keys, unsigned long long *part, size_t part_bytes, unsigned *count,
                        unsigned *flags, int num_sms, cudaStream_t s, bool pdl) {
  if (rows > kHeadMaxRows || D % 8) return cudaErrorInvalidValue;
  const bool norm = na != nullptr;
  const HeadNorm hn{na, nb, nw, eps};
  const size_t smem_tma = HeadSmem(D).total + 1024;  // + slack for the 1024-byte alignment
  if (D % 128 == 0 && smem_tma <= 227 * 1024 && encode_fn() && (reinterpret_cast<uintptr_t>(W) & 15) == 0) {
    CUtensorMap tm;
    cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)V};
    cuuint64_t strides[1] = {(cuuint64_t)D * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)kHtRows};
    cuuint32_t elem[2] = {1, 1};
    if (encode_fn()(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(W), dims, strides, box, elem,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
    auto kern = norm ? head_tma_kernel<true> : head_tma_kernel<false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_tma);
    if (e != cudaSuccess) return e;
    int grid = num_sms;
    const int max_grid = (int)(part_bytes / (sizeof(unsigned long long) * (rows ? rows : 1)));
    if (grid > max_grid) grid = max_grid;
    return launch_k(kern, dim3(grid), dim3(kHtThreads), smem_tma, s, pdl, tm, reinterpret_cast<const __half *>(x),
                    hn, rows, row_stride, D, V, vocab_offset, logits, amax, keys, part, count, flags);
  }
  const size_t smem = (size_t)rows * D * sizeof(float);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  auto kern = norm ? (rows == 1 ? head_kernel<true, 1> : head_kernel<true, kHeadMaxRows>)
                   : (rows == 1 ? head_kernel<false, 1> : head_kernel<false, kHeadMaxRows>);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  int grid = num_sms * kHeadCtasPerSm;
  const int max_grid = (int)(part_bytes / (sizeof(unsigned long long) * (rows ? rows : 1)));
  if (grid > max_grid) grid = max_grid;
  return launch_k(kern, dim3(grid), dim3(kHeadThreads), smem, s, pdl, reinterpret_cast<const __half *>(x), hn, rows,
                  row_stride, D, reinterpret_cast<const __half *>(W), V, vocab_offset, logits, amax, keys, part,
                  count);
}

cudaError_t launch_argmax(const float *logits, int rows, int V, int32_t *out, cudaStream_t s, bool pdl) {
  return launch_k(argmax_kernel, dim3(rows), dim3(1024), 0, s, pdl, logits, V, out);
}

cudaError_t launch_pick_keys(const unsigned long long *keys, int rows, int32_t *ids, cudaStream_t s, bool pdl) {
  return launch_k(pick_keys_kernel, dim3(1), dim3(rows < 1024 ? ((rows + 31) / 32) * 32 : 1024), 0, s, pdl, keys,
                  rows, ids);
}

cudaError_t launch_spec_accept(const int32_t *drafts, const int32_t *picks, int batch, int k, int32_t *pos_t,
                               int32_t *pos_d, int32_t *next_t, int32_t *next_d, int32_t *out, int out_cap,
                               int32_t *out_len, int32_t *accepted, cudaStream_t s, bool pdl) {
  return launch_k(spec_accept_kernel, dim3((batch + 127) / 128), dim3(128), 0, s, pdl, drafts, picks, batch, k, pos_t,
                  pos_d, next_t, next_d, out, out_cap, out_len, accepted);
}

cudaError_t launch_add_i32(int32_t *p, int n, int delta, cudaStream_t s, bool pdl) {
  return launch_k(add_i32_kernel, dim3(1), dim3(n < 1024 ? ((n + 31) / 32) * 32 : 1024), 0, s, pdl, p, n, delta);
}

}  // namespace wg
