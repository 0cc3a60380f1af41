// The kernels around the Q4 matmuls in a decoder layer: embedding, fused residual add + RMS norm, qk-norm + RoPE + KV-cache append,
// causal GQA attention over fp16 caches, SwiGLU, LFM2's gated short
// convolution with an fp16 rolling state, the fp16 output head and argmax.
//
// Activation layout: row-major [rows][features]; the residual stream is fp32
// (the reference keeps it in f32 textures), matmul inputs fp16. Positions
// come from a device counter so that a decode step can be replayed from a
// CUDA graph without re-recording.
#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "decoder_kernels.cuh"
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

__global__ void rope_kv_kernel(const float *qkv, int H, int Hkv, int Dh, const int *pos0, float theta,
                               const float *q_norm, const float *k_norm, float eps, __half *q_out,
                               __half *k_cache, __half *v_cache, int cache_len, unsigned *flags) {
  __shared__ float red[32];
  const int r = blockIdx.x, h = blockIdx.y;  // h < H: query head; else kv head h - H
  const int half = Dh / 2, j = threadIdx.x;
  const int pos = *pos0 + r;
  const size_t row = (size_t)r * (H + 2 * Hkv) * Dh;
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
// Split-K ("flash decoding") over a thread-block cluster: the cluster of
// kAttnCluster CTAs serves one (query row, KV head) pair and every query
// head of its group; CTA c takes the c-th slice of the row's keys 0..pos.
// Per slice, 64-key tiles of K and V are staged in shared memory (16-byte
// loads, K rows padded by 16 bytes so that a warp's row-strided reads hit
// distinct banks), scores for all G = H / Hkv heads are formed from shared
// memory, and an online softmax keeps (max, sum, acc) per head. The slices
// are merged through distributed shared memory: CTA c finishes outputs c,
// c + C, ... of the group's G * Dh. No global scratch, so one launch per
// step and nothing to allocate.

constexpr int kAttnCluster = 8;
constexpr int kAttnThreads = 128;
constexpr int kAttnTile = 64;
constexpr int kAttnMaxGroup = 16;

struct AttnSmem {
  int Dh, G;
  size_t q, k, v, p, corr, m, l, acc, total;  // byte offsets
  __host__ __device__ AttnSmem(int Dh_, int G_) : Dh(Dh_), G(G_) {
    size_t o = 0;
    q = o;
    o += (size_t)G * Dh * 4;
    k = o;
    o += (size_t)kAttnTile * (Dh + 8) * 2;
    v = o;
    o += (size_t)kAttnTile * Dh * 2;
    p = o;
    o += (size_t)G * kAttnTile * 4;
    corr = o;
    o += (size_t)G * 4;
    m = o;
    o += (size_t)G * 4;
    l = o;
    o += (size_t)G * 4;
    acc = o;
    o += (size_t)G * Dh * 4;
    total = o;
  }
};

__device__ __forceinline__ float dot8(uint4 k, const float *q) {
  const __half2 *h = reinterpret_cast<const __half2 *>(&k);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float2 f = __half22float2(h[i]);
    s += f.x * q[2 * i] + f.y * q[2 * i + 1];
  }
  return s;
}

__global__ void __cluster_dims__(kAttnCluster, 1, 1) __launch_bounds__(kAttnThreads)
    attention_kernel(const __half *q, int H, int Hkv, int Dh, const __half *k_cache, const __half *v_cache,
                     int cache_len, const int *pos0, __half *out) {
  extern __shared__ __align__(16) unsigned char smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int G = H / Hkv;
  const AttnSmem lay(Dh, G);
  float *sq = reinterpret_cast<float *>(smem + lay.q);
  __half *sk = reinterpret_cast<__half *>(smem + lay.k);
  __half *sv = reinterpret_cast<__half *>(smem + lay.v);
  float *sp = reinterpret_cast<float *>(smem + lay.p);
  float *scorr = reinterpret_cast<float *>(smem + lay.corr);
  float *sm = reinterpret_cast<float *>(smem + lay.m);
  float *sl = reinterpret_cast<float *>(smem + lay.l);
  float *sacc = reinterpret_cast<float *>(smem + lay.acc);

  const int c = (int)cluster.block_rank();
  const int hk = blockIdx.y, r = blockIdx.z;
  const int tid = threadIdx.x;
  const int L = max(0, min(*pos0 + r + 1, cache_len));
  const int per = (L + kAttnCluster - 1) / kAttnCluster;
  const int t0 = min(L, c * per), t1 = min(L, t0 + per);

  // queries of the group (already scaled by 1/sqrt(Dh))
  const __half *qg = q + ((size_t)r * H + (size_t)hk * G) * Dh;
  for (int i = tid; i < G * Dh; i += kAttnThreads) sq[i] = __half2float(qg[i]);
  for (int g = tid; g < G; g += kAttnThreads) {
    sm[g] = -INFINITY;
    sl[g] = 0.0f;
  }
  for (int i = tid; i < G * Dh; i += kAttnThreads) sacc[i] = 0.0f;

  const __half *kb = k_cache + (size_t)hk * cache_len * Dh;
  const __half *vb = v_cache + (size_t)hk * cache_len * Dh;
  const int vecs = Dh / 8;  // 16-byte vectors per key row
  const int kstride = Dh + 8;
  for (int tt = t0; tt < t1; tt += kAttnTile) {
    const int nt = min(kAttnTile, t1 - tt);
    __syncthreads();  // previous tile fully consumed
    for (int i = tid; i < nt * vecs; i += kAttnThreads) {
      const int t = i / vecs, e = i - t * vecs;
      const uint4 kv = __ldg(reinterpret_cast<const uint4 *>(kb + (size_t)(tt + t) * Dh) + e);
      const uint4 vv = __ldg(reinterpret_cast<const uint4 *>(vb + (size_t)(tt + t) * Dh) + e);
      *reinterpret_cast<uint4 *>(sk + t * kstride + e * 8) = kv;
      *reinterpret_cast<uint4 *>(sv + t * Dh + e * 8) = vv;
    }
    __syncthreads();
    // scores: entry i = g * 64 + t
    for (int i = tid; i < G * kAttnTile; i += kAttnThreads) {
      const int g = i / kAttnTile, t = i - g * kAttnTile;
      float s = -INFINITY;
      if (t < nt) {
        s = 0.0f;
        const uint4 *kr = reinterpret_cast<const uint4 *>(sk + t * kstride);
        const float *qr = sq + g * Dh;
        for (int e = 0; e < vecs; e++) s += dot8(kr[e], qr + e * 8);
      }
      sp[i] = s;
    }
    __syncthreads();
    // per head: new max, rescale factor, probabilities (one warp per head)
    for (int g = tid >> 5; g < G; g += kAttnThreads / 32) {
      const int lane = tid & 31;
      float mx = fmaxf(sp[g * kAttnTile + lane], sp[g * kAttnTile + lane + 32]);
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mold = sm[g], mnew = fmaxf(mold, mx);
      const float p0 = expf(sp[g * kAttnTile + lane] - mnew), p1 = expf(sp[g * kAttnTile + lane + 32] - mnew);
      sp[g * kAttnTile + lane] = p0;
      sp[g * kAttnTile + lane + 32] = p1;
      const float ps = warp_sum(p0 + p1);
      __syncwarp();
      if (lane == 0) {
        const float corr = mold == -INFINITY ? 0.0f : expf(mold - mnew);
        sl[g] = sl[g] * corr + ps;
        sm[g] = mnew;
        scorr[g] = corr;
      }
    }
    __syncthreads();
    // acc[g][d] = acc * corr + sum_t p[g][t] v[t][d]; thread owns entries tid, tid + 128, ...
    for (int i = tid; i < G * Dh; i += kAttnThreads) {
      const int g = i / Dh, d = i - g * Dh;
      const float *pg = sp + g * kAttnTile;
      float a = 0.0f;
      for (int t = 0; t < nt; t++) a += pg[t] * __half2float(sv[t * Dh + d]);
      sacc[i] = sacc[i] * scorr[g] + a;
    }
  }
  cluster.sync();
  // merge the slices: this CTA finishes outputs c, c + C, ... (in units of
  // 128-entry chunks, so each thread finishes whole entries)
  for (int i = c * kAttnThreads + tid; i < G * Dh; i += kAttnCluster * kAttnThreads) {
    const int g = i / Dh;
    float M = -INFINITY;
    for (int j = 0; j < kAttnCluster; j++) {
      const float *rm = cluster.map_shared_rank(sm, j);
      M = fmaxf(M, rm[g]);
    }
    float lsum = 0.0f, a = 0.0f;
    if (M != -INFINITY) {
      for (int j = 0; j < kAttnCluster; j++) {
        const float mj = cluster.map_shared_rank(sm, j)[g];
        if (mj == -INFINITY) continue;
        const float w = expf(mj - M);
        lsum += cluster.map_shared_rank(sl, j)[g] * w;
        a += cluster.map_shared_rank(sacc, j)[i] * w;
      }
    }
    out[((size_t)r * H + (size_t)hk * G) * Dh + i] = __float2half_rn(lsum > 0.0f ? a / lsum : 0.0f);
  }
  cluster.sync();  // keep this CTA's shared memory alive until every peer has read it
}

// ---- SwiGLU (REDUCE_SWIGLU kernels.ts:1066-1077) ---------------------------

__global__ void swiglu_kernel(const float *gu, int rows, int I, void *out, int out_dtype) {
  const size_t n = (size_t)rows * I;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / I, c = i - r * I;
    const float g = gu[r * 2 * I + c], u = gu[r * 2 * I + I + c];
    store_out(out, out_dtype, i, g / (1.0f + expf(-g)) * u);
  }
}

// ---- gated short conv (shortConv / convState kernels.ts:1380-1437) --------
// bcx [rows][3D] = B | C | x; y_t = B_t x_t; out_t = C_t * sum_k w[c][k]
// y_{t - (W-1-k)}; y before the batch from the fp16 state [W-1][D] (oldest
// first), which then holds the batch's last W-1 values of y.

constexpr int kMaxConvWidth = 8;

__global__ void short_conv_kernel(const float *bcx, int rows, int D, int W, const float *w, __half *state,
                                  void *out, int out_dtype) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= D) return;
  float hist[kMaxConvWidth];  // hist[i]: y_{t - (W-1) + i} for the taps before t
  for (int i = 0; i < W - 1; i++) hist[i] = __half2float(state[(size_t)i * D + c]);
  float wk[kMaxConvWidth];
  for (int k = 0; k < W; k++) wk[k] = w[(size_t)c * W + k];
  for (int t = 0; t < rows; t++) {
    const float *row = bcx + (size_t)t * 3 * D;
    const float y = row[c] * row[2 * D + c];
    float a = wk[W - 1] * y;
    for (int k = 0; k < W - 1; k++) a += wk[k] * hist[k];
    store_out(out, out_dtype, (size_t)t * D + c, row[D + c] * a);
    for (int k = 0; k < W - 2; k++) hist[k] = hist[k + 1];
    if (W > 1) hist[W - 2] = y;
  }
  for (int i = 0; i < W - 1; i++) state[(size_t)i * D + c] = __float2half_rn(hist[i]);
}

// ---- fp16 output head + argmax (head engine.ts:8557, pick :8352) -----------
// logits[r][v] = x[r] . W[v]; warp per vocab row, 16-byte loads, x staged
// in shared memory as fp32.

constexpr int kHeadMaxRows = 8;

__global__ void head_kernel(const __half *x, int rows, int D, const __half *W, int V, float *logits) {
  extern __shared__ float xs[];  // [rows][D]
  for (int i = threadIdx.x; i < rows * D; i += blockDim.x) xs[i] = __half2float(x[i]);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int v = blockIdx.x * warps + (threadIdx.x >> 5); v < V; v += gridDim.x * warps) {
    const uint4 *wr = reinterpret_cast<const uint4 *>(W + (size_t)v * D);
    float acc[kHeadMaxRows];
#pragma unroll
    for (int r = 0; r < kHeadMaxRows; r++) acc[r] = 0.0f;
    for (int c = lane; c < D / 8; c += 32) {
      const uint4 u = __ldg(wr + c);
      const __half2 *hp = reinterpret_cast<const __half2 *>(&u);
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
        const float *xr = xs + r * D + c * 8;
#pragma unroll
        for (int i = 0; i < 8; i++) acc[r] += wf[i] * xr[i];
      }
    }
#pragma unroll
    for (int r = 0; r < kHeadMaxRows; r++) {
      if (r >= rows) break;
      const float s = warp_sum(acc[r]);
      if (lane == 0) logits[(size_t)r * V + v] = s;
    }
  }
}

// Per row: the index of the largest logit, the lowest index on ties.
__global__ void argmax_kernel(const float *logits, int V, int32_t *out) {
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

__global__ void add_i32_kernel(int32_t *p, int delta) { *p += delta; }

}  // namespace

cudaError_t launch_embed(const int32_t *ids, int rows, const void *table, int V, int D, float *out,
                         cudaStream_t s) {
  embed_kernel<<<rows, 256, 0, s>>>(ids, rows, reinterpret_cast<const __half *>(table), V, D, out);
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm(float *x, const float *add, const float *w, float eps, int rows, int D, void *out,
                           int out_dtype, cudaStream_t s) {
  rmsnorm_kernel<<<rows, D >= 1024 ? 1024 : ((D + 31) / 32) * 32, 0, s>>>(x, add, w, eps, D, out, out_dtype);
  return cudaGetLastError();
}

cudaError_t launch_rope_kv(const float *qkv, int rows, int H, int Hkv, int Dh, const int *pos0, float theta,
                           const float *q_norm, const float *k_norm, float eps, void *q_out, void *k_cache,
                           void *v_cache, int cache_len, unsigned *flags, cudaStream_t s) {
  rope_kv_kernel<<<dim3(rows, H + Hkv), Dh / 2, 0, s>>>(qkv, H, Hkv, Dh, pos0, theta, q_norm, k_norm, eps,
                                                       reinterpret_cast<__half *>(q_out),
                                                       reinterpret_cast<__half *>(k_cache),
                                                       reinterpret_cast<__half *>(v_cache), cache_len, flags);
  return cudaGetLastError();
}

cudaError_t launch_attention(const void *q, int rows, int H, int Hkv, int Dh, const void *k_cache,
                             const void *v_cache, int cache_len, const int *pos0, void *out, cudaStream_t s) {
  if (H % Hkv || H / Hkv > kAttnMaxGroup || Dh % 8 || Dh > 256) return cudaErrorInvalidValue;
  const AttnSmem lay(Dh, H / Hkv);
  const size_t smem = lay.total;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  attention_kernel<<<dim3(kAttnCluster, Hkv, rows), kAttnThreads, smem, s>>>(
      reinterpret_cast<const __half *>(q), H, Hkv, Dh, reinterpret_cast<const __half *>(k_cache),
      reinterpret_cast<const __half *>(v_cache), cache_len, pos0, reinterpret_cast<__half *>(out));
  return cudaGetLastError();
}

cudaError_t launch_swiglu(const float *gu, int rows, int I, void *out, int out_dtype, cudaStream_t s) {
  const size_t n = (size_t)rows * I;
  const size_t blocks = (n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096;
  swiglu_kernel<<<(unsigned)(blocks ? blocks : 1), 256, 0, s>>>(gu, rows, I, out, out_dtype);
  return cudaGetLastError();
}

cudaError_t launch_short_conv(const float *bcx, int rows, int D, int W, const float *w, void *state, void *out,
                              int out_dtype, cudaStream_t s) {
  if (W < 1 || W > kMaxConvWidth) return cudaErrorInvalidValue;
  short_conv_kernel<<<(D + 127) / 128, 128, 0, s>>>(bcx, rows, D, W, w, reinterpret_cast<__half *>(state), out,
                                                    out_dtype);
  return cudaGetLastError();
}

cudaError_t launch_head(const void *x, int rows, int D, const void *W, int V, float *logits, int num_sms,
                        cudaStream_t s) {
  if (rows > kHeadMaxRows || D % 8) return cudaErrorInvalidValue;
  const size_t smem = (size_t)rows * D * sizeof(float);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  head_kernel<<<num_sms * 4, 256, smem, s>>>(reinterpret_cast<const __half *>(x), rows, D,
                                            reinterpret_cast<const __half *>(W), V, logits);
  return cudaGetLastError();
}

cudaError_t launch_argmax(const float *logits, int rows, int V, int32_t *out, cudaStream_t s) {
  argmax_kernel<<<rows, 1024, 0, s>>>(logits, V, out);
  return cudaGetLastError();
}

cudaError_t launch_add_i32(int32_t *p, int delta, cudaStream_t s) {
  add_i32_kernel<<<1, 1, 0, s>>>(p, delta);
  return cudaGetLastError();
}

}  // namespace wg
